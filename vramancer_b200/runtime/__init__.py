"""Host-side native runtime (C++17, module vramancer_b200._runtime; sources beside this
file): HMAC-SHA256, XOR parity, file spill / restore, framed TCP tensor transport, KV
page allocator, basic tokenizer.  This module adds the tensor-aware Python surface.

Reference parity: rust_core/src/lib.rs (PyO3 runtime: hmac sign/verify/batch
:983-1008, TCP tensor send/recv :857-980, file dump/load :1012-1052, XOR parity
:1057-1108, basic tokenizer :1501-1558), csrc/swarm_core.cpp, csrc/file_offload.cpp.
"""
from __future__ import annotations

import importlib
import json
from typing import Dict, List, Optional, Sequence, Tuple

import torch

_mod = None


def native():
    """The compiled runtime module; raises ImportError with the build command when absent."""
    global _mod
    if _mod is None:
        try:
            _mod = importlib.import_module("vramancer_b200._runtime")
        except ImportError as e:  # pragma: no cover - exercised only without a build
            raise ImportError("vramancer_b200._runtime is not built: run `python setup.py build_ext --inplace`") from e
    return _mod


# ---------------------------------------------------------------- crypto
def sha256(data) -> bytes:
    return native().sha256(_buf(data))


def sign(key: bytes, data) -> bytes:
    """HMAC-SHA256 tag (32 bytes) of `data` (bytes-like or a CPU tensor)."""
    return native().hmac_sha256(bytes(key), _buf(data))


def verify(key: bytes, data, tag: bytes) -> bool:
    """Constant-time check of an HMAC-SHA256 tag."""
    return native().hmac_verify(bytes(key), _buf(data), bytes(tag))


def sign_batch(key: bytes, items: Sequence, threads: int = 4) -> List[bytes]:
    return native().hmac_batch(bytes(key), [_buf(x) for x in items], threads)


# ---------------------------------------------------------------- parity
def xor_parity(shards: Sequence, threads: int = 4) -> bytearray:
    """Parity shard (XOR) of equal-length shards."""
    return native().xor_parity([_buf(s) for s in shards], threads)


def xor_repair(shards: Sequence[Optional[object]], parity) -> bytearray:
    """Rebuilds the single missing shard (the one given as None) from the others and
    the parity."""
    missing = [i for i, s in enumerate(shards) if s is None]
    if len(missing) != 1:
        raise ValueError(f"xor_repair: exactly one shard must be missing, got {len(missing)}")
    return native().xor_parity([_buf(s) for s in shards if s is not None] + [_buf(parity)])


# ---------------------------------------------------------------- file spill
def _buf(x):
    if isinstance(x, torch.Tensor):
        if x.is_cuda:
            raise ValueError("host buffer expected (got a CUDA tensor)")
        return x.contiguous().view(torch.uint8).numpy()
    return x


def _host_view(t: torch.Tensor) -> torch.Tensor:
    if t.is_cuda:
        h = torch.empty(t.shape, dtype=t.dtype, pin_memory=True)
        h.copy_(t)
        return h
    return t.contiguous()


def dump_tensor(path: str, t: torch.Tensor, offset: int = 0, sync: bool = False) -> int:
    """Writes the raw bytes of `t` (any device; CUDA through a pinned host copy) to
    `path` at `offset`; returns the byte count."""
    h = _host_view(t)
    return native().file_write(path, h.data_ptr(), h.numel() * h.element_size(), offset, False, sync)


def load_tensor(path: str, out: torch.Tensor, offset: int = 0) -> torch.Tensor:
    """Reads raw bytes from `path` into `out` (any device) and returns it."""
    nbytes = out.numel() * out.element_size()
    if out.is_cuda:
        h = torch.empty(out.shape, dtype=out.dtype, pin_memory=True)
        native().file_read(path, h.data_ptr(), nbytes, offset, False)
        out.copy_(h, non_blocking=False)
        return out
    if not out.is_contiguous():
        raise ValueError("load_tensor: contiguous destination expected")
    native().file_read(path, out.data_ptr(), nbytes, offset, False)
    return out


class AsyncFileIO:
    """Overlapped spill / restore of pinned host buffers on a worker-thread pool.  The
    caller keeps each buffer alive until its ticket has been waited for."""

    def __init__(self, workers: int = 4):
        self._io = native().AsyncIO(workers)
        self._keep: Dict[int, torch.Tensor] = {}

    def write(self, path: str, host: torch.Tensor, offset: int = 0) -> int:
        host = host.contiguous()
        t = self._io.submit_write(path, host.data_ptr(), host.numel() * host.element_size(), offset, False)
        self._keep[t] = host
        return t

    def read(self, path: str, host: torch.Tensor, offset: int = 0) -> int:
        if host.is_cuda or not host.is_contiguous():
            raise ValueError("AsyncFileIO.read: contiguous host tensor expected")
        t = self._io.submit_read(path, host.data_ptr(), host.numel() * host.element_size(), offset, False)
        self._keep[t] = host
        return t

    def wait(self, ticket: int) -> int:
        try:
            return self._io.wait(ticket)
        finally:
            self._keep.pop(ticket, None)

    def done(self, ticket: int) -> bool:
        return self._io.done(ticket)

    @property
    def pending(self) -> int:
        return self._io.pending()


# ---------------------------------------------------------------- transport
_DT = {str(d): d for d in (torch.float32, torch.float16, torch.bfloat16, torch.int64, torch.int32,
                           torch.int16, torch.int8, torch.uint8, torch.bool, torch.float64)}


def send_tensors(conn, tensors: Dict[str, torch.Tensor], meta: Optional[dict] = None, key: bytes = b"",
                 chunk: int = 16 << 20) -> int:
    """Sends named tensors (any device) and a JSON-able `meta` as one frame; every
    chunk carries an HMAC tag when `key` is given.  Returns the payload bytes."""
    hosts, entries, off = [], [], 0
    for name, t in tensors.items():
        h = _host_view(t.detach())
        n = h.numel() * h.element_size()
        off = (off + 15) & ~15          # every tensor 16-byte aligned: views of any dtype on receipt
        entries.append({"name": name, "dtype": str(h.dtype), "shape": list(h.shape), "offset": off, "nbytes": n})
        hosts.append(h)
        off += n
    payload = torch.zeros(off, dtype=torch.uint8, pin_memory=torch.cuda.is_available())
    for h, e in zip(hosts, entries):
        if e["nbytes"]:
            payload[e["offset"]:e["offset"] + e["nbytes"]].copy_(h.reshape(-1).view(torch.uint8))
    header = json.dumps({"tensors": entries, "meta": meta or {}}).encode()
    conn.send_frame(header, payload.data_ptr(), off, bytes(key), chunk)
    return off


def recv_tensors(conn, key: bytes = b"", device: Optional[str] = None) -> Tuple[Dict[str, torch.Tensor], dict]:
    """Receives one frame sent by send_tensors; raises on a bad signature."""
    header, payload = conn.recv_frame(bytes(key))
    hdr = json.loads(bytes(header).decode())
    raw = torch.frombuffer(payload, dtype=torch.uint8) if len(payload) else torch.empty(0, dtype=torch.uint8)
    out = {}
    for e in hdr["tensors"]:
        seg = raw[e["offset"]:e["offset"] + e["nbytes"]]
        t = seg.view(_DT[e["dtype"]]).reshape(e["shape"]).clone()
        out[e["name"]] = t.to(device) if device else t
    return out, hdr.get("meta", {})


def connect(host: str, port: int, timeout: float = 30.0):
    return native().connect(host, port, timeout)


def listen(host: str = "127.0.0.1", port: int = 0):
    return native().Listener(host, port)


# ---------------------------------------------------------------- pages / tokens
def page_allocator(num_pages: int):
    return native().PageAllocator(num_pages)


def basic_tokenize(texts: Sequence[str], vocab: int, threads: int = 4) -> List[List[int]]:
    return native().basic_tokenize(list(texts), vocab, threads)
