"""Cross-node pipeline parallelism: a layer range served by another machine.

A worker node runs
    python -m vramancer_b200.cluster.stage_server --model qwen2.5-14b --layers 24:48 \
        --port 18951 --device cuda:0 --key-file secret
which holds layers [24, 48) (plus the head when the range ends at the last layer)
and their paged KV pool.  The master puts a `RemoteStage` in its LocalPipeline; each
forward sends the batch metadata and the residual stream as one signed tensor frame
(C++ runtime, HMAC-SHA256 per chunk) and receives the stage output (hidden states, or
logits from the last stage).  Copy-on-write page copies are forwarded too, so the
remote pool mirrors the master's page tables.

Reference parity: core/cross_node.py and the VTP worker of core/network/llm_transport.py
(master runs local layers and ships hidden states to remote workers over TCP port
18951 or HTTP; a worker loads a partial model).
"""
from __future__ import annotations

import argparse
import threading
from dataclasses import fields
from typing import Dict, Optional, Sequence

import torch

from .. import runtime as rt
from ..kv.pool import KVPool, KVPoolSpec, kv_dtype_from_str
from ..models.config import get_config
from ..models.transformer import DecoderModel, ForwardBatch
from ..models.weights import random_weights

DEFAULT_PORT = 18951
_BATCH_TENSORS = [f.name for f in fields(ForwardBatch) if f.name not in ("is_decode", "max_q_len", "attn_splits")]


def _pack_batch(batch: ForwardBatch) -> Dict[str, torch.Tensor]:
    return {k: getattr(batch, k) for k in _BATCH_TENSORS if getattr(batch, k) is not None}


def _unpack_batch(t: Dict[str, torch.Tensor], meta: dict, device) -> ForwardBatch:
    kw = {k: (t[k].to(device) if k in t else None) for k in _BATCH_TENSORS}
    return ForwardBatch(is_decode=meta["is_decode"], max_q_len=meta["max_q_len"], attn_splits=meta["attn_splits"],
                        **kw)


class StageServer:
    """Serves one pipeline stage (layers [start, end)) over signed TCP frames."""

    def __init__(self, model, start: int, end: int, *, host: str = "127.0.0.1", port: int = DEFAULT_PORT,
                 device: str = "cpu", dtype: torch.dtype = torch.float32, kv_cache_dtype: str = "fp32",
                 num_pages: int = 256, seed: int = 0, key: bytes = b"", weights=None):
        cfg = get_config(model) if isinstance(model, str) else model
        self.cfg = cfg
        self.device = torch.device(device)
        w = weights if weights is not None else random_weights(
            cfg, device=self.device, dtype=dtype, seed=seed, layers=range(start, end), embed=start == 0,
            head=end == cfg.num_layers)
        self.model = DecoderModel(cfg, w, device=self.device, dtype=dtype, first_layer=start, last_layer=end)
        spec = KVPoolSpec(num_pages, end - start, self.model.kvh, cfg.head_dim, dtype=kv_dtype_from_str(kv_cache_dtype))
        self.pool = KVPool(spec, self.device)
        self.key = key
        self.listener = rt.listen(host, port)
        self.requests = 0
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None

    @property
    def port(self) -> int:
        return self.listener.port

    def start(self) -> "StageServer":
        self._thread = threading.Thread(target=self.serve_forever, daemon=True)
        self._thread.start()
        return self

    def serve_forever(self) -> None:
        while not self._stop.is_set():
            conn = self.listener.accept(0.2)
            if conn is None:
                continue
            try:
                self._serve_connection(conn)
            finally:
                conn.close()

    def _serve_connection(self, conn) -> None:
        while not self._stop.is_set():
            try:
                tensors, meta = rt.recv_tensors(conn, key=self.key)
            except RuntimeError:
                return                      # peer closed, or a frame failed its signature
            op = meta.get("op")
            self.requests += 1
            try:
                self._handle(conn, op, tensors, meta)
            except Exception as e:  # noqa: BLE001 - reported to the master, the server keeps serving
                rt.send_tensors(conn, {}, {"ok": False, "error": f"{type(e).__name__}: {e}"}, key=self.key)
            if op == "shutdown":
                return

    def _handle(self, conn, op, tensors, meta) -> None:
        if True:
            if op == "forward":
                batch = _unpack_batch(tensors, meta, self.device)
                hidden = tensors.get("hidden")
                with torch.no_grad():
                    out = self.model.forward(batch, self.pool, hidden=None if hidden is None else hidden.to(self.device))
                rt.send_tensors(conn, {"out": out}, {"ok": True}, key=self.key)
            elif op == "copy_pages":
                for src, dst in meta["pairs"]:
                    self.pool.cache[dst].copy_(self.pool.cache[src])
                rt.send_tensors(conn, {}, {"ok": True}, key=self.key)
            elif op == "ping":
                rt.send_tensors(conn, {}, {"ok": True, "layers": [self.model.first_layer, self.model.last_layer]},
                                key=self.key)
            elif op == "shutdown":
                rt.send_tensors(conn, {}, {"ok": True}, key=self.key)
                self._stop.set()
            else:
                rt.send_tensors(conn, {}, {"ok": False, "error": f"unknown op {op!r}"}, key=self.key)

    def close(self) -> None:
        self._stop.set()
        if self._thread is not None:
            self._thread.join(2)
        self.listener.close()


class RemoteStage:
    """Master-side proxy of a StageServer; behaves like a DecoderModel stage inside
    LocalPipeline (forward / copy_pages / device)."""

    def __init__(self, host: str, port: int = DEFAULT_PORT, *, device: str = "cpu", key: bytes = b"",
                 timeout: float = 60.0):
        self.addr = (host, port)
        self.device = torch.device(device)       # where outputs land on the master
        self.key = key
        self.conn = rt.connect(host, port, timeout)
        self._lock = threading.Lock()
        meta = self._call({}, {"op": "ping"})[1]
        self.first_layer, self.last_layer = meta["layers"]

    def _call(self, tensors, meta):
        with self._lock:
            rt.send_tensors(self.conn, tensors, meta, key=self.key)
            return rt.recv_tensors(self.conn, key=self.key)

    def forward(self, batch: ForwardBatch, pool=None, hidden: Optional[torch.Tensor] = None) -> torch.Tensor:
        t = _pack_batch(batch)
        if hidden is not None:
            t["hidden"] = hidden
        out, meta = self._call(t, {"op": "forward", "is_decode": batch.is_decode, "max_q_len": batch.max_q_len,
                                   "attn_splits": batch.attn_splits})
        if not meta.get("ok", False):
            raise RuntimeError(f"remote stage {self.addr} failed: {meta}")
        return out["out"].to(self.device)

    def copy_pages(self, pairs: Sequence) -> None:
        self._call({}, {"op": "copy_pages", "pairs": [list(p) for p in pairs]})

    def shutdown_server(self) -> None:
        try:
            self._call({}, {"op": "shutdown"})
        finally:
            self.conn.close()

    def close(self) -> None:
        self.conn.close()


def main(argv=None):
    ap = argparse.ArgumentParser(description="serve a pipeline stage (layer range) to a remote master")
    ap.add_argument("--model", required=True)
    ap.add_argument("--layers", required=True, help="start:end")
    ap.add_argument("--host", default="0.0.0.0")
    ap.add_argument("--port", type=int, default=DEFAULT_PORT)
    ap.add_argument("--device", default="cuda:0" if torch.cuda.is_available() else "cpu")
    ap.add_argument("--kv-pages", type=int, default=4096)
    ap.add_argument("--kv-cache-dtype", default=None)
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--key-file", default=None, help="file holding the shared HMAC key")
    a = ap.parse_args(argv)
    start, end = (int(x) for x in a.layers.split(":"))
    cuda = a.device.startswith("cuda")
    key = open(a.key_file, "rb").read().strip() if a.key_file else b""
    srv = StageServer(a.model, start, end, host=a.host, port=a.port, device=a.device,
                      dtype=torch.bfloat16 if cuda else torch.float32,
                      kv_cache_dtype=a.kv_cache_dtype or ("bf16" if cuda else "fp32"), num_pages=a.kv_pages,
                      seed=a.seed, key=key)
    print(f"stage server: layers [{start}, {end}) on {a.device}, port {srv.port}", flush=True)
    srv.serve_forever()


if __name__ == "__main__":
    main()
