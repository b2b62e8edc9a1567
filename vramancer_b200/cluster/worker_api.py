"""HTTP side of cross-node pipeline parallelism: the worker routes of the serving API
and the distributed generate entry point.

A node exposes (through `serving/api.py`):
  GET  /api/worker/model_info     the layer range this node holds
  POST /api/worker/load_partial   {"model", "start_layer", "end_layer", "device", "seed",
                                   "tcp_port"}: load layers [start, end) (plus embedding
                                   for start 0, plus the head for the last range); with
                                   tcp_port a signed-frame stage server is started too
  POST /api/worker/forward_layers {"hidden" | "input_ids", "positions"}: run the local
                                   layers over a whole sequence (stateless, a scratch
                                   KV pool per call) and return the hidden states, or
                                   the last row's logits from the last range
  POST /api/distributed/generate  {"model", "prompt_ids", "max_tokens", "split",
                                   "workers": [{"host", "port"}]}: layers [0, split) here,
                                   the rest on stage servers (TCP frames, paged KV kept
                                   on each node), continuous batching on this node
  POST /api/swarm/awaken          {"macs": [...], "broadcast", "port"}: Wake-on-LAN magic
                                   packets for sleeping worker nodes

Tensors cross HTTP as {"dtype", "shape", "data": base64 of the raw little-endian bytes}.
The stateless HTTP forward is the compatibility path; generation runs over the TCP
stage servers, which keep their KV pages between steps.

Reference parity: core/production_api.py:1271-1380 (/api/distributed/generate, worker
routes), core/cross_node.py:660-848 (worker_forward, distributed_generate),
/api/swarm/awaken (wake-on-LAN of worker nodes).
"""
from __future__ import annotations

import base64
import socket
import threading
from typing import Any, Dict, List, Optional, Sequence

import torch

_DTYPES = {"float32": torch.float32, "bfloat16": torch.bfloat16, "float16": torch.float16, "int32": torch.int32,
           "int64": torch.int64}


def encode_tensor(t: torch.Tensor) -> Dict[str, Any]:
    t = t.detach().contiguous().cpu()
    name = str(t.dtype).replace("torch.", "")
    if name not in _DTYPES:
        raise ValueError(f"unsupported dtype {t.dtype}")
    raw = t.view(torch.uint8).numpy().tobytes() if t.numel() else b""
    return {"dtype": name, "shape": list(t.shape), "data": base64.b64encode(raw).decode()}


def decode_tensor(d: Dict[str, Any]) -> torch.Tensor:
    dt = _DTYPES.get(d.get("dtype", ""))
    if dt is None:
        raise ValueError(f"unsupported dtype {d.get('dtype')!r}")
    shape = [int(x) for x in d["shape"]]
    raw = base64.b64decode(d["data"])
    n = 1
    for s in shape:
        n *= s
    esz = torch.empty(0, dtype=dt).element_size()
    if len(raw) != n * esz:
        raise ValueError(f"tensor payload has {len(raw)} bytes, shape {shape} needs {n * esz}")
    if n == 0:
        return torch.empty(shape, dtype=dt)
    return torch.frombuffer(bytearray(raw), dtype=torch.uint8).view(dt).reshape(shape).clone()


class NodeWorker:
    """The layer range this node serves over HTTP (and optionally over TCP frames)."""

    def __init__(self):
        self.lock = threading.Lock()
        self.cfg = None
        self.model = None
        self.model_name = None
        self.start = self.end = 0
        self.device = torch.device("cpu")
        self.dtype = torch.float32
        self.tcp = None          # StageServer

    def model_info(self) -> Dict[str, Any]:
        if self.model is None:
            return {"loaded": False}
        c = self.cfg
        return {"loaded": True, "model": self.model_name, "start_layer": self.start, "end_layer": self.end,
                "num_layers": c.num_layers, "hidden_size": c.hidden_size, "vocab_size": c.vocab_size,
                "has_embed": self.start == 0, "has_head": self.end == c.num_layers, "device": str(self.device),
                "dtype": str(self.dtype).replace("torch.", ""),
                "tcp_port": self.tcp.port if self.tcp is not None else None}

    def load_partial(self, model: str, start: int, end: int, *, device: str = "cpu", dtype: str = "float32",
                     seed: int = 0, tcp_port: Optional[int] = None, tcp_host: str = "127.0.0.1", key: bytes = b"",
                     num_pages: int = 256) -> Dict[str, Any]:
        from ..models.config import get_config
        from ..models.transformer import DecoderModel
        from ..models.weights import random_weights
        cfg = get_config(model)
        end = cfg.num_layers if end is None or end < 0 else int(end)
        start = int(start)
        if not (0 <= start < end <= cfg.num_layers):
            raise ValueError(f"layer range [{start}, {end}) outside [0, {cfg.num_layers})")
        dt = _DTYPES[dtype]
        dev = torch.device(device)
        w = random_weights(cfg, device=dev, dtype=dt, seed=seed, layers=range(start, end), embed=start == 0,
                           head=end == cfg.num_layers)
        m = DecoderModel(cfg, w, device=dev, dtype=dt, first_layer=start, last_layer=end)
        with self.lock:
            if self.tcp is not None:
                self.tcp.close()
                self.tcp = None
            self.cfg, self.model, self.model_name = cfg, m, model
            self.start, self.end, self.device, self.dtype = start, end, dev, dt
            if tcp_port is not None:
                from .stage_server import StageServer
                self.tcp = StageServer(cfg, start, end, host=tcp_host, port=int(tcp_port), num_pages=num_pages,
                                       seed=seed, key=key, device=device, dtype=dt,
                                       kv_cache_dtype="fp32" if dt == torch.float32 else "bf16").start()
        return self.model_info()

    def forward_layers(self, *, hidden: Optional[torch.Tensor] = None, input_ids: Optional[torch.Tensor] = None,
                       positions: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Stateless forward of one whole sequence [T, H] (or ids for the first range)."""
        from ..kv.pool import KVPool, KVPoolSpec
        from ..models.transformer import ForwardBatch
        if self.model is None:
            raise RuntimeError("no layers loaded: POST /api/worker/load_partial first")
        m, cfg, dev = self.model, self.cfg, self.device
        if self.start == 0:
            if input_ids is None:
                raise ValueError("the first layer range takes input_ids")
            T = int(input_ids.numel())
        else:
            if hidden is None or hidden.dim() != 2 or hidden.shape[1] != cfg.hidden_size:
                raise ValueError(f"hidden must be [T, {cfg.hidden_size}]")
            T = int(hidden.shape[0])
        if T <= 0:
            raise ValueError("empty sequence")
        pos = positions if positions is not None else torch.arange(T, dtype=torch.int32)
        pages = (T + 15) // 16
        pool = KVPool(KVPoolSpec(pages, m.num_local_layers, m.kvh, cfg.head_dim, dtype=self.dtype), dev)
        i32 = lambda v: torch.as_tensor(v, dtype=torch.int32).to(dev)   # noqa: E731
        batch = ForwardBatch(input_ids=i32(input_ids.flatten() if input_ids is not None else torch.zeros(T)),
                             positions=i32(pos), slot_mapping=i32(torch.arange(T)),
                             block_tables=i32(torch.arange(pages).view(1, pages)), context_lens=i32([T]),
                             is_decode=False, cu_q=i32([0, T]), max_q_len=T,
                             logits_rows=torch.tensor([T - 1], device=dev))
        with self.lock:
            h = hidden.to(dev, self.dtype) if hidden is not None else None
            return m.forward(batch, pool, hidden=h)

    def close(self) -> None:
        with self.lock:
            if self.tcp is not None:
                self.tcp.close()
                self.tcp = None


def distributed_generate(model: str, prompts: Sequence[Sequence[int]], max_tokens: int, split: int,
                         workers: Sequence[Dict[str, Any]], *, device: str = "cpu", dtype: str = "float32",
                         seed: int = 0, key: bytes = b"", num_pages: int = 256, max_model_len: int = 2048,
                         temperature: float = 0.0) -> List[List[int]]:
    """Layers [0, split) on this node, the following ranges on the workers' stage servers
    (in order), continuous batching here; returns the generated ids of each prompt."""
    from ..engine.engine import LLMEngine, SamplingParams
    from ..engine.runner import ModelRunner
    from ..kv.paged import PagedKVCacheManager
    from ..kv.pool import KVPool, KVPoolSpec
    from ..models.config import get_config
    from ..models.transformer import DecoderModel
    from ..models.weights import random_weights
    from ..parallel.pipeline import LocalPipeline
    from .stage_server import RemoteStage
    cfg = get_config(model)
    dt = _DTYPES[dtype]
    dev = torch.device(device)
    w = random_weights(cfg, device=dev, dtype=dt, seed=seed, layers=range(0, split), embed=True, head=False)
    m0 = DecoderModel(cfg, w, device=dev, dtype=dt, first_layer=0, last_layer=split)
    p0 = KVPool(KVPoolSpec(num_pages, split, m0.kvh, cfg.head_dim, dtype=dt), dev)
    stages = [(m0, p0)]
    remotes = []
    expect = split
    try:
        for wk in workers:
            r = RemoteStage(str(wk.get("host", "127.0.0.1")), int(wk["port"]), device=device, key=key)
            remotes.append(r)
            if r.first_layer != expect:
                raise ValueError(f"worker {wk} serves layers from {r.first_layer}, expected {expect}")
            expect = r.last_layer
            stages.append((r, None))
        if expect != cfg.num_layers:
            raise ValueError(f"the workers stop at layer {expect} of {cfg.num_layers}")
        pipe = LocalPipeline(stages)
        runner = ModelRunner(pipe, None, max_batch=max(1, len(prompts)), max_model_len=max_model_len,
                             use_cuda_graph=False)
        eng = LLMEngine(runner, PagedKVCacheManager(num_pages))
        reqs = eng.generate(prompts, SamplingParams(max_tokens=max_tokens, temperature=temperature))
        return [list(r.output_ids) for r in reqs]
    finally:
        for r in remotes:
            r.close()


def wake_on_lan(macs: Sequence[str], broadcast: str = "255.255.255.255", port: int = 9) -> int:
    """Sends a Wake-on-LAN magic packet (6 x 0xFF, then the MAC 16 times) per address;
    returns how many were sent."""
    sent = 0
    with socket.socket(socket.AF_INET, socket.SOCK_DGRAM) as s:
        s.setsockopt(socket.SOL_SOCKET, socket.SO_BROADCAST, 1)
        for mac in macs:
            hexs = mac.replace(":", "").replace("-", "").replace(".", "")
            if len(hexs) != 12:
                raise ValueError(f"bad MAC address {mac!r}")
            payload = b"\xff" * 6 + bytes.fromhex(hexs) * 16
            s.sendto(payload, (broadcast, int(port)))
            sent += 1
    return sent
