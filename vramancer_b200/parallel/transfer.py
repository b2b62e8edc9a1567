"""GPU-to-GPU tensor transfers: topology probe and per-pair transport choice.

Methods, in order of preference for a (src, dst) GPU pair in this process:
  CUDA_P2P     peer copy (cudaMemcpyPeerAsync through torch) on a dedicated copy
               stream of the source GPU; NVLink / NVSwitch on B200 boxes
  P2P_KERNEL   KV pages: the page-copy kernel (csrc/migrate.cu) pushes whole pages
               over NVLink with 16-byte stores (transfer_kv_cache)
  CPU_STAGED   no peer access: chunks through two pinned host buffers, the H2D of one
               chunk overlapping the D2H of the next
  NCCL         another process (rank) of the default group: dist.send / dist.recv
  CPU_ONLY     host tensors
Every transfer is timed with CUDA events on its stream; results keep bytes, time and
GB/s, and `stats()` aggregates them per method.

Reference parity: core/transfer_manager.py:69-1000 (TransportMethod, TransferResult,
GPUTopology, TransferManager.send_activation / send_tensor / transfer_kv_cache /
prefetch_layers / sync_activations / get_topology / stats / benchmark / shutdown) and
the accelerate hook patch core/inference_pipeline.py:445-495 (patch_accelerate).
"""
from __future__ import annotations

import enum
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional, Sequence, Tuple

import torch


class TransportMethod(enum.Enum):
    CUDA_P2P = "cuda_p2p"
    P2P_KERNEL = "p2p_kernel"
    CPU_STAGED = "cpu_staged"
    NCCL = "nccl"
    CPU_ONLY = "cpu_only"
    SAME_DEVICE = "same_device"


@dataclass
class TransferResult:
    method: TransportMethod
    source_gpu: int
    target_gpu: int
    bytes_transferred: int
    duration_s: float
    bandwidth_gbs: float = 0.0

    def __post_init__(self):
        if self.duration_s > 0 and self.bytes_transferred > 0:
            self.bandwidth_gbs = self.bytes_transferred / self.duration_s / 1e9


@dataclass
class GPUTopology:
    num_gpus: int = 0
    p2p_matrix: Dict[Tuple[int, int], bool] = field(default_factory=dict)
    nvlink_links: Dict[int, int] = field(default_factory=dict)     # active NVLinks per GPU (NVML)
    device_names: Dict[int, str] = field(default_factory=dict)
    device_caps: Dict[int, Tuple[int, int]] = field(default_factory=dict)

    def p2p(self, a: int, b: int) -> bool:
        return a == b or self.p2p_matrix.get((a, b), False)


def _nvlink_counts(nvml=None) -> Dict[int, int]:
    """Active NVLink links per GPU through NVML ({} when NVML is unavailable)."""
    try:
        if nvml is None:
            import pynvml as nvml  # nvidia_ml_py
        nvml.nvmlInit()
        out = {}
        for i in range(nvml.nvmlDeviceGetCount()):
            h = nvml.nvmlDeviceGetHandleByIndex(i)
            n = 0
            for link in range(18):
                try:
                    if nvml.nvmlDeviceGetNvLinkState(h, link):
                        n += 1
                except Exception:  # noqa: BLE001 - link index beyond this GPU's links
                    break
            out[i] = n
        return out
    except Exception:  # noqa: BLE001
        return {}


def detect_topology(nvml=None) -> GPUTopology:
    topo = GPUTopology()
    if not torch.cuda.is_available():
        return topo
    n = torch.cuda.device_count()
    topo.num_gpus = n
    for i in range(n):
        p = torch.cuda.get_device_properties(i)
        topo.device_names[i] = p.name
        topo.device_caps[i] = (p.major, p.minor)
        for j in range(n):
            if i != j:
                topo.p2p_matrix[(i, j)] = bool(torch.cuda.can_device_access_peer(i, j))
    topo.nvlink_links = _nvlink_counts(nvml)
    return topo


class TransferManager:
    def __init__(self, topology: Optional[GPUTopology] = None, staging_chunk_mb: int = 32, enable_peer: bool = True):
        self.topology = topology if topology is not None else detect_topology()
        self.chunk = staging_chunk_mb << 20
        self._streams: Dict[int, torch.cuda.Stream] = {}
        self._staging: Dict[int, List[torch.Tensor]] = {}
        self._lock = threading.Lock()
        self.results: List[TransferResult] = []
        self._peer_enabled = set()
        self.enable_peer = enable_peer

    # ---------------------------------------------------------------- helpers
    def get_topology(self) -> GPUTopology:
        return self.topology

    def method_for(self, src: int, dst: int) -> TransportMethod:
        if src < 0 or dst < 0:
            return TransportMethod.CPU_ONLY
        if src == dst:
            return TransportMethod.SAME_DEVICE
        if self.topology.p2p(src, dst):
            return TransportMethod.CUDA_P2P
        return TransportMethod.CPU_STAGED

    def _stream(self, dev: int) -> torch.cuda.Stream:
        with self._lock:
            s = self._streams.get(dev)
            if s is None:
                s = torch.cuda.Stream(device=dev)
                self._streams[dev] = s
            return s

    def _ensure_peer(self, src: int, dst: int) -> None:
        if not self.enable_peer or (src, dst) in self._peer_enabled:
            return
        from .. import ops
        try:
            ops.native().enable_peer_access(src, dst)
            ops.native().enable_peer_access(dst, src)
        except Exception:  # noqa: BLE001 - torch's copy still works without explicit access
            pass
        self._peer_enabled.add((src, dst))

    def _record(self, r: TransferResult) -> TransferResult:
        from ..utils import observability as obs
        m = getattr(r.method, "value", str(r.method))
        obs.METRICS.transfer_bytes.labels(m).inc(r.bytes_transferred)
        obs.METRICS.transfer_seconds.labels(m).observe(r.duration_s)
        with self._lock:
            self.results.append(r)
            if len(self.results) > 10000:
                del self.results[:5000]
        return r

    # ---------------------------------------------------------------- transfers
    def send_activation(self, source_gpu: int, target_gpu: int, tensor: torch.Tensor,
                        stream: Optional[torch.cuda.Stream] = None, out: Optional[torch.Tensor] = None,
                        sync: bool = True) -> Tuple[torch.Tensor, TransferResult]:
        """Copies `tensor` (on source_gpu) to target_gpu; returns (copy, result).
        With sync=False the copy is only ordered on the copy stream (the caller's
        current stream of target_gpu waits for it)."""
        nbytes = tensor.numel() * tensor.element_size()
        method = self.method_for(source_gpu, target_gpu)
        if method == TransportMethod.CPU_ONLY:
            t0 = time.perf_counter()
            dst = tensor.to("cpu" if target_gpu < 0 else f"cuda:{target_gpu}")
            return dst, self._record(TransferResult(method, source_gpu, target_gpu, nbytes, time.perf_counter() - t0))
        if method == TransportMethod.SAME_DEVICE:
            return tensor, self._record(TransferResult(method, source_gpu, target_gpu, 0, 0.0))
        dst_dev = torch.device("cuda", target_gpu)
        if out is None:
            out = torch.empty(tensor.shape, dtype=tensor.dtype, device=dst_dev)
        s = stream or self._stream(source_gpu)
        with torch.cuda.device(source_gpu):
            s.wait_stream(torch.cuda.current_stream(source_gpu))
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(s)
            with torch.cuda.stream(s):
                if method == TransportMethod.CUDA_P2P:
                    self._ensure_peer(source_gpu, target_gpu)
                    out.copy_(tensor, non_blocking=True)
                else:
                    self._staged(tensor, out, s)
            e1.record(s)
        torch.cuda.current_stream(target_gpu).wait_event(e1)
        tensor.record_stream(s)
        out.record_stream(s)
        dur = 0.0
        if sync:
            e1.synchronize()
            dur = e0.elapsed_time(e1) / 1e3
        return out, self._record(TransferResult(method, source_gpu, target_gpu, nbytes, dur))

    def _staged(self, src: torch.Tensor, dst: torch.Tensor, s: torch.cuda.Stream) -> None:
        """src GPU -> pinned host (two buffers, alternating) -> dst GPU."""
        flat_s = src.contiguous().view(-1).view(torch.uint8)
        flat_d = dst.view(-1).view(torch.uint8)
        n = flat_s.numel()
        bufs = self._staging.get(src.device.index)
        if bufs is None or bufs[0].numel() < min(self.chunk, n):
            bufs = [torch.empty(min(self.chunk, max(n, 1)), dtype=torch.uint8, pin_memory=True) for _ in range(2)]
            self._staging[src.device.index] = bufs
        up = self._stream(dst.device.index)
        done = [torch.cuda.Event(), torch.cuda.Event()]
        for i, off in enumerate(range(0, n, self.chunk)):
            b = bufs[i & 1]
            m = min(self.chunk, n - off)
            if i >= 2:
                s.wait_event(done[i & 1])              # the buffer's previous H2D has finished
            b[:m].copy_(flat_s[off:off + m], non_blocking=True)
            ev = torch.cuda.Event()
            ev.record(s)
            up.wait_event(ev)
            with torch.cuda.stream(up):
                flat_d[off:off + m].copy_(b[:m], non_blocking=True)
            done[i & 1].record(up)
        s.wait_stream(up)

    def send_tensor(self, tensor: torch.Tensor, target_gpu: int, **kw) -> torch.Tensor:
        src = tensor.device.index if tensor.is_cuda else -1
        return self.send_activation(src, target_gpu, tensor, **kw)[0]

    def sync_activations(self, gpus: Optional[Sequence[int]] = None) -> None:
        for d in gpus if gpus is not None else list(self._streams):
            self._stream(d).synchronize()

    def transfer_kv_cache(self, source_gpu: int, target_gpu: int, src_pool: torch.Tensor, dst_pool: torch.Tensor,
                          src_pages: Sequence[int], dst_pages: Sequence[int]) -> TransferResult:
        """Copies whole KV pages between pools on two GPUs with the page-copy kernel."""
        from ..kv.migration import migrate_pages
        nbytes = len(src_pages) * (src_pool.numel() // src_pool.shape[0]) * src_pool.element_size()
        method = TransportMethod.P2P_KERNEL if self.topology.p2p(source_gpu, target_gpu) else TransportMethod.CPU_STAGED
        t0 = time.perf_counter()
        migrate_pages(src_pool, dst_pool, list(src_pages), list(dst_pages),
                      method="kernel" if method == TransportMethod.P2P_KERNEL else "cpu_staged")
        torch.cuda.synchronize(target_gpu)
        return self._record(TransferResult(method, source_gpu, target_gpu, nbytes, time.perf_counter() - t0))

    def prefetch_layers(self, source_gpu: int, target_gpu: int, layer_tensors: Dict[str, torch.Tensor]
                        ) -> Dict[str, Tuple[torch.Tensor, TransferResult]]:
        """Starts copies of every named tensor on the copy stream without waiting;
        the target GPU's current stream is ordered after them."""
        return {k: self.send_activation(source_gpu, target_gpu, v, sync=False) for k, v in layer_tensors.items()}

    def send_nccl(self, tensor: torch.Tensor, dst_rank: int) -> TransferResult:
        import torch.distributed as dist
        t0 = time.perf_counter()
        dist.send(tensor, dst_rank)
        return self._record(TransferResult(TransportMethod.NCCL, dist.get_rank(), dst_rank,
                                           tensor.numel() * tensor.element_size(), time.perf_counter() - t0))

    def recv_nccl(self, tensor: torch.Tensor, src_rank: int) -> TransferResult:
        import torch.distributed as dist
        t0 = time.perf_counter()
        dist.recv(tensor, src_rank)
        return self._record(TransferResult(TransportMethod.NCCL, src_rank, dist.get_rank(),
                                           tensor.numel() * tensor.element_size(), time.perf_counter() - t0))

    # ---------------------------------------------------------------- reporting
    def stats(self) -> Dict[str, Any]:
        per: Dict[str, Dict[str, float]] = {}
        for r in self.results:
            d = per.setdefault(r.method.value, {"count": 0, "bytes": 0, "seconds": 0.0})
            d["count"] += 1
            d["bytes"] += r.bytes_transferred
            d["seconds"] += r.duration_s
        for d in per.values():
            d["avg_gbs"] = d["bytes"] / d["seconds"] / 1e9 if d["seconds"] > 0 else 0.0
        return {"num_gpus": self.topology.num_gpus, "transfers": len(self.results), "by_method": per,
                "p2p_pairs": sum(1 for v in self.topology.p2p_matrix.values() if v),
                "nvlink_links": self.topology.nvlink_links}

    def benchmark(self, sizes_mb: Optional[List[float]] = None, warmup: int = 2, iterations: int = 5,
                  pairs: Optional[Sequence[Tuple[int, int]]] = None) -> List[Dict[str, Any]]:
        """GB/s per (src, dst, size) measured with CUDA events."""
        sizes_mb = sizes_mb or [1, 16, 256]
        n = self.topology.num_gpus
        pairs = pairs or [(i, j) for i in range(n) for j in range(n) if i != j][:8]
        rows = []
        for src, dst in pairs:
            for mb in sizes_mb:
                x = torch.empty(int(mb * (1 << 20)), dtype=torch.uint8, device=f"cuda:{src}")
                out = torch.empty_like(x, device=f"cuda:{dst}")
                for _ in range(warmup):
                    self.send_activation(src, dst, x, out=out)
                rs = [self.send_activation(src, dst, x, out=out)[1] for _ in range(iterations)]
                best = max(r.bandwidth_gbs for r in rs)
                rows.append({"src": src, "dst": dst, "mb": mb, "method": rs[0].method.value,
                             "gbs": round(best, 2)})
        return rows

    def shutdown(self) -> None:
        self.sync_activations()
        self._streams.clear()
        self._staging.clear()


def patch_accelerate(tm: TransferManager, min_bytes: int = 512 * 1024) -> bool:
    """Routes accelerate's cuda->cuda `send_to_device` of tensors >= min_bytes through
    `tm` (when accelerate is installed); returns whether the patch was applied."""
    try:
        import accelerate.utils.operations as ops_mod  # type: ignore
    except Exception:  # noqa: BLE001
        return False
    orig = ops_mod.send_to_device

    def send_to_device(tensor, device, *a, **kw):
        if isinstance(tensor, torch.Tensor) and tensor.is_cuda and \
                tensor.numel() * tensor.element_size() >= min_bytes:
            dev = torch.device(device) if not isinstance(device, int) else torch.device("cuda", device)
            if dev.type == "cuda" and dev.index is not None and dev.index != tensor.device.index:
                return tm.send_tensor(tensor, dev.index)
        return orig(tensor, device, *a, **kw)

    ops_mod.send_to_device = send_to_device
    return True
