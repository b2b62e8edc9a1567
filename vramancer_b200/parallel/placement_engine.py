"""Block-level placement with pluggable strategies, weighted by link health.

`PlacementEngine.place(block)` picks the device (or memory tier) for one block of
weights / KV ({"size_mb", "layer_type", "priority", ...}); `place_model(cfg, ...)` cuts
a whole model into per-GPU layer ranges with the dynamic program of
`parallel.placement.compute_optimal_placement` over the model's per-layer costs.

Strategies (`register_strategy(name, fn)` adds more):
  "profiled"  measured speed x free memory, so a fast GPU with room wins (default)
  "vram"      the device with the most free memory
  "balanced"  the least-loaded device by blocks placed so far
Every score is multiplied by the device's link health from a `Connectome`: an
exponentially weighted record of each node's measured transfer latency and failures,
so a GPU behind a slow or flaky link (or a remote node) draws fewer blocks.  A block
that fits on no GPU goes to the host tier ("cpu"), one larger than the host budget to
"nvme".

Reference parity: core/orchestrator/placement_engine.py:64-352 (PlacementEngine with
"profiled" / "vram" / "balanced" strategies, register_strategy, place, place_model,
connectome health weighting via core/network/connectome.py).
"""
from __future__ import annotations

import threading
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence

from . import placement


class Connectome:
    """Per-node link health in (0, 1]: 1 for a link at the best latency seen with no
    failures.  `record` folds in one measured transfer (EWMA, factor `alpha`)."""

    def __init__(self, alpha: float = 0.2, fail_penalty: float = 0.5):
        self.alpha, self.fail_penalty = alpha, fail_penalty
        self._lat: Dict[str, float] = {}
        self._rel: Dict[str, float] = {}
        self._lock = threading.Lock()

    def record(self, node: str, latency_ms: float, ok: bool = True) -> None:
        with self._lock:
            if ok:
                prev = self._lat.get(node)
                self._lat[node] = latency_ms if prev is None else (1 - self.alpha) * prev + self.alpha * latency_ms
            r = self._rel.get(node, 1.0)
            self._rel[node] = (1 - self.alpha) * r + self.alpha * (1.0 if ok else 0.0)

    def weight(self, node: str) -> float:
        """Health of a node's link: (best latency / its latency) x reliability, where a
        reliability below 1 is further scaled by `fail_penalty`; unknown nodes get 1."""
        with self._lock:
            lat = self._lat.get(node)
            rel = self._rel.get(node, 1.0)
            best = min(self._lat.values()) if self._lat else None
        w = 1.0 if lat is None or best is None or lat <= 0 else min(1.0, best / lat)
        if rel < 1.0:
            w *= rel * self.fail_penalty + (1 - self.fail_penalty) * rel * rel
        return max(w, 1e-6)

    def snapshot(self) -> Dict[str, Dict[str, float]]:
        with self._lock:
            return {n: {"latency_ms": self._lat.get(n, 0.0), "reliability": self._rel.get(n, 1.0)}
                    for n in set(self._lat) | set(self._rel)}


@dataclass
class DeviceState:
    index: int
    name: str = "gpu"
    total_mb: float = 0.0
    free_mb: float = 0.0
    speed: float = 1.0            # relative throughput (GPU profile TFLOPS)
    placed: int = 0               # blocks placed so far
    node: str = field(default="")

    def __post_init__(self):
        if not self.node:
            self.node = f"gpu_{self.index}"


class PlacementEngine:
    def __init__(self, devices: Optional[Sequence[DeviceState]] = None, monitor=None,
                 connectome: Optional[Connectome] = None, host_budget_mb: float = 48 * 1024):
        self.connectome = connectome or Connectome()
        self.monitor = monitor
        self.host_budget_mb = host_budget_mb
        self.host_used_mb = 0.0
        self.devices: List[DeviceState] = list(devices) if devices is not None else self._detect()
        self._strategies: Dict[str, Callable[[Dict[str, object]], Optional[int]]] = {
            "profiled": self._score_profiled, "vram": self._score_vram, "balanced": self._score_balanced}
        self._lock = threading.Lock()

    # ---------------------------------------------------------------- devices
    def _detect(self) -> List[DeviceState]:
        out = []
        for g in placement.detect_gpus():
            prof = placement.lookup_gpu_profile(g.name)
            out.append(DeviceState(g.index, g.name, g.total_gb * 1024, g.free_gb * 1024, prof.bf16_tflops or 1.0))
        return out

    def refresh(self) -> None:
        """Free memory from the monitor's latest samples (bytes used / total per GPU)."""
        if self.monitor is None:
            return
        for d in self.monitor.poll():
            i = int(d["index"])
            for dev in self.devices:
                if dev.index == i and d.get("mem_total"):
                    dev.total_mb = d["mem_total"] / 2 ** 20
                    dev.free_mb = (d["mem_total"] - d["mem_used"]) / 2 ** 20

    def register_strategy(self, name: str, fn: Callable[[DeviceState, Dict[str, object]], float]) -> None:
        """fn(device, block) -> score (higher wins; <= 0 means "not here")."""
        self._strategies[name] = lambda block, fn=fn: self._argmax(lambda d: fn(d, block), block)

    # ---------------------------------------------------------------- strategies
    def _argmax(self, score: Callable[[DeviceState], float], block: Dict[str, object]) -> Optional[int]:
        need = float(block.get("size_mb", 0.0))
        best, best_s = None, 0.0
        for i, d in enumerate(self.devices):
            if d.free_mb < need:
                continue
            sc = score(d) * self.connectome.weight(d.node)
            if sc > best_s:
                best, best_s = i, sc
        return best

    def _score_profiled(self, block):
        return self._argmax(lambda d: d.speed * max(d.free_mb, 0.0), block)

    def _score_vram(self, block):
        return self._argmax(lambda d: max(d.free_mb, 0.0), block)

    def _score_balanced(self, block):
        return self._argmax(lambda d: 1.0 / (1 + d.placed), block)

    # ---------------------------------------------------------------- API
    def place(self, block: Dict[str, object], strategy: Optional[str] = None) -> Dict[str, object]:
        """{"level": "gpu" | "cpu" | "nvme", "gpu_id": index or -1, "reason": str}; the
        chosen device's free memory is charged with the block."""
        name = strategy or "profiled"
        fn = self._strategies.get(name, self._score_profiled)
        need = float(block.get("size_mb", 0.0))
        with self._lock:
            i = fn(block)
            if i is not None:
                d = self.devices[i]
                d.free_mb -= need
                d.placed += 1
                return {"level": "gpu", "gpu_id": d.index, "reason": f"{name}: best score on {d.node}"}
            if self.host_used_mb + need <= self.host_budget_mb:
                self.host_used_mb += need
                return {"level": "cpu", "gpu_id": -1, "reason": "no GPU has room"}
            return {"level": "nvme", "gpu_id": -1, "reason": "beyond the host budget"}

    def place_model(self, cfg, num_gpus: int = 0, hop_cost_ms: float = 0.0, batch_tokens: int = 1,
                    objective: str = "bottleneck") -> List[tuple]:
        """Per-GPU layer ranges [(start, end)] for a model config: per-layer time and
        memory from `placement.layer_costs`, GPU speed x link health, GPU free memory."""
        devs = self.devices[: num_gpus or len(self.devices)]
        if not devs:
            raise ValueError("no GPUs to place on")
        t, m = placement.layer_costs(cfg, batch_tokens)            # bytes per layer
        speed = [d.speed * self.connectome.weight(d.node) for d in devs]
        mem = [d.free_mb * 2 ** 20 for d in devs]
        return placement.compute_optimal_placement(t, m, speed, mem, hop_cost_ms, objective)
