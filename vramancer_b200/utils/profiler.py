"""Per-layer profiling and profile-driven placement.

`LayerProfiler.profile_model(llm)` times each decoder layer of a loaded model on its
device (CUDA events around every layer of one prefill-shaped forward; wall clock on
CPU) and counts its parameters; `profile_gpus()` measures GEMM throughput and copy
bandwidth per GPU; `plan(profiles, speeds)` turns them into contiguous layer ranges
(placement.compute_optimal_placement: DP minimising the slowest stage).

Reference parity: core/layer_profiler.py:135-700 (LayerProfile, GPUProfile,
PlacementPlan, LayerProfiler.profile_model / profile_gpus / DP placement).
"""
from __future__ import annotations

import time
from dataclasses import dataclass
from typing import List, Optional, Sequence

import torch


@dataclass
class LayerProfile:
    index: int
    time_ms: float
    params: int
    bytes: int


@dataclass
class GPUProfile:
    index: int
    name: str
    tflops_bf16: float
    copy_gbs: float


@dataclass
class PlacementPlan:
    layer_ranges: List[range]
    stage_ms: List[float]


class LayerProfiler:
    def profile_model(self, llm, tokens: int = 64, reps: int = 3) -> List[LayerProfile]:
        from ..engine.runner import PrefillItem
        model = llm.model
        cuda = model.device.type == "cuda"
        times = {i: [] for i in range(model.first_layer, model.last_layer)}
        orig = model.layer

        def timed(i, *a, **k):
            if cuda:
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                out = orig(i, *a, **k)
                e1.record()
                times[i].append((e0, e1))
            else:
                t0 = time.perf_counter()
                out = orig(i, *a, **k)
                times[i].append((time.perf_counter() - t0) * 1e3)
            return out

        ids = list(range(1, tokens + 1))
        model.layer = timed
        try:
            for r in range(reps):
                rid = f"__profile{r}"
                llm.kv.allocate(rid, len(ids))
                it = PrefillItem(ids, 0, llm.kv.slots_for(rid, 0, len(ids)), llm.kv.block_table(rid), len(ids), True)
                llm.runner.prefill_logits([it])
                llm.kv.free(rid)
            if cuda:
                torch.cuda.synchronize()
        finally:
            del model.layer
        out = []
        for i, ts in times.items():
            vals = [a.elapsed_time(b) for a, b in ts] if cuda else ts
            w = [v for k, v in model.w.items() if k.startswith(f"layers.{i}.") and isinstance(v, torch.Tensor)]
            out.append(LayerProfile(i, min(vals) if vals else 0.0, sum(t.numel() for t in w),
                                    sum(t.numel() * t.element_size() for t in w)))
        return out

    def profile_gpus(self, size: int = 8192, copy_mb: int = 512) -> List[GPUProfile]:
        res = []
        for g in range(torch.cuda.device_count() if torch.cuda.is_available() else 0):
            dev = f"cuda:{g}"
            a = torch.randn(size, size, device=dev, dtype=torch.bfloat16)
            b = torch.randn(size, size, device=dev, dtype=torch.bfloat16)
            x = torch.empty(copy_mb << 20, dtype=torch.uint8, device=dev)
            y = torch.empty_like(x)
            for _ in range(2):
                a @ b
                y.copy_(x)
            e = [torch.cuda.Event(enable_timing=True) for _ in range(4)]
            e[0].record()
            for _ in range(5):
                a @ b
            e[1].record()
            e[2].record()
            for _ in range(5):
                y.copy_(x)
            e[3].record()
            torch.cuda.synchronize(dev)
            tflops = 5 * 2 * size ** 3 / (e[0].elapsed_time(e[1]) / 1e3) / 1e12
            gbs = 5 * 2 * (copy_mb << 20) / (e[2].elapsed_time(e[3]) / 1e3) / 1e9
            res.append(GPUProfile(g, torch.cuda.get_device_name(g), round(tflops, 1), round(gbs, 1)))
        return res

    def plan(self, profiles: Sequence[LayerProfile], speeds: Sequence[float],
             mem_limits: Optional[Sequence[float]] = None) -> PlacementPlan:
        from ..parallel.placement import compute_optimal_placement
        t = [p.time_ms for p in profiles]
        mem = [p.bytes for p in profiles]
        limits = list(mem_limits) if mem_limits else [float(sum(mem)) + 1.0] * len(speeds)
        spans = compute_optimal_placement(t, mem, list(speeds), limits)
        ranges = [range(a, b) for a, b in spans]
        stage = [sum(t[a:b]) / max(s, 1e-9) for (a, b), s in zip(spans, speeds)]
        return PlacementPlan(ranges, stage)
