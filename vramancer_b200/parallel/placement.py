"""GPU discovery, heterogeneous profiles and layer placement (model splitting).

* `GPU_PROFILES` / `lookup_gpu_profile`: per-model characteristics (HBM, bandwidth,
  dense bf16 TFLOP/s, interconnect).  B200 is in the table (the reference's DB stops
  at H100).
* `detect_gpus`, `probe_p2p`, `detect_vm`: what is present and how GPUs can talk.
* `compute_scores`, `split_layers`: VRAM-, compute- or balanced-proportional layer
  counts (balanced = VRAM * sqrt(normalised compute), as the reference's hetero
  config does).
* `compute_optimal_placement`: contiguous layer ranges chosen by dynamic
  programming from per-layer latency / memory profiles and per-GPU speed, with the
  activation hop between stages charged at the link bandwidth; objective either the
  pipeline bottleneck (max stage time, the throughput-optimal choice) or the sum of
  stage times (the reference's latency objective).
* `split_model_into_blocks` / `assign_blocks_to_gpus`: the reference's public names.
* `auto_configure`: one call that returns tiers, split, lending ratios and a
  `max_memory`-style map.

Reference parity: core/model_splitter.py:71-423, core/hetero_config.py:50-606,
core/layer_profiler.py:612-760.
"""
from __future__ import annotations

import math
import os
import subprocess
from dataclasses import asdict, dataclass, field
from typing import Dict, List, Optional, Sequence, Tuple

import torch


@dataclass(frozen=True)
class GPUProfile:
    name: str
    arch: str
    vram_gb: float
    bw_gbs: float
    bf16_tflops: float
    link: str = "pcie4"
    link_gbs: float = 25.0
    tier: int = 2


GPU_PROFILES: Dict[str, GPUProfile] = {p.name: p for p in [
    GPUProfile("B200", "blackwell-sm100", 180, 7700, 2250, "nvlink5", 900, 0),
    GPUProfile("B100", "blackwell-sm100", 180, 7700, 1750, "nvlink5", 900, 0),
    GPUProfile("GB200", "blackwell-sm100", 186, 8000, 2500, "nvlink5", 900, 0),
    GPUProfile("H200", "hopper-sm90", 141, 4800, 989, "nvlink4", 450, 0),
    GPUProfile("H100", "hopper-sm90", 80, 3350, 989, "nvlink4", 450, 0),
    GPUProfile("A100", "ampere-sm80", 80, 2039, 312, "nvlink3", 300, 1),
    GPUProfile("L40S", "ada-sm89", 48, 864, 362, "pcie4", 25, 1),
    GPUProfile("RTX 5090", "blackwell-sm120", 32, 1792, 209, "pcie5", 50, 1),
    GPUProfile("RTX 5070 Ti", "blackwell-sm120", 16, 896, 88, "pcie5", 50, 2),
    GPUProfile("RTX 4090", "ada-sm89", 24, 1008, 165, "pcie4", 25, 1),
    GPUProfile("RTX 3090", "ampere-sm86", 24, 936, 71, "pcie4", 25, 2),
    GPUProfile("CPU", "cpu", 0, 100, 2, "host", 20, 3),
]}


def lookup_gpu_profile(name: str) -> GPUProfile:
    n = (name or "").upper().replace("NVIDIA", "").replace("GEFORCE", "").strip()
    best = None
    for key, p in GPU_PROFILES.items():
        k = key.upper()
        if k in n and (best is None or len(k) > len(best.name)):
            best = p
    if best is None:
        return GPUProfile(name or "unknown", "unknown", 0, 500, 50, "pcie4", 25, 2)
    return best


@dataclass
class GPUInfo:
    index: int
    name: str
    total_bytes: int
    free_bytes: int
    capability: Tuple[int, int] = (0, 0)
    sms: int = 0
    profile: GPUProfile = field(default_factory=lambda: GPU_PROFILES["CPU"])

    @property
    def total_gb(self) -> float:
        return self.total_bytes / 2 ** 30

    @property
    def free_gb(self) -> float:
        return self.free_bytes / 2 ** 30

    def to_dict(self):
        d = asdict(self)
        d["profile"] = asdict(self.profile)
        return d


def detect_gpus() -> List[GPUInfo]:
    out: List[GPUInfo] = []
    if not torch.cuda.is_available():
        return out
    order = os.environ.get("VRM_GPU_ORDER")
    idx = [int(x) for x in order.split(",")] if order else list(range(torch.cuda.device_count()))
    for i in idx:
        p = torch.cuda.get_device_properties(i)
        try:
            free, total = torch.cuda.mem_get_info(i)
        except Exception:
            free, total = p.total_memory, p.total_memory
        out.append(GPUInfo(i, p.name, total, free, (p.major, p.minor), p.multi_processor_count,
                           lookup_gpu_profile(p.name)))
    return out


def probe_p2p(gpus: Optional[Sequence[int]] = None) -> Dict[str, object]:
    """Peer-access matrix from the runtime (NVLink/NVSwitch systems report all True)."""
    if not torch.cuda.is_available():
        return {"matrix": [], "all_p2p": False, "method": "none"}
    ids = list(gpus) if gpus is not None else list(range(torch.cuda.device_count()))
    m = [[(a == b) or bool(torch.cuda.can_device_access_peer(a, b)) for b in ids] for a in ids]
    return {"matrix": m, "all_p2p": all(all(r) for r in m), "method": "cudaDeviceCanAccessPeer"}


def detect_vm() -> Dict[str, object]:
    info = {"virtualized": False, "hypervisor": None}
    try:
        with open("/proc/cpuinfo") as f:
            if "hypervisor" in f.read():
                info["virtualized"] = True
        vendor = open("/sys/class/dmi/id/sys_vendor").read().strip() if os.path.exists(
            "/sys/class/dmi/id/sys_vendor") else ""
        for h in ("QEMU", "KVM", "VMware", "Microsoft", "Xen", "Proxmox"):
            if h.lower() in vendor.lower():
                info["hypervisor"] = h
                info["virtualized"] = True
    except Exception:
        pass
    return info


# ----------------------------------------------------------------------------- scores / splits
def compute_scores(gpus: Sequence[GPUInfo], strategy: str = "balanced") -> List[float]:
    if not gpus:
        return []
    vram = [g.free_bytes for g in gpus]
    comp = [g.profile.bf16_tflops if g.profile.bf16_tflops > 0 else (g.capability[0] * 10 + g.capability[1]) * g.sms
            for g in gpus]
    cmax = max(comp) or 1.0
    if strategy == "vram":
        return [float(v) for v in vram]
    if strategy == "compute":
        return [float(c) for c in comp]
    return [v * math.sqrt(c / cmax) for v, c in zip(vram, comp)]


def split_layers(num_layers: int, weights: Sequence[float]) -> List[int]:
    """Integer layer counts proportional to weights (largest remainder), each >= 1."""
    n = len(weights)
    if n == 0:
        return []
    if n > num_layers:
        raise ValueError("more devices than layers")
    tot = sum(weights) or 1.0
    raw = [num_layers * w / tot for w in weights]
    counts = [max(1, int(math.floor(r))) for r in raw]
    while sum(counts) > num_layers:
        i = max(range(n), key=lambda j: counts[j] - raw[j])
        counts[i] -= 1
    while sum(counts) < num_layers:
        i = max(range(n), key=lambda j: raw[j] - counts[j])
        counts[i] += 1
    return counts


def ranges_from_counts(counts: Sequence[int]) -> List[Tuple[int, int]]:
    out, s = [], 0
    for c in counts:
        out.append((s, s + c))
        s += c
    return out


def compute_optimal_placement(layer_time: Sequence[float], layer_mem: Sequence[float], gpu_speed: Sequence[float],
                              gpu_mem: Sequence[float], hop_cost: float = 0.0,
                              objective: str = "bottleneck") -> List[Tuple[int, int]]:
    """Contiguous partition of layers over the GPUs in order.

    Stage time on GPU g = sum(layer_time[i]) / gpu_speed[g] (+ hop_cost for the
    activation transfer into the stage when it is not the first).  Memory of a
    stage must fit gpu_mem[g].  objective = "bottleneck" minimises the slowest stage
    (pipeline throughput); "sum" minimises the total (single-request latency).
    Returns [(start, end)] per GPU (empty ranges allowed when a GPU is not needed).
    """
    L, G = len(layer_time), len(gpu_speed)
    pre_t = [0.0]
    pre_m = [0.0]
    for t, m in zip(layer_time, layer_mem):
        pre_t.append(pre_t[-1] + t)
        pre_m.append(pre_m[-1] + m)
    INF = float("inf")
    # dp[g][i]: best objective covering layers [0, i) with GPUs [0, g)
    dp = [[INF] * (L + 1) for _ in range(G + 1)]
    arg = [[-1] * (L + 1) for _ in range(G + 1)]
    dp[0][0] = 0.0
    for g in range(1, G + 1):
        for i in range(L + 1):
            for j in range(i + 1):   # GPU g-1 takes layers [j, i)
                if dp[g - 1][j] == INF:
                    continue
                mem = pre_m[i] - pre_m[j]
                if mem > gpu_mem[g - 1] + 1e-9:
                    continue
                t = (pre_t[i] - pre_t[j]) / max(gpu_speed[g - 1], 1e-12)
                if i > j and j > 0:
                    t += hop_cost
                val = max(dp[g - 1][j], t) if objective == "bottleneck" else dp[g - 1][j] + t
                if val < dp[g][i] - 1e-15:
                    dp[g][i] = val
                    arg[g][i] = j
    if dp[G][L] == INF:
        raise ValueError("model does not fit in the given GPU memory")
    out = []
    i = L
    for g in range(G, 0, -1):
        j = arg[g][i]
        out.append((j, i))
        i = j
    return out[::-1]


def layer_costs(cfg, batch_tokens: int = 1, dtype_bytes: int = 2) -> Tuple[List[float], List[float]]:
    """Analytic per-layer decode time proxy (bytes streamed) and weight memory."""
    H = cfg.hidden_size
    attn = H * (cfg.q_size + 2 * cfg.kv_size) + cfg.q_size * H
    if cfg.is_moe:
        mlp_active = cfg.experts_per_token * 3 * H * cfg.expert_intermediate_size
        mlp_mem = cfg.num_experts * 3 * H * cfg.expert_intermediate_size
    else:
        mlp_active = mlp_mem = (2 if cfg.is_gpt2 else 3) * H * cfg.intermediate_size
    t = float((attn + mlp_active) * dtype_bytes)
    m = float((attn + mlp_mem) * dtype_bytes)
    return [t] * cfg.num_layers, [m] * cfg.num_layers


@dataclass
class Block:
    index: int
    start: int
    end: int
    device: str

    @property
    def num_layers(self) -> int:
        return self.end - self.start


def split_model_into_blocks(cfg, devices: Sequence[str], *, strategy: str = "balanced",
                            gpus: Optional[Sequence[GPUInfo]] = None, profile: bool = False,
                            weights: Optional[Sequence[float]] = None) -> List[Block]:
    """Layer blocks for pipeline stages on `devices` (e.g. ["cuda:0", "cuda:1"] or
    ["cpu", "cpu"]).  Explicit `weights` override detection (equal split when no GPU
    information is available); profile=True uses the DP placement."""
    n = len(devices)
    if weights is None:
        if gpus and len(gpus) == n:
            if profile:
                lt, lm = layer_costs(cfg)
                speed = [g.profile.bw_gbs for g in gpus]
                mem = [g.free_bytes * 0.9 for g in gpus]
                ranges = compute_optimal_placement(lt, lm, speed, mem, objective="bottleneck")
                return [Block(i, a, b, d) for i, ((a, b), d) in enumerate(zip(ranges, devices))]
            weights = compute_scores(gpus, strategy)
        else:
            weights = [1.0] * n
    counts = split_layers(cfg.num_layers, weights)
    return [Block(i, a, b, d) for i, ((a, b), d) in enumerate(zip(ranges_from_counts(counts), devices))]


def assign_blocks_to_gpus(blocks: Sequence[Block], devices: Sequence[str]) -> Dict[int, str]:
    return {b.index: devices[i % len(devices)] for i, b in enumerate(blocks)}


def compute_max_memory(headroom: float = 0.05, cpu_gib: int = 48) -> Dict[object, str]:
    """{gpu_index: "NGiB", "cpu": "48GiB"} from free memory minus headroom."""
    out: Dict[object, str] = {}
    for g in detect_gpus():
        out[g.index] = f"{int(g.free_bytes * (1 - headroom) / 2 ** 30)}GiB"
    out["cpu"] = f"{cpu_gib}GiB"
    return out


def auto_configure(strategy: str = "balanced", num_layers: int = 0) -> Dict[str, object]:
    gpus = detect_gpus()
    tiers = {g.index: g.profile.tier for g in gpus}
    scores = compute_scores(gpus, strategy)
    tot = sum(scores) or 1.0
    ratios = [s / tot for s in scores]
    lend = {g.index: (0.7 if g.profile.tier == 0 else 0.5 if g.profile.tier == 1 else 0.3) for g in gpus}
    cfg = {"gpus": [g.to_dict() for g in gpus], "strategy": strategy, "split_ratios": ratios, "tiers": tiers,
           "lend_ratios": lend, "p2p": probe_p2p(), "vm": detect_vm(), "max_memory": compute_max_memory()}
    if num_layers and gpus:
        cfg["layer_counts"] = split_layers(num_layers, scores)
    return cfg
