"""Environment heuristics: quantisation, backend and peer-access recommendations.

Reference parity: core/auto_detect.py (recommend_quantization, detect_virtualization,
should_disable_p2p, recommend_backend).
"""
from __future__ import annotations

from typing import Dict, Optional

BYTES_PER_PARAM = {"none": 2.0, "fp8": 1.0, "nvfp4": 0.5625}   # bf16 / fp8 / e2m1 + e4m3 per 16


def model_gb(params_b: float, quant: str = "none", overhead: float = 1.2) -> float:
    return params_b * BYTES_PER_PARAM[quant] * overhead


def recommend_quantization(vram_gb: float, params_b: float, kv_headroom: float = 0.25) -> str:
    """Least aggressive format whose weights leave `kv_headroom` of VRAM for the KV cache."""
    for q in ("none", "fp8", "nvfp4"):
        if model_gb(params_b, q) <= vram_gb * (1 - kv_headroom):
            return q
    return "nvfp4"


def detect_virtualization() -> Dict[str, object]:
    from ..parallel.placement import detect_vm
    return detect_vm()


def should_disable_p2p(vm: Optional[Dict[str, object]] = None) -> bool:
    """Peer access through a hypervisor without NVLink passthrough is unreliable."""
    vm = vm if vm is not None else detect_virtualization()
    return bool(vm.get("virtualized")) and vm.get("hypervisor") not in (None, "none", "")


def recommend_backend(model: str) -> str:
    from ..backends import native_supports
    if str(model).lower().endswith(".gguf"):
        return "llamacpp"
    return "native" if native_supports(model) else "huggingface"
