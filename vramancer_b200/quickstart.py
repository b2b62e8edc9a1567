"""`vramancer quickstart`: pick the largest catalog model that fits the detected GPUs,
and with --run / --serve launch it.

Estimated footprint = params x bytes/param x 1.2 + 1.5 GB (bytes/param: nvfp4 0.60,
fp8 1.0, bf16 2.0); Blackwell GPUs prefer NVFP4 when it buys a larger model.

Reference parity: vramancer/quickstart.py:23-131 (CATALOG, _BPP, recommend,
run_quickstart).
"""
from __future__ import annotations

from typing import Callable, Dict, List, Optional

CATALOG: Dict[str, List[Dict]] = {
    "code-assistant": [
        {"model": "Qwen/Qwen2.5-Coder-32B-Instruct", "params_b": 32.8},
        {"model": "Qwen/Qwen2.5-Coder-14B-Instruct", "params_b": 14.8},
        {"model": "Qwen/Qwen2.5-Coder-7B-Instruct", "params_b": 7.6},
        {"model": "Qwen/Qwen2.5-Coder-1.5B-Instruct", "params_b": 1.5},
    ],
    "chat": [
        {"model": "Qwen/Qwen2.5-72B-Instruct", "params_b": 72.7},
        {"model": "Qwen/Qwen2.5-32B-Instruct", "params_b": 32.8},
        {"model": "Qwen/Qwen2.5-14B-Instruct", "params_b": 14.8},
        {"model": "Qwen/Qwen2.5-7B-Instruct", "params_b": 7.6},
        {"model": "Qwen/Qwen2.5-0.5B-Instruct", "params_b": 0.5},
    ],
    "summarize": [
        {"model": "Qwen/Qwen2.5-14B-Instruct", "params_b": 14.8},
        {"model": "Qwen/Qwen2.5-7B-Instruct", "params_b": 7.6},
        {"model": "Qwen/Qwen2.5-3B-Instruct", "params_b": 3.1},
    ],
}
BYTES_PER_PARAM = {"nvfp4": 0.60, "fp8": 1.0, "bf16": 2.0}


def estimate_gb(params_b: float, quant: str) -> float:
    return params_b * BYTES_PER_PARAM[quant] * 1.2 + 1.5


def recommend(use_case: str, vram_gb: float, blackwell: bool = True) -> Optional[Dict]:
    quants = ["bf16", "fp8", "nvfp4"] if blackwell else ["bf16", "fp8"]
    for entry in CATALOG.get(use_case, CATALOG["chat"]):
        for q in quants:
            need = estimate_gb(entry["params_b"], q)
            if need <= vram_gb:
                return {"model": entry["model"], "quantization": q, "estimated_gb": round(need, 1),
                        "vram_gb": round(vram_gb, 1), "use_case": use_case}
    return None


def command_for(rec: Dict, serve: bool = False) -> List[str]:
    """The `vramancer run | serve` command line that launches a recommendation."""
    cmd = ["vramancer", "serve" if serve else "run", rec["model"]]
    if rec["quantization"] != "bf16":
        cmd += ["--quantization", rec["quantization"]]
    return cmd


def run_quickstart(use_case: str = "chat", run: bool = False, serve: bool = False, *, prompt: Optional[str] = None,
                   port: int = 5030, gpus=None, launcher: Optional[Callable[[str, object], int]] = None) -> Optional[Dict]:
    """Recommends a model for the detected GPUs; with run / serve it also launches it
    through the same code path as `vramancer run` / `vramancer serve` (interactive
    generation, or one prompt with `prompt`; the API server on `port`).  The result
    carries the command line and, when launched, the launcher's exit code."""
    if gpus is None:
        from .parallel.placement import detect_gpus
        gpus = detect_gpus()
    vram = sum(g.free_gb for g in gpus)
    rec = recommend(use_case, vram, blackwell=any(g.capability[0] >= 10 for g in gpus))
    if rec is None:
        return None
    rec["command"] = " ".join(command_for(rec, serve=serve))
    if not (run or serve):
        return rec
    from types import SimpleNamespace
    q = None if rec["quantization"] == "bf16" else rec["quantization"]
    if serve:
        ns = SimpleNamespace(model=rec["model"], model_pos=None, backend="auto", gpus=None, tp=1, host="0.0.0.0",
                             port=port, quantization=q, cluster=True, profile=None, max_model_len=None,
                             num_layers=None)
        kind = "serve"
    else:
        ns = SimpleNamespace(model=rec["model"], prompt=prompt, max_tokens=256, temperature=0.7, backend="auto",
                             gpus=None, quantization=q, num_layers=None)
        kind = "run"
    if launcher is None:
        from . import cli
        launcher = lambda k, a: cli._cmd_serve(a) if k == "serve" else cli._cmd_run(a)   # noqa: E731
    rec["launched"] = kind
    rec["exit_code"] = launcher(kind, ns)
    return rec
