"""Mixture-of-experts layer: top-k softmax router over SwiGLU experts.

On CUDA the routed experts run on the device without a host round trip (capturable in
the decode CUDA graph): router GEMM and top-k, then csrc/moe.cu plans the expert-grouped
rows and token blocks, gathers the activations, the grouped tcgen05 GEMM
(csrc/gemm_tc.cu, moe_grouped_swap_kernel) runs gate/up with the fused SiLU*up
epilogue and down over every block, and the combine sums each token's top-k rows (plus
the shared expert) in k order.  On the CPU (the oracle) tokens are grouped by expert
with one sort and each expert runs as a dense MLP.

Reference parity: the reference has no MoE of its own (vLLM / llama.cpp only, plus
the expert placement hooks of core/expert_pinning.py:115-642).
"""
from __future__ import annotations

from typing import Optional, Tuple

import torch

from .. import ops
from ..models.config import ModelConfig

DEVICE_MOE = True       # CUDA MoE layers need no host synchronisation (graph-capturable)

_usage_hook = None      # parallel.expert_placement.ExpertUsage (or None)


def set_usage_hook(usage) -> None:
    """Every MoE layer call reports its routing to `usage.observe(ids)` (None: off).  On
    CUDA the routing is then computed twice per call (once for the hook)."""
    global _usage_hook
    _usage_hook = usage


def route(cfg: ModelConfig, x: torch.Tensor, router_w: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
    """Returns (weights [T, k] fp32, expert ids [T, k] int64).  On CUDA the softmax /
    top-k / renormalisation run in the same kernel as the MoE layer's own routing."""
    logits = ops.linear(x, router_w)
    if x.is_cuda:
        ids, w = ops.native().moe_route(logits, cfg.experts_per_token, bool(cfg.norm_topk_prob), 16)[:2]
        return w, ids
    probs = torch.softmax(logits.float(), dim=-1)
    w, ids = torch.topk(probs, cfg.experts_per_token, dim=-1)
    if cfg.norm_topk_prob:
        w = w / w.sum(-1, keepdim=True)
    return w, ids


def expert_mlp(x: torch.Tensor, gate_up: torch.Tensor, down: torch.Tensor) -> torch.Tensor:
    h = ops.linear(x, gate_up, epilogue=ops.EPI_SILU_MUL)
    return ops.linear(h, down)


def moe_forward(cfg: ModelConfig, x: torch.Tensor, router_w: torch.Tensor, experts_gate_up: torch.Tensor,
                experts_down: torch.Tensor, *, shared_gate_up: Optional[torch.Tensor] = None,
                shared_down: Optional[torch.Tensor] = None,
                shared_gate: Optional[torch.Tensor] = None,
                expert_offset: int = 0, residual: Optional[torch.Tensor] = None,
                norm_w: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
    """x [T, H] -> [T, H].  experts_* hold experts [expert_offset, expert_offset + E_local).
    With `residual` the output is added into it in place (bf16) and the result is
    RMSNorm(residual) * norm_w when `norm_w` is given (the next layer's input), else None."""
    if _usage_hook is not None and x.shape[0] > 0:
        _usage_hook.observe(route(cfg, x, router_w)[1])
    if x.is_cuda and expert_offset == 0 and experts_gate_up.shape[0] == cfg.num_experts:
        return _moe_device(cfg, x, router_w, experts_gate_up, experts_down, shared_gate_up, shared_down,
                           shared_gate, residual, norm_w)
    T, H = x.shape
    w, ids = route(cfg, x, router_w)
    out = torch.zeros(T, H, dtype=torch.float32, device=x.device)
    flat = ids.flatten()
    order = torch.argsort(flat, stable=True)
    e_local = experts_gate_up.shape[0]
    counts = torch.bincount(flat - expert_offset if expert_offset else flat,
                            minlength=max(cfg.num_experts, e_local)).cpu().tolist()
    tok_of = order // cfg.experts_per_token
    wflat = w.flatten()[order]
    start = 0
    for e, n in enumerate(counts):
        if n == 0:
            continue
        sel = slice(start, start + n)
        start += n
        le = e
        if le < 0 or le >= e_local:
            continue
        toks = tok_of[sel]
        y = expert_mlp(x.index_select(0, toks).contiguous(), experts_gate_up[le], experts_down[le])
        out.index_add_(0, toks, y.float() * wflat[sel].unsqueeze(1))
    if shared_gate_up is not None:
        ys = expert_mlp(x, shared_gate_up, shared_down).float()
        if shared_gate is not None:
            ys = ys * torch.sigmoid(ops.linear(x, shared_gate).float())
        out += ys
    if residual is None:
        return out.to(x.dtype)
    residual.copy_((residual.float() + out).to(residual.dtype))
    return ops.rmsnorm(residual, norm_w, cfg.norm_eps) if norm_w is not None else None


def moe_block_rows(tokens: int, topk: int, experts: int) -> int:
    """Token rows per block of the grouped GEMM: the average rows per expert, rounded
    up to an MMA width (16 / 32 / 64 / 128)."""
    avg = -(-tokens * topk // max(1, experts))
    for bn in (16, 32, 64):
        if avg <= bn:
            return bn
    return 128


def _moe_device(cfg: ModelConfig, x: torch.Tensor, router_w, gate_up, down, shared_gate_up, shared_down,
                shared_gate, residual, norm_w) -> Optional[torch.Tensor]:
    add = None
    if shared_gate_up is not None:
        ys = expert_mlp(x, shared_gate_up, shared_down)
        if shared_gate is not None:
            ys = (ys.float() * torch.sigmoid(ops.linear(x, shared_gate).float())).to(x.dtype)
        add = ys.contiguous()
    logits = ops.linear(x, router_w)
    bn = moe_block_rows(x.shape[0], cfg.experts_per_token, cfg.num_experts)
    out = ops.native().moe_layer(x.contiguous(), logits, cfg.experts_per_token, bool(cfg.norm_topk_prob),
                                 gate_up.contiguous(), down.contiguous(), bn, add, residual, norm_w, cfg.norm_eps)
    return out if (residual is None or norm_w is not None) else None
