"""Expert parallelism: MoE experts sharded over the ranks, attention data-parallel.

Rank r holds experts [r * E / W, (r + 1) * E / W) and every non-expert weight; each
rank runs its own sequences (own KV cache, own scheduler) and the ranks meet at every
MoE layer.  On CUDA one layer is seven kernels with no host round trip
(csrc/moe_ep.cu, csrc/moe.cu, csrc/gemm_tc.cu):
  route+plan  local softmax / top-k and the per-expert plan
  counts      per-expert counts -> every rank (peer stores + flag)
  dispatch    routed rows -> the owner's receive buffer over NVLink, tagged (rank, pair)
  owner plan  block list over the local experts once every rank's rows have landed
  gate/up     grouped tcgen05 GEMM over the received rows
  down        grouped GEMM whose epilogue stores each row back into its source rank
  combine     weighted k-order sum (+ residual + next RMSNorm) after every owner's flag
Buffers are CUDA IPC allocations exchanged once (like the fused all-reduce); the
call counter lives on the device, so the layer can be captured in a CUDA graph.

Every rank must run the same sequence of MoE layer calls (a rank with nothing to do
runs a one-token dummy step: engine.EPSync).  On the CPU (gloo) the same semantics
run through collectives: all-gather of the tokens, local experts on every token,
all-reduce of the partial outputs.

Reference parity: the reference has no expert parallelism (vLLM / llama.cpp MoE only;
core/expert_pinning.py:281-640 stages cold experts from a lender GPU).
"""
from __future__ import annotations

from typing import List, Optional, Tuple

import torch
import torch.distributed as dist

from .. import ops
from ..models.config import ModelConfig


class ExpertParallel:
    """Expert-parallel group state for one process (one rank)."""

    def __init__(self, cfg: ModelConfig, group=None, max_tokens: int = 1024, device=None):
        if not cfg.is_moe:
            raise ValueError("expert parallelism needs a MoE model")
        self.cfg = cfg
        self.group = group
        self.world = dist.get_world_size(group) if dist.is_initialized() else 1
        self.rank = dist.get_rank(group) if dist.is_initialized() else 0
        if cfg.num_experts % self.world:
            raise ValueError(f"{cfg.num_experts} experts do not divide over {self.world} ranks")
        self.E = cfg.num_experts
        self.E_local = self.E // self.world
        self.max_tokens = max_tokens
        self.device = torch.device(device) if device is not None else (
            torch.device("cuda", torch.cuda.current_device()) if torch.cuda.is_available() else torch.device("cpu"))
        self.native = self.device.type == "cuda"
        if self.native:
            self._setup_buffers()

    # ------------------------------------------------------------------ buffers
    def _setup_buffers(self) -> None:
        cfg, W = self.cfg, self.world
        H, k = cfg.hidden_size, cfg.experts_per_token
        self.p_cap = self.max_tokens * k
        self.r_rows = W * self.p_cap + 128
        sizes = [2 * W * self.E * 4,                  # cnt
                 2 * self.r_rows * H * 2,             # xrecv
                 2 * self.r_rows * 4,                 # meta
                 2 * self.p_cap * H * 2,              # yback
                 max(64, 3 * W * 4)]                  # flags
        nat = ops.native()
        with torch.cuda.device(self.device):
            self.local = [nat.symm_malloc(n) for n in sizes]
            handles = [nat.ipc_handle(p) for p in self.local]
            allh: List = [None] * W
            if W > 1:
                dist.all_gather_object(allh, handles, group=self.group)
            else:
                allh = [handles]
            table, self._opened = [[None] * W for _ in sizes], []
            for r in range(W):
                for j in range(len(sizes)):
                    if r == self.rank:
                        table[j][r] = self.local[j]
                    else:
                        p = nat.ipc_open(allh[r][j])
                        self._opened.append(p)
                        table[j][r] = p
            self.ptrs = torch.tensor([p for row in table for p in row], dtype=torch.int64, device=self.device)
            self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
            self.done = torch.zeros(2, dtype=torch.int32, device=self.device)
        self.desc = [self.rank, W, self.E, H, self.p_cap, self.r_rows] + list(self.local)
        if W > 1:
            dist.barrier(group=self.group)

    def expert_range(self) -> Tuple[int, int]:
        return self.rank * self.E_local, (self.rank + 1) * self.E_local

    # ------------------------------------------------------------------ forward
    def forward(self, x: torch.Tensor, router_w: torch.Tensor, gate_up: torch.Tensor, down: torch.Tensor, *,
                add: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None,
                norm_w: Optional[torch.Tensor] = None) -> Optional[torch.Tensor]:
        """This rank's tokens x [T, H] through the sharded experts (gate_up / down hold
        the local experts).  Same return convention as parallel.moe.moe_forward."""
        cfg = self.cfg
        if not self.native:
            return self._forward_collective(x, router_w, gate_up, down, add, residual, norm_w)
        from .moe import moe_block_rows
        if x.shape[0] > self.max_tokens:
            raise ValueError(f"{x.shape[0]} tokens exceed the expert-parallel capacity {self.max_tokens}")
        logits = (ops.linear(x, router_w) if x.shape[0] else
                  torch.empty(0, router_w.shape[0], dtype=x.dtype, device=x.device))
        bn = moe_block_rows(max(1, x.shape[0]) * self.world, cfg.experts_per_token, cfg.num_experts)
        out = ops.native().moe_ep_layer(x.contiguous(), logits, cfg.experts_per_token, bool(cfg.norm_topk_prob),
                                        gate_up.contiguous(), down.contiguous(), bn, self.ptrs, self.desc,
                                        self.epoch, self.done, add, residual, norm_w, cfg.norm_eps)
        return out if (residual is None or norm_w is not None) else None

    def _forward_collective(self, x, router_w, gate_up, down, add, residual, norm_w):
        """Reference semantics over collectives (gloo on the CPU): every rank applies its
        experts to every rank's tokens and the partial outputs are summed."""
        from .moe import expert_mlp, route
        cfg, W = self.cfg, self.world
        T = torch.tensor([x.shape[0]], dtype=torch.int64)
        Ts = [torch.zeros_like(T) for _ in range(W)]
        dist.all_gather(Ts, T, group=self.group)
        Ts = [int(t) for t in Ts]
        Tmax = max(Ts)
        pad = torch.zeros(Tmax, x.shape[1], dtype=x.dtype)
        pad[: x.shape[0]] = x
        xs = [torch.empty_like(pad) for _ in range(W)]
        dist.all_gather(xs, pad, group=self.group)
        xall = torch.cat([xs[r][: Ts[r]] for r in range(W)], 0)
        w, ids = route(cfg, xall, router_w)
        lo, hi = self.expert_range()
        part = torch.zeros(xall.shape[0], xall.shape[1], dtype=torch.float32)
        for e in range(lo, hi):
            sel = (ids == e)
            rows = sel.any(-1).nonzero().flatten()
            if rows.numel() == 0:
                continue
            y = expert_mlp(xall.index_select(0, rows).contiguous(), gate_up[e - lo], down[e - lo]).float()
            part.index_add_(0, rows, y * (w * sel).sum(-1, keepdim=True)[rows])
        dist.all_reduce(part, group=self.group)
        off = sum(Ts[: self.rank])
        out = part[off: off + x.shape[0]]
        if add is not None:
            out = out + add.float()
        if residual is None:
            return out.to(x.dtype)
        residual.copy_((residual.float() + out).to(residual.dtype))
        return ops.rmsnorm(residual, norm_w, cfg.norm_eps) if norm_w is not None else None


def shard_experts(t: torch.Tensor, rank: int, world: int) -> torch.Tensor:
    """Rows [rank * E / world, (rank + 1) * E / world) of an [E, ...] expert tensor."""
    E = t.shape[0]
    if E % world:
        raise ValueError(f"{E} experts do not divide over {world} ranks")
    n = E // world
    return t[rank * n:(rank + 1) * n].contiguous()
