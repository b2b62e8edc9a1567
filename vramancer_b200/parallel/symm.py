"""Symmetric buffers for the fused GEMM + all-reduce of tensor-parallel decode.

Every rank allocates (cudaMalloc) a receive buffer (two halves x one bf16 slot per
source rank) and a flag word per source rank, exports CUDA IPC handles, gathers its
peers' handles over the process group and opens them.  A row-parallel projection is
then two kernels of this package:
  push    the stream-K GEMM stores its partial (bf16) into its slot on every rank over
          NVLink and flags the peers when its last CTA finishes (csrc/gemm_tc.cu);
  reduce  the next norm kernel waits for the peers' flags, sums the slots in rank
          order from local memory, adds bias + residual and normalises
          (csrc/ar_norm.cu), giving bitwise-identical results on every rank.
Set up once per process before any CUDA graph capture; the buffers live until exit.

Reference parity: core/tensor_parallel.py:67-80 all-reduces partial sums with
torch.cuda.nccl.all_reduce; there is no fused path.
"""
from __future__ import annotations

import math
import os
from typing import Optional

import torch
import torch.distributed as dist

from .. import ops


MODE_ADD, MODE_RMSNORM, MODE_LAYERNORM = 0, 1, 2


class FusedAllReduce:
    def __init__(self, group=None, max_tokens: int = 128, max_features: int = 16384, device=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device or f"cuda:{torch.cuda.current_device()}")
        self.max_tokens = max_tokens
        # below this many tokens NCCL's small-message all-reduce is faster than the
        # push + flag round trip (B200, TP=2: bs1 178 vs 171 tok/s; bs32 4557 vs 4653)
        self.min_tokens = int(os.environ.get("VRM_FUSED_AR_MIN_TOKENS", "16"))
        self.per_thread_fence = os.environ.get("VRM_AR_THREAD_FENCE", "0") == "1"
        self.half_floats = max_features * max_tokens
        nat = ops.native()
        with torch.cuda.device(self.device):
            # receive buffer: [2 halves][world source ranks][half_floats] bf16; flags [world]
            self.xbuf = nat.symm_malloc(2 * self.world * self.half_floats * 2)
            self.flags = nat.symm_malloc(max(16, self.world * 4))
            handles = [nat.ipc_handle(self.xbuf), nat.ipc_handle(self.flags)]
            allh = [None] * self.world
            dist.all_gather_object(allh, handles, group=group)
            xs, fs = [], []
            self._opened = []
            for r, (hx, hf) in enumerate(allh):
                if r == self.rank:
                    xs.append(self.xbuf)
                    fs.append(self.flags)
                else:
                    px, pf = nat.ipc_open(hx), nat.ipc_open(hf)
                    self._opened += [px, pf]
                    xs.append(px)
                    fs.append(pf)
            self.xbuf_ptrs = torch.tensor(xs, dtype=torch.int64, device=self.device)
            self.flag_ptrs = torch.tensor(fs, dtype=torch.int64, device=self.device)
            self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
            self.done = torch.zeros(1, dtype=torch.int32, device=self.device)
        dist.barrier(group=group)

    def supports(self, m: int, n: int) -> bool:
        return self.min_tokens <= m <= min(128, self.max_tokens) and n % 8 == 0 and n * m <= self.half_floats \
            and n <= 16384

    def push(self, x: torch.Tensor, w: torch.Tensor) -> None:
        """Row-parallel GEMM x @ w.T whose partial goes to every rank's receive buffer."""
        ops.native().gemm_ar_push(x, w, self.xbuf_ptrs, self.flag_ptrs, self.epoch, self.done, self.rank,
                                  self.world, self.half_floats, self.per_thread_fence)

    def reduce(self, T: int, H: int, bias: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None,
               out: Optional[torch.Tensor] = None, norm_w: Optional[torch.Tensor] = None,
               norm_b: Optional[torch.Tensor] = None, eps: float = 1e-6, layernorm: bool = False) -> None:
        """Waits for the peers' partials of the last push, then
        s = sum(partials) (+ bias) (+ residual) -> residual; out = s or norm(s)."""
        mode = MODE_ADD if norm_w is None else (MODE_LAYERNORM if layernorm else MODE_RMSNORM)
        ops.native().ar_norm(self.xbuf, self.flags, self.epoch, self.rank, self.world, self.half_floats, T, H,
                             bias, residual, norm_w, norm_b, out, mode, float(eps))

    def linear(self, x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None, *,
               residual: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """out = allreduce_over_ranks(x @ w.T) (+ bias) (+ residual): push + reduce."""
        T, H = x.shape[0], w.shape[0]
        if out is None:
            out = torch.empty(T, H, dtype=x.dtype, device=x.device)
        if residual is not None and out is not residual:
            out.copy_(residual)          # the reduce kernel updates its residual in place
        self.push(x, w)
        self.reduce(T, H, bias, out if residual is not None else None, out)
        return out
