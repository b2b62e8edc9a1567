"""Symmetric buffers for the fused GEMM + all-reduce of tensor-parallel decode.

Every rank allocates (cudaMalloc) a receive buffer (two halves x one slot per source
rank) and a flag array,
exports CUDA IPC handles, gathers its peers' handles over the process group and opens
them; the device then holds [world]-long arrays of the ranks' buffer and flag
pointers, which the row-parallel GEMM epilogue uses to publish its tiles, wait for
the peers' tiles and reduce them (csrc/gemm_tc.cu, ARParams).  Set up once per
process before any CUDA graph capture; the buffers live until exit.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.distributed as dist

from .. import ops


class FusedAllReduce:
    def __init__(self, group=None, max_tokens: int = 128, max_features: int = 8192, device=None):
        self.group = group
        self.world = dist.get_world_size(group)
        self.rank = dist.get_rank(group)
        self.device = torch.device(device or f"cuda:{torch.cuda.current_device()}")
        self.max_tiles = math.ceil(max_features / 128)
        self.half_floats = self.max_tiles * 128 * max_tokens
        nat = ops.native()
        with torch.cuda.device(self.device):
            # receive buffer: [2 halves][world source ranks][half_floats] fp32
            self.xbuf = nat.symm_malloc(2 * self.world * self.half_floats * 4)
            self.flags = nat.symm_malloc(self.world * self.max_tiles * 4)
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
        return m <= 128 and math.ceil(n / 128) <= self.max_tiles and n * m <= self.half_floats

    def linear(self, x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None, *,
               residual: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
        """out = allreduce_over_ranks(x @ w.T) (+ bias) (+ residual), in one kernel."""
        if out is None:
            out = torch.empty(x.shape[0], w.shape[0], dtype=x.dtype, device=x.device)
        ops.native().gemm_ar_out(x, w, bias, out, residual, self.xbuf_ptrs, self.flag_ptrs, self.epoch, self.done,
                                 self.rank, self.world, self.max_tiles, self.half_floats)
        return out
