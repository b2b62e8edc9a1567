"""Symmetric buffers for the fused GEMM + all-reduce of tensor-parallel decode.

Every rank allocates (cudaMalloc) a receive buffer (two halves x one bf16 slot per
source rank), fills it with the empty pattern 0x8000 (bf16 -0.0), exports a CUDA IPC
handle, gathers its peers' handles over the process group and opens them.  A
row-parallel projection is then two kernels of this package:
  push    the stream-K GEMM (bf16, or e4m3 weights and activations) stores its partial
          (bf16, -0.0 stored as +0.0) into its slot on every rank over NVLink: posted
          stores, no fence, no flag (csrc/gemm_tc.cu);
  reduce  the next norm kernel polls the slots until no value is empty, sums them in
          rank order from local memory, adds bias + residual and normalises, empties
          the slots and advances the epoch that picks the half (csrc/ar_norm.cu):
          bitwise-identical results on every rank, one NVLink write latency per call.
It serves every decode batch of up to max_tokens tokens.  Set up once per process
before any CUDA graph capture; the buffers live until exit.

Reference parity: core/tensor_parallel.py:67-80 all-reduces partial sums with
torch.cuda.nccl.all_reduce; there is no fused path.
"""
from __future__ import annotations

import os
from typing import Optional

import torch
import torch.distributed as dist

from .. import ops


MODE_ADD, MODE_RMSNORM, MODE_LAYERNORM = 0, 1, 2


EMPTY_BF16 = 0x8000


class FusedAllReduce:
    def __init__(self, group=None, max_tokens: int = 128, max_features: int = 16384, device=None,
                 local: bool = False):
        """`local=True` builds a one-rank instance without a process group: the kernels
        run exactly as on a tensor-parallel rank, with only this GPU's slot (used to
        time a TP shard's compute on one GPU)."""
        self.group = group
        self.world = 1 if local else dist.get_world_size(group)
        self.rank = 0 if local else dist.get_rank(group)
        if self.world not in (1, 2, 4, 8):
            raise ValueError("fused all-reduce: world size must be 1, 2, 4 or 8")
        self.device = torch.device(device or f"cuda:{torch.cuda.current_device()}")
        self.max_tokens = min(128, max_tokens)
        self.min_tokens = int(os.environ.get("VRM_FUSED_AR_MIN_TOKENS", "1"))
        self.half_floats = max_features * self.max_tokens
        nat = ops.native()
        with torch.cuda.device(self.device):
            # receive buffer: [2 halves][world source ranks][half_floats] bf16, all empty
            n = 2 * self.world * self.half_floats
            self.xbuf = nat.symm_malloc(n * 2)
            nat.symm_fill_u16(self.xbuf, n, EMPTY_BF16)
            handles = [nat.ipc_handle(self.xbuf)] if not local else [None]
            allh = [handles]
            if not local:
                allh = [None] * self.world
                dist.all_gather_object(allh, handles, group=group)
            xs = []
            self._opened = []
            for r, (hx,) in enumerate(allh):
                if r == self.rank:
                    xs.append(self.xbuf)
                else:
                    px = nat.ipc_open(hx)
                    self._opened.append(px)
                    xs.append(px)
            self.xbuf_ptrs = torch.tensor(xs, dtype=torch.int64, device=self.device)
            self.epoch = torch.zeros(1, dtype=torch.int32, device=self.device)
            self.done = torch.zeros(1, dtype=torch.int32, device=self.device)
        if not local:
            dist.barrier(group=group)

    def supports(self, m: int, n: int) -> bool:
        return self.min_tokens <= m <= self.max_tokens and n % 8 == 0 and n * m <= self.half_floats \
            and n <= 16384

    def push(self, x: torch.Tensor, w: torch.Tensor, scale_x: Optional[torch.Tensor] = None,
             scale_w: Optional[torch.Tensor] = None) -> None:
        """Row-parallel GEMM x @ w.T (e4m3 operands: times scale_x[m] * scale_w[n]) whose
        partial goes to every rank's receive buffer."""
        ops.native().gemm_ar_push(x, w, self.xbuf_ptrs, self.epoch, self.rank, self.world, self.half_floats,
                                  scale_x, scale_w)

    def push_reduce(self, x: torch.Tensor, w: torch.Tensor, residual: torch.Tensor,
                    bias: Optional[torch.Tensor] = None, ssq_out: Optional[torch.Tensor] = None,
                    spin_limit: int = 0) -> None:
        """One kernel: row-parallel GEMM x @ w.T whose partial goes to every rank, then
        the launch's warps sum every rank's partial in rank order (+ bias) into
        `residual` (in place) and store the RMSNorm sums of the new residual per
        128-feature chunk in ssq_out [chunks, >= tokens] (the next GEMM normalises
        from them).  bf16 weights, decode batches (<= max_tokens)."""
        ops.native().gemm_ar_push(x, w, self.xbuf_ptrs, self.epoch, self.rank, self.world, self.half_floats,
                                  None, None, residual, bias, ssq_out, self.done, int(spin_limit))

    def supports_reduce(self, m: int, w) -> bool:
        return (getattr(w, "_vrm_quant", None) is None and isinstance(w, torch.Tensor)
                and w.dtype == torch.bfloat16 and self.supports(m, w.shape[0]) and w.shape[0] % 4 == 0)

    def push_weight(self, x: torch.Tensor, w) -> None:
        """push() for any weight format of a row-parallel projection: bf16, FP8Weight
        (activations quantised per row to e4m3 first) or NVFP4Weight (decode, W4A16)."""
        kind = getattr(w, "_vrm_quant", None)
        if kind is None:
            self.push(x, w)
        elif kind == "fp8":
            xq, sx = ops.native().fp8_rows_quantize(x.contiguous())
            self.push(xq, w.q, sx, w.scale)
        elif kind == "nvfp4":
            ops.native().nvfp4_gemm_ar_push(x, w.q, w.s, w.gs, w.N, self.xbuf_ptrs, self.epoch, self.rank,
                                            self.world, self.half_floats)
        else:
            raise ValueError(f"fused all-reduce: unsupported weight format {kind!r}")

    def supports_weight(self, m: int, w) -> bool:
        kind = getattr(w, "_vrm_quant", None)
        if kind == "nvfp4" and m > ops.native().nvfp4_gemm_max_m():
            return False
        return kind in (None, "fp8", "nvfp4") and self.supports(m, w.shape[0])

    def reduce(self, T: int, H: int, bias: Optional[torch.Tensor] = None, residual: Optional[torch.Tensor] = None,
               out: Optional[torch.Tensor] = None, norm_w: Optional[torch.Tensor] = None,
               norm_b: Optional[torch.Tensor] = None, eps: float = 1e-6, layernorm: bool = False,
               spin_limit: int = 0, err: Optional[torch.Tensor] = None) -> None:
        """Waits for every rank's partial of the last push, then
        s = sum(partials) (+ bias) (+ residual) -> residual; out = s or norm(s)."""
        mode = MODE_ADD if norm_w is None else (MODE_LAYERNORM if layernorm else MODE_RMSNORM)
        ops.native().ar_norm(self.xbuf, self.epoch, self.done, self.rank, self.world, self.half_floats, T, H,
                             bias, residual, norm_w, norm_b, out, mode, float(eps), int(spin_limit), err)

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
