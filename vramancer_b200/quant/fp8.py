"""FP8 (e4m3) W8A8 weights: one scale per output channel, activations quantised per
token on the fly, GEMM on the tensor cores' fp8 path (tcgen05 kind::f8f6f4).

    w = quantize(w_bf16)                 # FP8Weight on w's device
    y = ops.linear(x, w, ...)            # per-token activation quantisation + W8A8 GEMM
    weights = quantize_model_weights(weights, cfg)

Convention: scale[r] = amax(|row r|) / 448 (1 for a zero row), q = e4m3_rn_sat(x / scale);
y[m, n] = sum_k q_x[m, k] q_w[n, k] * scale_x[m] * scale_w[n].  The functions ending in
_ref restate the CUDA kernels (csrc/fp8.cu, csrc/gemm_tc.cu gemm_fp8) on the host.

Reference parity: the reference's 8-bit mode is bitsandbytes LLM.int8 (core/backends.py
HuggingFaceBackend quantisation switch, `-q int8`); here 8-bit weights use the e4m3
format the B200 tensor cores run natively.
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Dict, Optional

import torch

from .. import ops

E4M3_MAX = 448.0
QUANTIZED_KEYS = ("qkv_w", "o_w", "gate_up_w", "down_w", "fc_w", "proj_w")


@dataclass
class FP8Weight:
    q: torch.Tensor          # uint8 [N, K] (e4m3 bits)
    scale: torch.Tensor      # fp32 [N]
    N: int
    K: int
    _vrm_quant = "fp8"

    @property
    def shape(self):
        return torch.Size((self.N, self.K))

    @property
    def device(self):
        return self.q.device

    @property
    def dtype(self):
        return torch.bfloat16

    @property
    def is_cuda(self) -> bool:
        return self.q.is_cuda

    def nbytes(self) -> int:
        return self.q.numel() + 4 * self.scale.numel()

    def dequantize(self) -> torch.Tensor:
        return dequantize_rows_ref(self.q, self.scale)

    def linear(self, x: torch.Tensor, bias: Optional[torch.Tensor] = None, *, out: Optional[torch.Tensor] = None,
               epilogue: int = ops.EPI_NONE, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        if x.is_cuda:
            xq, sx = ops.native().fp8_rows_quantize(x.contiguous())
            if out is None:
                n = self.N // 2 if epilogue == ops.EPI_SILU_MUL else self.N
                out = torch.empty(x.shape[0], n, dtype=x.dtype, device=x.device)
            ops.native().gemm_fp8_out(xq, sx, self.q, self.scale, bias, out, epilogue, residual)
            return out
        xq, sx = quantize_rows_ref(x)
        xd = dequantize_rows_ref(xq, sx).to(x.dtype)
        return ops.linear(xd, self.dequantize().to(x.dtype), bias, out=out, epilogue=epilogue, residual=residual)


def quantize_rows_ref(x: torch.Tensor):
    """(q uint8 [R, K], scale fp32 [R]) on the host, as fp8_rows_quantize."""
    xf = x.detach().float().cpu()
    amax = xf.abs().amax(1)
    scale = torch.where(amax > 0, amax / torch.full_like(amax, E4M3_MAX), torch.ones_like(amax))
    q = (xf / scale[:, None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn).view(torch.uint8)
    return q, scale


def dequantize_rows_ref(q: torch.Tensor, scale: torch.Tensor) -> torch.Tensor:
    return q.cpu().view(torch.float8_e4m3fn).float() * scale.cpu().float()[:, None]


def quantize(w: torch.Tensor) -> FP8Weight:
    if w.dim() != 2:
        raise ValueError("fp8: 2-D weight expected")
    if w.is_cuda:
        q, s = ops.native().fp8_rows_quantize(w.to(torch.bfloat16).contiguous())
    else:
        q, s = quantize_rows_ref(w)
    return FP8Weight(q, s, w.shape[0], w.shape[1])


def quantizable(w) -> bool:
    return isinstance(w, torch.Tensor) and w.dim() == 2 and w.shape[1] % 128 == 0


def quantize_model_weights(weights: Dict[str, torch.Tensor], cfg=None, keys=QUANTIZED_KEYS) -> Dict[str, object]:
    """Every layer projection to FP8 (embeddings, norms, biases, lm_head, MoE experts stay bf16)."""
    out = dict(weights)
    for name, w in weights.items():
        if name.rsplit(".", 1)[-1] in keys and quantizable(w):
            out[name] = quantize(w)
    return out
