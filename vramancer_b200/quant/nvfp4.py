"""NVFP4 weights (e2m1 values, e4m3 scale per 16 K-elements, fp32 per-tensor scale).

    w = quantize(w_bf16)            # NVFP4Weight, on w's device
    y = ops.linear(x, w, ...)       # W4A16 warp-MMA GEMM for M <= 32 (decode); above,
                                    # fused activation quantisation + W4A4 block-scaled
                                    # tcgen05 GEMM (csrc/nvfp4_bs.cu, prefill)
    weights = quantize_model_weights(weights, cfg)    # every layer projection

Convention: gs = amax / (6 * 448); block scale s = e4m3_rn_sat(block_amax / 6 / gs);
q = e2m1_rn_sat(w / (s * gs)) with ties to the even code.  The CPU functions here are
the oracle for the CUDA kernels (csrc/nvfp4.cu) and run the same math on the host.

Reference parity: core/nvfp4_direct.py (DirectFP4Linear: quantise bf16 weights, M = 1
GEMV kernel, dequantise + torch.mm otherwise) and core/fused_act_quant.py (the
reference's activation quantisation, W4A4).  Here weights are W4 and activations stay
16-bit, so there is no activation quantisation on the hot path.
"""
from __future__ import annotations

import os
from dataclasses import dataclass
from typing import Dict, Optional

import torch

from .. import ops

FP4_MAX = 6.0
E4M3_MAX = 448.0
E2M1_VALUES = (0.0, 0.5, 1.0, 1.5, 2.0, 3.0, 4.0, 6.0)
_BOUNDS = (0.25, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0)

# projections quantised by quantize_model_weights
QUANTIZED_KEYS = ("qkv_w", "o_w", "gate_up_w", "down_w", "fc_w", "proj_w")


# Decode GEMM kernel (M <= 128 tokens): "mma" = warp-MMA W4A16 over fragment-order codes,
# "tc" = tcgen05 W4A16 over the block-scaled copy (VRM_NVFP4_DECODE)
DECODE_KERNEL = os.environ.get("VRM_NVFP4_DECODE", "mma")


@dataclass
class NVFP4Weight:
    q: torch.Tensor      # uint8 [N * K / 2], fragment order
    s: torch.Tensor      # uint8 [N * K / 16], e4m3 block scales, fragment order
    gs: torch.Tensor     # fp32 [1], per-tensor scale
    N: int
    K: int
    # the same codes and scales in the block-scaled layout of csrc/nvfp4_bs.cu (row-major
    # codes [N, K/2] + 128x4 scale atoms) for the tcgen05 W4A4 GEMM of prefill batches
    q_rows: Optional[torch.Tensor] = None
    s_atoms: Optional[torch.Tensor] = None
    _vrm_quant = "nvfp4"

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
        extra = 0 if self.q_rows is None else self.q_rows.numel() + self.s_atoms.numel()
        return self.q.numel() + self.s.numel() + 4 + extra

    def dequantize(self) -> torch.Tensor:
        if self.q.is_cuda:
            return ops.native().nvfp4_dequantize(self.q, self.s, self.gs, self.N, self.K)
        return dequantize_ref(self)          # host: fp32, the CPU paths compute in fp32

    def linear(self, x: torch.Tensor, bias: Optional[torch.Tensor] = None, *, out: Optional[torch.Tensor] = None,
               epilogue: int = ops.EPI_NONE, residual: Optional[torch.Tensor] = None) -> torch.Tensor:
        if (x.is_cuda and x.shape[0] <= 128 and self.q_rows is not None and DECODE_KERNEL == "tc"
                and self.N % 128 == 0 and x.dtype == torch.bfloat16):
            # decode: W4A16 on tcgen05 (codes dequantised to f16 tiles in shared memory)
            if out is None:
                n = self.N // 2 if epilogue == ops.EPI_SILU_MUL else self.N
                out = torch.empty(x.shape[0], n, dtype=x.dtype, device=x.device)
            ops.native().nvfp4_tc_gemm_out(x.contiguous(), self.q_rows, self.s_atoms, self.gs, bias, out, epilogue,
                                           residual)
            return out
        if x.is_cuda and x.shape[0] <= 32:
            # decode: W4A16, bandwidth-bound (fragment-order codes, warp-level MMAs)
            if out is None:
                n = self.N // 2 if epilogue == ops.EPI_SILU_MUL else self.N
                out = torch.empty(x.shape[0], n, dtype=x.dtype, device=x.device)
            ops.native().nvfp4_gemm_out(x, self.q, self.s, self.gs, self.N, bias, out, epilogue, residual)
            return out
        if x.is_cuda and self.q_rows is not None and x.dtype == torch.bfloat16:
            # prefill: fused activation quantisation (per-token scale) + W4A4 block-scaled
            # tcgen05 GEMM with the epilogue in the kernel
            M = x.shape[0]
            qa, sfa, gsa = ops.native().nvfp4_rows_quantize(x.contiguous(), (M + 127) // 128 * 128, None)
            return ops.native().nvfp4_bs_gemm(qa, sfa, gsa, M, self.q_rows, self.s_atoms, self.gs, bias, residual,
                                              epilogue, out)
        return ops.linear(x, self.dequantize(), bias, out=out, epilogue=epilogue, residual=residual)


# ---------------------------------------------------------------- fragment order
def _frag_index(N: int, K: int):
    """(rows, cols) [N/16, K/64, 32, 16, 2] of every nibble in q's fragment order and
    (rows, blocks) [N/16, K/64, 8, 4, 2] of every byte of s."""
    st = torch.arange(N // 16).view(-1, 1, 1, 1, 1, 1)
    tl = torch.arange(K // 64).view(1, -1, 1, 1, 1, 1)
    ln = torch.arange(32).view(1, 1, -1, 1, 1, 1)
    j = torch.arange(4).view(1, 1, 1, -1, 1, 1)
    i = torch.arange(4).view(1, 1, 1, 1, -1, 1)
    e = torch.arange(2).view(1, 1, 1, 1, 1, -1)
    rows = st * 16 + ln // 4 + 8 * (i & 1)
    cols = tl * 64 + j * 16 + (ln % 4) * 2 + 8 * (i >> 1) + e
    shape = (N // 16, K // 64, 32, 16, 2)
    rows = rows.expand(N // 16, K // 64, 32, 4, 4, 2).reshape(shape)
    cols = cols.expand(N // 16, K // 64, 32, 4, 4, 2).reshape(shape)
    r = torch.arange(8).view(1, 1, -1, 1, 1)
    jj = torch.arange(4).view(1, 1, 1, -1, 1)
    h = torch.arange(2).view(1, 1, 1, 1, -1)
    srows = (st.view(-1, 1, 1, 1, 1) * 16 + r + 8 * h).expand(N // 16, K // 64, 8, 4, 2)
    sblk = (tl.view(1, -1, 1, 1, 1) * 4 + jj).expand(N // 16, K // 64, 8, 4, 2)
    return rows, cols, srows, sblk


def e2m1_codes(v: torch.Tensor) -> torch.Tensor:
    """Round-to-nearest-even e2m1 code (sign in bit 3), saturating at 6."""
    a = v.abs().float()
    bounds = torch.tensor(_BOUNDS, dtype=torch.float32)
    code = torch.bucketize(a, bounds, right=False)            # ties -> lower code
    tie = (code < 7) & (a == bounds[code.clamp(max=6)])
    code = torch.where(tie & (code % 2 == 1), code + 1, code)  # ties -> even code
    return (code | torch.where(v < 0, 8, 0)).to(torch.uint8)


def e2m1_values(codes: torch.Tensor) -> torch.Tensor:
    lut = torch.tensor(E2M1_VALUES, dtype=torch.float32)
    mag = lut[(codes & 7).long()]
    return torch.where((codes & 8) != 0, -mag, mag)


def global_scale(w: torch.Tensor) -> torch.Tensor:
    amax = w.abs().amax().float().reshape(1)
    # tensor / tensor: a true division on every device (CUDA divides by a Python
    # scalar through its reciprocal, which can differ in the last bit)
    gs = amax / torch.full_like(amax, FP4_MAX * E4M3_MAX)
    return torch.where(gs > 0, gs, torch.ones_like(gs))


def block_scales_ref(w: torch.Tensor, gs: torch.Tensor) -> torch.Tensor:
    """e4m3 bytes [N, K/16] (row-major)."""
    N, K = w.shape
    bamax = w.float().abs().view(N, K // 16, 16).amax(-1)
    s = (bamax / FP4_MAX / gs.float()).clamp(max=E4M3_MAX)
    return s.to(torch.float8_e4m3fn).view(torch.uint8)


def quantize_ref(w: torch.Tensor, gs: Optional[torch.Tensor] = None) -> NVFP4Weight:
    """Host restatement of the quantisation kernels (the test oracle)."""
    w = w.detach().cpu()
    N, K = w.shape
    if N % 16 or K % 64:
        raise ValueError(f"nvfp4: N must be a multiple of 16 and K of 64, got {N}x{K}")
    gs = global_scale(w) if gs is None else gs.detach().cpu().float().reshape(1)
    s8 = block_scales_ref(w, gs)
    sf = s8.view(torch.float8_e4m3fn).float()
    denom = (sf * gs).repeat_interleave(16, dim=1)
    v = torch.where(denom > 0, w.float() / denom, torch.zeros_like(denom))
    codes = e2m1_codes(v)
    rows, cols, srows, sblk = _frag_index(N, K)
    nib = codes[rows, cols]                                     # [..., 16, 2]
    q = (nib[..., 0] | (nib[..., 1] << 4)).to(torch.uint8).reshape(-1)
    s = s8[srows, sblk].reshape(-1)
    return NVFP4Weight(q, s, gs, N, K)


def dequantize_ref(w: NVFP4Weight) -> torch.Tensor:
    """fp32 [N, K] = e2m1 * e4m3 * gs, from the fragment-order bytes."""
    N, K = w.N, w.K
    q = w.q.cpu().view(N // 16, K // 64, 32, 16)
    s = w.s.cpu().view(N // 16, K // 64, 8, 4, 2)
    rows, cols, srows, sblk = _frag_index(N, K)
    codes = torch.stack([q & 15, q >> 4], dim=-1)
    vals = torch.empty(N, K, dtype=torch.float32)
    vals[rows.reshape(-1), cols.reshape(-1)] = e2m1_values(codes).reshape(-1)
    sc = torch.empty(N, K // 16, dtype=torch.uint8)
    sc[srows.reshape(-1), sblk.reshape(-1)] = s.reshape(-1)
    sf = sc.view(torch.float8_e4m3fn).float().repeat_interleave(16, dim=1)
    return vals * sf * w.gs.cpu().float()


# ---------------------------------------------------------------- block-scaled rows (tcgen05 mxf4nvf4 format)
# Row-major codes q [rows, K/2] (element 2i in the low nibble of byte i) and e4m3 block
# scales in 512-byte atoms of 128 rows x 4 blocks: atom (row // 128, k // 64), byte
# (row % 32) * 16 + (row // 32 % 4) * 4 + k // 16 % 4 (csrc/nvfp4_bs.cu).
def sf_to_atoms(s8: torch.Tensor) -> torch.Tensor:
    """uint8 [rows, K/16] row-major block scales (rows % 128 == 0) -> the atom layout."""
    rows, nb = s8.shape
    return s8.view(rows // 128, 4, 32, nb // 4, 4).permute(0, 3, 2, 1, 4).reshape(-1).contiguous()


def atoms_to_sf(atoms: torch.Tensor, rows: int, K: int) -> torch.Tensor:
    return atoms.view(rows // 128, K // 64, 32, 4, 4).permute(0, 3, 2, 1, 4).reshape(rows, K // 16)


def quantize_rows_ref(x: torch.Tensor, rows: Optional[int] = None, gs: Optional[torch.Tensor] = None):
    """Host restatement of nvfp4_rows_quantize: (q, scale atoms, per-row gs or empty)."""
    x = x.detach().cpu().float()
    valid, K = x.shape
    rows = rows or (valid + 127) // 128 * 128
    if gs is None:
        amax = x.abs().amax(1)
        gsr = torch.where(amax > 0, amax / torch.full_like(amax, FP4_MAX * E4M3_MAX), torch.ones_like(amax))
    else:
        gsr = gs.detach().cpu().float().reshape(1).expand(valid)
    bam = x.view(valid, K // 16, 16).abs().amax(-1)
    s8 = (bam / FP4_MAX / gsr[:, None]).clamp(max=E4M3_MAX).to(torch.float8_e4m3fn).view(torch.uint8)
    denom = (s8.view(torch.float8_e4m3fn).float() * gsr[:, None]).repeat_interleave(16, dim=1)
    v = torch.where(denom > 0, x / denom, torch.zeros_like(denom))
    codes = e2m1_codes(v)
    q = torch.zeros(rows, K // 2, dtype=torch.uint8)
    q[:valid] = codes[:, 0::2] | (codes[:, 1::2] << 4)
    sp = torch.zeros(rows, K // 16, dtype=torch.uint8)
    sp[:valid] = s8
    g = torch.zeros(rows) if gs is None else torch.empty(0)
    if gs is None:
        g[:valid] = gsr
    return q, sf_to_atoms(sp), g


def dequantize_rows_ref(q: torch.Tensor, atoms: torch.Tensor, gs: torch.Tensor, valid: int) -> torch.Tensor:
    """fp32 [valid, K] from block-scaled rows (gs: per-row [rows] or per-tensor [1])."""
    q = q.cpu()
    rows, K = q.shape[0], q.shape[1] * 2
    codes = torch.stack([q & 15, q >> 4], dim=-1).reshape(rows, K)
    sf = atoms_to_sf(atoms.cpu(), rows, K).view(torch.float8_e4m3fn).float().repeat_interleave(16, dim=1)
    g = gs.cpu().float()
    g = g[:rows].view(rows, 1) if g.numel() > 1 else g.view(1, 1)
    return (e2m1_values(codes) * sf * g)[:valid]


# ---------------------------------------------------------------- public API
def quantize(w: torch.Tensor) -> NVFP4Weight:
    """NVFP4 copy of a 2-D weight [N, K] (N % 16 == 0, K % 64 == 0), on w's device."""
    if w.dim() != 2:
        raise ValueError("nvfp4: 2-D weight expected")
    if not w.is_cuda:
        return quantize_ref(w)
    w = w.to(torch.bfloat16).contiguous()
    gs = global_scale(w)
    q, s = ops.native().nvfp4_quantize(w, gs)
    qr = sa = None
    N, K = w.shape
    if N % 128 == 0 and K % 256 == 0 and os.environ.get("VRM_NVFP4_PREFILL", "w4a4") == "w4a4":
        qr, sa, _ = ops.native().nvfp4_rows_quantize(w, N, gs)
    return NVFP4Weight(q, s, gs, N, K, qr, sa)


def quantizable(w: torch.Tensor) -> bool:
    return isinstance(w, torch.Tensor) and w.dim() == 2 and w.shape[0] % 16 == 0 and w.shape[1] % 64 == 0


def quantize_model_weights(weights: Dict[str, torch.Tensor], cfg=None, keys=QUANTIZED_KEYS,
                           include_lm_head: bool = False) -> Dict[str, object]:
    """Replaces every layer projection (and optionally lm_head) with its NVFP4 copy;
    embeddings, norms, biases and MoE experts stay bf16."""
    out = dict(weights)
    for name, w in weights.items():
        leaf = name.rsplit(".", 1)[-1]
        if (leaf in keys or (include_lm_head and name == "lm_head")) and quantizable(w):
            out[name] = quantize(w)
    return out


class DirectFP4Linear:
    """A linear layer over an NVFP4 weight: y = x @ W'^T (+ bias).

    Reference parity: core/nvfp4_direct.py DirectFP4Linear (a torch.nn.Module holding
    w_qdata / w_scale / w_per_tensor_scale)."""

    def __init__(self, weight: torch.Tensor, bias: Optional[torch.Tensor] = None):
        self.weight = weight if isinstance(weight, NVFP4Weight) else quantize(weight)
        self.bias = bias

    @classmethod
    def from_linear(cls, linear) -> "DirectFP4Linear":
        return cls(linear.weight.detach().to(torch.bfloat16), None if linear.bias is None else
                   linear.bias.detach().to(torch.bfloat16))

    @property
    def in_features(self) -> int:
        return self.weight.K

    @property
    def out_features(self) -> int:
        return self.weight.N

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        shp = x.shape
        y = self.weight.linear(x.reshape(-1, shp[-1]).to(torch.bfloat16).contiguous(), self.bias)
        return y.view(*shp[:-1], self.weight.N)
