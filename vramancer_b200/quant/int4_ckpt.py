"""GPTQ and AWQ integer-quantised checkpoints: unpacking and dequantisation.

The reference serves these through Hugging Face (`HuggingFaceBackend` with the GPTQ /
AWQ integrations).  Here the loader reads their tensors directly and dequantises each
linear layer once, at load time, into the dense layout of the rest of the engine
(bf16 on the GPU); `-q fp8` / `-q nvfp4` then re-quantise into the formats the B200
tensor cores run.  Integer codes with per-group zero points are not values of the
e2m1 / e4m3 grids, so a direct transcoding would not be exact.

Layouts (per linear layer with K inputs and N outputs, b bits, 32 / b codes per int32,
code j of a word at bits [b*j, b*j + b)):
  GPTQ  qweight int32 [K / (32/b), N]  code j of word (r, n) is row r * 32/b + j
        qzeros  int32 [G, N / (32/b)]  code j of word (g, c) is column c * 32/b + j
        scales  fp16  [G, N]; g_idx int32 [K] (the group of each input row; absent:
        row // group_size).  w[n, k] = scales[g, n] * (q[k, n] - z[g, n] - o), g = g_idx[k],
        o = 1 for checkpoint_format "gptq" (zeros stored minus one), 0 for "gptq_v2".
  AWQ   qweight int32 [K, N / 8], qzeros int32 [G, N / 8] (the "gemm" version, 4-bit):
        code j of word (r, c) is column 8c + (0, 2, 4, 6, 1, 3, 5, 7)[j];
        scales fp16 [G, N]; w[n, k] = scales[g, n] * (q[k, n] - z[g, n]), g = k // group.

Reference parity: core/backends.py (HuggingFaceBackend load with quantization="gptq" /
"awq"; the `-q gptq|awq` CLI choices of vramancer/main.py).
"""
from __future__ import annotations

from typing import Dict, Optional, Sequence

import torch

AWQ_ORDER = (0, 2, 4, 6, 1, 3, 5, 7)      # column offset held by code j of an AWQ word


class UnsupportedQuantization(ValueError):
    pass


def _codes(words: torch.Tensor, bits: int) -> torch.Tensor:
    """int32 [..., W] -> int64 [..., W, 32 / bits], code j at bits [bits*j, bits*j + bits)."""
    per = 32 // bits
    w = words.to(torch.int64) & 0xFFFFFFFF
    shifts = torch.arange(per, dtype=torch.int64) * bits
    return (w.unsqueeze(-1) >> shifts) & ((1 << bits) - 1)


def unpack_rows(qweight: torch.Tensor, bits: int = 4) -> torch.Tensor:
    """[K / per, N] words -> [K, N] codes; code j of word (r, n) is row r * per + j."""
    c = _codes(qweight, bits)                       # [R, N, per]
    return c.permute(0, 2, 1).reshape(-1, qweight.shape[1])


def unpack_cols(q: torch.Tensor, bits: int = 4, order: Optional[Sequence[int]] = None) -> torch.Tensor:
    """[R, N / per] words -> [R, N] codes; code j of word (r, c) is column c * per +
    order[j] (order = identity when None)."""
    c = _codes(q, bits)                             # [R, C, per]
    if order is not None:
        inv = [0] * len(order)
        for j, col in enumerate(order):
            inv[col] = j
        c = c[..., list(inv)]                       # column offset o comes from code inv[o]
    return c.reshape(q.shape[0], -1)


def gptq_dequantize(qweight: torch.Tensor, qzeros: torch.Tensor, scales: torch.Tensor,
                    g_idx: Optional[torch.Tensor] = None, *, bits: int = 4, group_size: int = 128,
                    zero_offset: int = 1) -> torch.Tensor:
    """Dense [N, K] fp32 weight of one GPTQ linear layer."""
    if 32 % bits:
        raise UnsupportedQuantization(f"GPTQ with {bits}-bit codes (only 2, 4 and 8 pack into int32 words)")
    q = unpack_rows(qweight, bits)                  # [K, N]
    K, N = q.shape
    z = unpack_cols(qzeros, bits)[:, :N]            # [G, N]
    if g_idx is None or g_idx.numel() == 0:
        gs = K if group_size is None or group_size <= 0 else group_size
        g = torch.arange(K) // gs
    else:
        g = g_idx.to(torch.int64)
    w = (q - z[g] - zero_offset).to(torch.float32) * scales.to(torch.float32)[g]
    return w.t().contiguous()


def awq_dequantize(qweight: torch.Tensor, qzeros: Optional[torch.Tensor], scales: torch.Tensor, *, bits: int = 4,
                   group_size: int = 128) -> torch.Tensor:
    """Dense [N, K] fp32 weight of one AWQ ("gemm" layout) linear layer."""
    if bits != 4:
        raise UnsupportedQuantization(f"AWQ with {bits}-bit codes (4-bit only)")
    q = unpack_cols(qweight, bits, AWQ_ORDER)       # [K, N]
    K, N = q.shape
    gs = K if group_size is None or group_size <= 0 else group_size
    g = torch.arange(K) // gs
    z = unpack_cols(qzeros, bits, AWQ_ORDER)[:, :N][g] if qzeros is not None else 0
    w = (q - z).to(torch.float32) * scales.to(torch.float32)[g]
    return w.t().contiguous()


LEAVES = ("qweight", "qzeros", "scales", "g_idx")


def check_config(qc: Dict) -> str:
    """The quant method of an HF `quantization_config` this loader reads ("gptq" or
    "awq"), or UnsupportedQuantization."""
    method = str(qc.get("quant_method", "")).lower()
    if method == "gptq":
        fmt = str(qc.get("checkpoint_format", "gptq")).lower()
        if fmt not in ("gptq", "gptq_v2"):
            raise UnsupportedQuantization(f"GPTQ checkpoint_format {fmt!r} (gptq or gptq_v2)")
        if int(qc.get("bits", 4)) not in (2, 4, 8):
            raise UnsupportedQuantization(f"GPTQ with {qc.get('bits')}-bit codes")
        return method
    if method == "awq":
        ver = str(qc.get("version", "gemm")).lower()
        if ver != "gemm" or int(qc.get("bits", qc.get("w_bit", 4))) != 4:
            raise UnsupportedQuantization(f"AWQ version {ver!r} / {qc.get('bits', qc.get('w_bit'))} bits "
                                          "(the 4-bit gemm layout)")
        return method
    raise UnsupportedQuantization(f"quant_method {method!r}")


def dequantize_module(qc: Dict, parts: Dict[str, torch.Tensor]) -> torch.Tensor:
    """Dense [N, K] fp32 weight of one linear layer from its checkpoint tensors
    (qweight, qzeros, scales, optional g_idx) and the checkpoint's quantization_config."""
    method = check_config(qc)
    gs = int(qc.get("group_size", qc.get("q_group_size", 128)))
    if method == "gptq":
        off = 0 if str(qc.get("checkpoint_format", "gptq")).lower() == "gptq_v2" else 1
        return gptq_dequantize(parts["qweight"], parts["qzeros"], parts["scales"], parts.get("g_idx"),
                               bits=int(qc.get("bits", 4)), group_size=gs, zero_offset=off)
    return awq_dequantize(parts["qweight"], parts.get("qzeros"), parts["scales"], group_size=gs)
