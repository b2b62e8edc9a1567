"""Four-bit KV rows: the format of `uint8` KV pools and its host-side oracle.

A row of D values (one token, one KV head, K or V) is stored in D/2 + D/8 bytes:

* bytes [0, D/2): codes, element 2i in the low nibble of byte i, 2i+1 in the high one;
* bytes [D/2, D/2 + D/8): one (scale, min) pair of fp16 per 32-element group.

value = code * scale + min, with scale = (max - min) / 15 and min rounded to fp16 first
and code = clamp(round_half_even((x - min) / scale), 0, 15) computed against those
rounded values (a constant group stores scale = 2^-14).  The CUDA kernels
(RoPE + KV write, and the fused write inside decode attention) store exactly this and
the decode / prefill kernels dequantise it into the bf16 MMA tile in shared memory.

Reference parity: the q4 page variant of csrc/paged_attention_kernel.cu (4-bit codes
with a per-group scale and zero point, dequantised in the attention loop); here the
group carries its minimum instead of a zero point so that one fp16 pair covers any
range without overflow, and groups are 32 dims to match the MMA's 16-byte chunks.
"""
from __future__ import annotations

import torch

GROUP = 32
_TINY_SCALE = 2.0 ** -14


def row_bytes(head_dim: int) -> int:
    """Bytes per stored row (80 for head_dim 128, 40 for 64)."""
    if head_dim % GROUP:
        raise ValueError(f"four-bit rows need head_dim % {GROUP} == 0, got {head_dim}")
    return head_dim // 2 + head_dim // 8


def head_dim_of(row: int) -> int:
    """Inverse of `row_bytes`."""
    return row * 8 // 5


def quantize(x: torch.Tensor) -> torch.Tensor:
    """[..., D] float -> [..., D/2 + D/8] uint8 four-bit rows."""
    D = x.shape[-1]
    lead = x.shape[:-1]
    g = x.float().reshape(*lead, D // GROUP, GROUP)
    mn, mx = g.amin(-1), g.amax(-1)
    hs = ((mx - mn) / 15.0).half()
    hs = torch.where(hs.float() > 0, hs, torch.full_like(hs, _TINY_SCALE))
    hm = mn.half()
    s, m = hs.float().unsqueeze(-1), hm.float().unsqueeze(-1)
    code = torch.clamp(torch.round((g - m) / s), 0, 15).to(torch.uint8).reshape(*lead, D)
    packed = code[..., 0::2] | (code[..., 1::2] << 4)
    sm = torch.stack([hs, hm], dim=-1).reshape(*lead, D // GROUP * 2).contiguous().view(torch.uint8)
    return torch.cat([packed, sm], dim=-1)


def dequantize(rows: torch.Tensor, head_dim: int = 0) -> torch.Tensor:
    """[..., D/2 + D/8] uint8 -> [..., D] float32."""
    D = head_dim or head_dim_of(rows.shape[-1])
    lead = rows.shape[:-1]
    codes = rows[..., : D // 2]
    lo, hi = (codes & 15).float(), (codes >> 4).float()
    q = torch.stack([lo, hi], dim=-1).reshape(*lead, D // GROUP, GROUP)
    sm = rows[..., D // 2:].contiguous().view(torch.float16).float().reshape(*lead, D // GROUP, 2)
    return (q * sm[..., :1] + sm[..., 1:]).reshape(*lead, D)
