"""Physical paged KV pool of one rank / pipeline stage.

Layout ``[num_pages, num_layers, 2, kv_heads, page_size, head_dim]`` (row bytes for uint8): a page holds
`page_size` tokens of every layer, so one page is one contiguous block (3 MiB for the
Qwen2.5-14B shape: 16 tok x 48 layers x 8 heads x 128 dim x bf16 x K,V).  That makes a
page the unit of migration between GPUs and of spill to host/NVMe, and the
(page, layer, k|v, head) chunk of page_size x head_dim elements is contiguous, which
is what the attention kernels stream.

fp8 pools store e4m3 values with one fp32 scale per (layer, k|v, kv_head).  uint8
pools store four-bit rows (`kv.q4`): the last dimension is the row's byte count,
head_dim * 5 / 8, and a page takes 5/16 of the bf16 page's bytes.  int8 pools store
TurboQuant records (`kv.turboquant`, 64 bytes per 128-dim row, 1/4 of bf16).

Reference parity: the pool tensor of core/paged_attention.py:277-351 (same page
shape and bytes/page, core/paged_attention.py:107-111).
"""
from __future__ import annotations

from dataclasses import dataclass
from typing import Optional

import torch

PAGE_SIZE = 16


def kv_dtype_from_str(s: str) -> torch.dtype:
    s = (s or "bf16").lower()
    if s in ("bf16", "bfloat16", "auto"):
        return torch.bfloat16
    if s in ("fp8", "fp8_e4m3", "e4m3", "float8_e4m3fn"):
        return torch.float8_e4m3fn
    if s in ("fp32", "float32"):
        return torch.float32
    if s in ("q4", "int4", "4bit", "uint8"):
        return torch.uint8
    if s in ("tq", "turboquant", "int8"):
        return torch.int8
    raise ValueError(f"unsupported kv cache dtype {s!r}")


@dataclass
class KVPoolSpec:
    num_pages: int
    num_layers: int
    kv_heads: int
    head_dim: int
    page_size: int = PAGE_SIZE
    dtype: torch.dtype = torch.bfloat16

    @property
    def row(self) -> int:
        """Last dimension of the pool tensor: head_dim, or the four-bit row's bytes."""
        if self.dtype == torch.uint8:
            from .q4 import row_bytes
            return row_bytes(self.head_dim)
        if self.dtype == torch.int8:
            if self.head_dim != 128:
                raise ValueError("TurboQuant KV pages need head_dim 128")
            return 64
        return self.head_dim

    @property
    def bytes_per_page(self) -> int:
        el = torch.empty(0, dtype=self.dtype).element_size()
        return 2 * self.num_layers * self.kv_heads * self.page_size * self.row * el

    @staticmethod
    def pages_for_budget(budget_bytes: int, num_layers: int, kv_heads: int, head_dim: int,
                         dtype: torch.dtype = torch.bfloat16, page_size: int = PAGE_SIZE) -> int:
        spec = KVPoolSpec(1, num_layers, kv_heads, head_dim, page_size, dtype)
        return max(1, budget_bytes // spec.bytes_per_page)


class KVPool:
    """Owns the page tensor (and fp8 scales) on one device."""

    def __init__(self, spec: KVPoolSpec, device="cpu", kv_scale: Optional[torch.Tensor] = None):
        self.spec = spec
        self.device = torch.device(device)
        shape = (spec.num_pages, spec.num_layers, 2, spec.kv_heads, spec.page_size, spec.row)
        # zero-initialised: stale slots past a sequence's length are finite
        self.cache = torch.zeros(shape, dtype=spec.dtype, device=self.device)
        self.is_fp8 = spec.dtype == torch.float8_e4m3fn
        # TurboQuant pages (int8 pool of 64-byte records): the compressor's rotation signs
        # and JL matrix on the pool's device
        self.is_tq = spec.dtype == torch.int8
        self.tq = None
        if self.is_tq:
            from .turboquant import KVCacheCompressor
            self.tq = KVCacheCompressor(head_dim=128).to(self.device)
        if self.is_fp8:
            if kv_scale is None:
                kv_scale = torch.ones(spec.num_layers, 2, spec.kv_heads, dtype=torch.float32)
            self.kv_scale = kv_scale.to(self.device, torch.float32).contiguous()
        else:
            self.kv_scale = None

    @property
    def num_pages(self) -> int:
        return self.spec.num_pages

    def page(self, idx: int) -> torch.Tensor:
        return self.cache[idx]

    def set_kv_scale(self, scale: torch.Tensor) -> None:
        """Per-(layer, k|v, kv_head) fp8 scales, e.g. from `calibrate_kv_scale`."""
        if self.kv_scale is not None:
            self.kv_scale.copy_(scale.to(self.kv_scale.device, torch.float32).view_as(self.kv_scale))

    def nbytes(self) -> int:
        return self.cache.numel() * self.cache.element_size()


def calibrate_kv_scale(k_amax: torch.Tensor, v_amax: torch.Tensor, margin: float = 1.25) -> torch.Tensor:
    """Per-head fp8 scales from observed |k|, |v| maxima ([layers, kv_heads] each):
    scale = amax * margin / 448 so that calibrated values use the e4m3 range."""
    s = torch.stack([k_amax, v_amax], dim=1).float() * margin / 448.0
    return torch.clamp(s, min=1e-6)
