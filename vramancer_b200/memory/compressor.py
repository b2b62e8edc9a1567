"""Byte / tensor compression and weight-only integer quantisation for cold tiers.

Codecs: zlib (always), lzma (stdlib), plus zstd / lz4 when importable.  Tensors are
compressed as raw bytes with dtype and shape kept beside them.  int4 weight packing:
per-group (default 128) asymmetric scale + zero point, two values per byte.

Reference parity: core/compressor.py:48-273 (Compressor: compress_bytes /
decompress_bytes, compress_tensor / decompress_tensor, compress_module,
quantize_dynamic_int8, quantize_weights_int4 / dequantize_int4).
"""
from __future__ import annotations

import lzma
import zlib
from typing import Any, Dict, Optional, Tuple

import torch

try:  # optional codecs
    import zstandard as _zstd  # type: ignore
except Exception:  # noqa: BLE001
    _zstd = None
try:
    import lz4.frame as _lz4  # type: ignore
except Exception:  # noqa: BLE001
    _lz4 = None

_DT = {str(d): d for d in (torch.float32, torch.float16, torch.bfloat16, torch.int64, torch.int32, torch.int16,
                           torch.int8, torch.uint8, torch.bool, torch.float64)}


def available_codecs():
    out = ["zlib", "lzma", "none"]
    if _zstd is not None:
        out.append("zstd")
    if _lz4 is not None:
        out.append("lz4")
    return out


class Compressor:
    def __init__(self, codec: str = "auto", level: int = 3):
        if codec == "auto":
            codec = "zstd" if _zstd is not None else ("lz4" if _lz4 is not None else "zlib")
        if codec not in available_codecs():
            raise ValueError(f"codec {codec!r} unavailable (have {available_codecs()})")
        self.codec, self.level = codec, level
        self.bytes_in = 0
        self.bytes_out = 0

    # ---------------------------------------------------------------- bytes
    def compress_bytes(self, data: bytes) -> bytes:
        self.bytes_in += len(data)
        if self.codec == "zlib":
            out = zlib.compress(data, self.level)
        elif self.codec == "lzma":
            out = lzma.compress(data, preset=min(self.level, 9))
        elif self.codec == "zstd":
            out = _zstd.ZstdCompressor(level=self.level).compress(data)
        elif self.codec == "lz4":
            out = _lz4.compress(data)
        else:
            out = bytes(data)
        self.bytes_out += len(out)
        return out

    def decompress_bytes(self, data: bytes) -> bytes:
        if self.codec == "zlib":
            return zlib.decompress(data)
        if self.codec == "lzma":
            return lzma.decompress(data)
        if self.codec == "zstd":
            return _zstd.ZstdDecompressor().decompress(data)
        if self.codec == "lz4":
            return _lz4.decompress(data)
        return bytes(data)

    @property
    def ratio(self) -> float:
        return self.bytes_in / self.bytes_out if self.bytes_out else 1.0

    # ---------------------------------------------------------------- tensors
    def compress_tensor(self, t: torch.Tensor) -> Dict[str, Any]:
        h = t.detach().to("cpu").contiguous()
        raw = h.view(torch.uint8).numpy().tobytes() if h.numel() else b""
        return {"codec": self.codec, "dtype": str(h.dtype), "shape": list(h.shape), "data": self.compress_bytes(raw)}

    def decompress_tensor(self, d: Dict[str, Any], device: str = "cpu") -> torch.Tensor:
        raw = self.decompress_bytes(d["data"]) if d["codec"] == self.codec else Compressor(d["codec"]).decompress_bytes(d["data"])
        dt = _DT[d["dtype"]]
        if not raw:
            return torch.empty(d["shape"], dtype=dt, device=device)
        t = torch.frombuffer(bytearray(raw), dtype=torch.uint8).view(dt).reshape(d["shape"])
        return t.to(device)

    def compress_module(self, state: Dict[str, torch.Tensor]) -> Dict[str, Any]:
        return {k: self.compress_tensor(v) for k, v in state.items()}

    def decompress_module(self, data: Dict[str, Any], device: str = "cpu") -> Dict[str, torch.Tensor]:
        return {k: self.decompress_tensor(v, device) for k, v in data.items()}

    # ---------------------------------------------------------------- weight quantisation
    @staticmethod
    def quantize_weights_int4(w: torch.Tensor, group: int = 128) -> Tuple[torch.Tensor, torch.Tensor, torch.Tensor]:
        """(packed uint8 [N, K/2], scale fp32 [N, K/group], zero fp32 [N, K/group]);
        q = clamp(round(w / scale) + zero, 0, 15), low nibble = even column."""
        N, K = w.shape
        if K % group or K % 2:
            raise ValueError("K must be a multiple of the group size and of 2")
        g = w.float().view(N, K // group, group)
        lo, hi = g.amin(-1, keepdim=True), g.amax(-1, keepdim=True)
        scale = ((hi - lo) / 15.0).clamp(min=1e-8)
        zero = torch.round(-lo / scale)
        q = torch.clamp(torch.round(g / scale) + zero, 0, 15).to(torch.uint8).view(N, K)
        packed = q[:, 0::2] | (q[:, 1::2] << 4)
        return packed.contiguous(), scale.squeeze(-1), zero.squeeze(-1)

    @staticmethod
    def dequantize_int4(packed: torch.Tensor, scale: torch.Tensor, zero: torch.Tensor, group: int = 128,
                        dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        N, K2 = packed.shape
        q = torch.empty(N, K2 * 2, dtype=torch.float32, device=packed.device)
        q[:, 0::2] = (packed & 15).float()
        q[:, 1::2] = (packed >> 4).float()
        g = q.view(N, -1, group)
        return ((g - zero.unsqueeze(-1)) * scale.unsqueeze(-1)).view(N, -1).to(dtype)

    @staticmethod
    def quantize_dynamic_int8(w: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """Per-row symmetric int8: (q int8 [N, K], scale fp32 [N])."""
        scale = w.float().abs().amax(-1).clamp(min=1e-8) / 127.0
        q = torch.clamp(torch.round(w.float() / scale[:, None]), -127, 127).to(torch.int8)
        return q, scale

    @staticmethod
    def dequantize_int8(q: torch.Tensor, scale: torch.Tensor, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        return (q.float() * scale[:, None]).to(dtype)

    def stats(self) -> Dict[str, float]:
        return {"codec": self.codec, "bytes_in": self.bytes_in, "bytes_out": self.bytes_out, "ratio": self.ratio}
