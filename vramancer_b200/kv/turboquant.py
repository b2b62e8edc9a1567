"""TurboQuant KV compression: randomized Hadamard rotation + PolarQuant angles + 1-bit
QJL residual sketch (arXiv:2504.19874, PolarQuant arXiv:2502.02617, QJL).

One key / value vector of D = 2^n dims becomes a fixed 64-byte record (D = 128,
3-bit angles, 64 JL signs):
  bytes  0..47   127 angle indices, 3 bits each, in the order level 0 (64 angles),
                 level 1 (32), ..., level 6 (1); angle i at bits [3i, 3i+3) of the
                 little-endian bit stream (slot 127 is padding)
  bytes 48..49   final radius (fp16) = norm of the rotated vector
  bytes 50..57   sign(P r) for the m = D/2 JL projections of the residual r
                 (bit j of byte 50 + j/8 = projection j)
  bytes 58..59   ||r|| (fp16)
  bytes 60..63   zero
i.e. 4 bits/dim versus 16 for bf16.

Encoding: x_rot = H(x * s) / sqrt(D) (s: fixed random signs); pairs (a, b) of each
level give angle atan2(b, a) and radius sqrt(a^2 + b^2); level 0 angles are in
[-pi, pi], deeper levels (radii are >= 0) in [0, pi/2]; each range is cut into
2^bits equal bins, decoded at the bin centre.  The residual r = x_rot - decode(x_rot)
is sketched as sign(P r) with P ~ N(0, 1/m) of shape [m, D].  Scores use the
asymmetric estimator <q, k> ~= <q_rot, k_hat_rot> + sqrt(pi/2)/m * ||r|| * <P q_rot, sign(P r)>.

The torch implementation here is the CPU path and the oracle of the CUDA kernels
(csrc/turboquant.cu: one warp per vector).

Reference parity: core/kv_quantizer.py:207-566 (KVCacheCompressor: compress,
decompress, attention_score, sparse_v_attend, bits_per_dim), core/turboquant_cache.py
(TurboQuantCache, an HF Cache with a full-precision window of recent tokens),
csrc/turboquant_kernel.cu (fused compress / decompress).  The reference scores the
unrotated q against rotated keys in one GPU path (core/turboquant_cuda.py:238-253); here
q is always rotated.
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Sequence, Tuple

import torch

RECORD_BYTES = 64


def _fwht(x: torch.Tensor) -> torch.Tensor:
    """Orthonormal Walsh-Hadamard transform over the last dim (power of two)."""
    d = x.shape[-1]
    y = x.reshape(-1, d).clone()
    h = 1
    while h < d:
        y = y.view(-1, d // (2 * h), 2, h)
        a, b = y[:, :, 0, :], y[:, :, 1, :]
        y = torch.stack([a + b, a - b], dim=2).reshape(-1, d)
        h *= 2
    return (y / math.sqrt(d)).view(x.shape)


class KVCacheCompressor:
    """Compress / decompress [..., D] key or value vectors (D = 128 with the default
    record layout; any power of two up to 256 with 3-bit angles)."""

    def __init__(self, head_dim: int = 128, bits_per_angle: int = 3, qjl_dim: Optional[int] = None, seed: int = 0,
                 device="cpu"):
        if head_dim & (head_dim - 1) or head_dim < 4:
            raise ValueError("head_dim must be a power of two >= 4")
        self.head_dim = head_dim
        self.bits = bits_per_angle
        self.levels = int(math.log2(head_dim))
        self.n_angles = head_dim - 1
        self.qjl_dim = qjl_dim or head_dim // 2
        g = torch.Generator().manual_seed(seed)
        self.signs = (torch.randint(0, 2, (head_dim,), generator=g).float() * 2 - 1).to(device)
        self.jl = (torch.randn(self.qjl_dim, head_dim, generator=g) / math.sqrt(self.qjl_dim)).to(device)
        self.angle_bytes = (self.n_angles * self.bits + 7) // 8
        self.sign_bytes = (self.qjl_dim + 7) // 8
        self.record_bytes = ((self.angle_bytes + 2 + self.sign_bytes + 2) + 15) // 16 * 16

    def to(self, device) -> "KVCacheCompressor":
        self.signs, self.jl = self.signs.to(device), self.jl.to(device)
        return self

    @property
    def bits_per_dim(self) -> float:
        return self.record_bytes * 8 / self.head_dim

    # ---------------------------------------------------------------- rotation
    def rotate(self, x: torch.Tensor) -> torch.Tensor:
        return _fwht(x.float() * self.signs)

    def unrotate(self, x: torch.Tensor) -> torch.Tensor:
        return _fwht(x.float()) * self.signs

    # ---------------------------------------------------------------- polar
    def _ranges(self, level: int) -> Tuple[float, float]:
        return (-math.pi, math.pi) if level == 0 else (0.0, math.pi / 2)

    def polar_encode(self, xr: torch.Tensor) -> Tuple[torch.Tensor, torch.Tensor]:
        """(angle indices [..., D-1] uint8, radius [...]) of rotated vectors."""
        nb = 1 << self.bits
        cur = xr
        idx = []
        for level in range(self.levels):
            p = cur.reshape(*cur.shape[:-1], -1, 2)
            a, b = p[..., 0], p[..., 1]
            ang = torch.atan2(b, a)
            lo, hi = self._ranges(level)
            q = torch.clamp(torch.floor((ang - lo) / (hi - lo) * nb), 0, nb - 1)
            idx.append(q.to(torch.uint8))
            cur = torch.sqrt(a * a + b * b)
        return torch.cat(idx, dim=-1), cur.squeeze(-1)

    def polar_decode(self, idx: torch.Tensor, radius: torch.Tensor) -> torch.Tensor:
        nb = 1 << self.bits
        cur = radius.float().unsqueeze(-1)
        offs = [0]
        for level in range(self.levels):
            offs.append(offs[-1] + (self.head_dim >> (level + 1)))
        for level in range(self.levels - 1, -1, -1):
            lo, hi = self._ranges(level)
            q = idx[..., offs[level]:offs[level + 1]].float()
            ang = lo + (q + 0.5) * (hi - lo) / nb
            a, b = cur * torch.cos(ang), cur * torch.sin(ang)
            cur = torch.stack([a, b], dim=-1).reshape(*a.shape[:-1], -1)
        return cur

    # ---------------------------------------------------------------- records
    def _pack_angles(self, idx: torch.Tensor) -> torch.Tensor:
        n = idx.shape[:-1]
        bits = ((idx.long().unsqueeze(-1) >> torch.arange(self.bits, device=idx.device)) & 1).reshape(*n, -1)
        pad = self.angle_bytes * 8 - bits.shape[-1]
        if pad:
            bits = torch.cat([bits, torch.zeros(*n, pad, dtype=bits.dtype, device=bits.device)], dim=-1)
        w = (1 << torch.arange(8, device=idx.device)).long()
        return (bits.reshape(*n, -1, 8) * w).sum(-1).to(torch.uint8)

    def _unpack_angles(self, b: torch.Tensor) -> torch.Tensor:
        n = b.shape[:-1]
        bits = ((b.long().unsqueeze(-1) >> torch.arange(8, device=b.device)) & 1).reshape(*n, -1)
        bits = bits[..., :self.n_angles * self.bits].reshape(*n, self.n_angles, self.bits)
        return (bits * (1 << torch.arange(self.bits, device=b.device))).sum(-1).to(torch.uint8)

    def _pack_signs(self, s: torch.Tensor) -> torch.Tensor:
        n = s.shape[:-1]
        w = (1 << torch.arange(8, device=s.device)).long()
        return (s.long().reshape(*n, -1, 8) * w).sum(-1).to(torch.uint8)

    def _unpack_signs(self, b: torch.Tensor) -> torch.Tensor:
        return ((b.long().unsqueeze(-1) >> torch.arange(8, device=b.device)) & 1).reshape(*b.shape[:-1], -1)

    def compress(self, x: torch.Tensor) -> torch.Tensor:
        """[..., D] -> uint8 records [..., record_bytes]."""
        if x.is_cuda and self.head_dim == 128 and self.bits == 3 and self.qjl_dim == 64:
            from .. import ops
            return ops.native().tq_compress(x.contiguous(), self.signs.to(x.device), self.jl.to(x.device))
        xr = self.rotate(x)
        idx, rad = self.polar_encode(xr)
        rad16 = rad.to(torch.float16)
        rec = self.polar_decode(idx, rad16.float())
        r = xr - rec
        s = (r @ self.jl.t() > 0)
        nrm = torch.linalg.vector_norm(r, dim=-1).to(torch.float16)
        out = torch.zeros(*x.shape[:-1], self.record_bytes, dtype=torch.uint8, device=x.device)
        a = self.angle_bytes
        out[..., :a] = self._pack_angles(idx)
        out[..., a:a + 2] = rad16.unsqueeze(-1).view(torch.uint8)
        out[..., a + 2:a + 2 + self.sign_bytes] = self._pack_signs(s)
        out[..., a + 2 + self.sign_bytes:a + 4 + self.sign_bytes] = nrm.unsqueeze(-1).view(torch.uint8)
        return out

    def _fields(self, rec: torch.Tensor):
        a = self.angle_bytes
        idx = self._unpack_angles(rec[..., :a])
        rad = rec[..., a:a + 2].contiguous().view(torch.float16).squeeze(-1)
        sg = self._unpack_signs(rec[..., a + 2:a + 2 + self.sign_bytes])
        nrm = rec[..., a + 2 + self.sign_bytes:a + 4 + self.sign_bytes].contiguous().view(torch.float16).squeeze(-1)
        return idx, rad, sg, nrm

    def decompress_rotated(self, rec: torch.Tensor) -> torch.Tensor:
        idx, rad, _, _ = self._fields(rec)
        return self.polar_decode(idx, rad.float())

    def decompress(self, rec: torch.Tensor, dtype: torch.dtype = torch.bfloat16) -> torch.Tensor:
        """Records -> [..., D] vectors (polar part only; the QJL sketch refines scores)."""
        if rec.is_cuda and self.head_dim == 128 and self.bits == 3 and self.qjl_dim == 64:
            from .. import ops
            return ops.native().tq_decompress(rec.contiguous(), self.signs.to(rec.device)).to(dtype)
        return self.unrotate(self.decompress_rotated(rec)).to(dtype)

    # ---------------------------------------------------------------- attention on records
    def attention_score(self, q: torch.Tensor, rec: torch.Tensor, qjl: bool = True) -> torch.Tensor:
        """q [..., Q, D], records [..., N, R] -> scores [..., Q, N] ~= q . k."""
        qr = self.rotate(q)
        idx, rad, sg, nrm = self._fields(rec)
        khat = self.polar_decode(idx, rad.float())
        s = qr @ khat.transpose(-1, -2)
        if qjl:
            qp = qr @ self.jl.t()
            sgn = sg.float() * 2 - 1
            s = s + math.sqrt(math.pi / 2) / self.qjl_dim * (qp @ sgn.transpose(-1, -2)) * nrm.float().unsqueeze(-2)
        return s

    def sparse_v_attend(self, q: torch.Tensor, k_rec: torch.Tensor, v_rec: torch.Tensor, scale: float,
                        keep: float = 0.1, min_keep: int = 16) -> torch.Tensor:
        """softmax(q k^T * scale) v, decompressing only the values of the top `keep`
        share of tokens by weight (the rest carry negligible mass).  q [Q, D],
        records [N, R] -> [Q, D]."""
        w = torch.softmax(self.attention_score(q, k_rec) * scale, dim=-1)
        n = w.shape[-1]
        k = max(min(n, min_keep), int(math.ceil(keep * n)))
        top = torch.topk(w, k, dim=-1)
        idx = top.indices
        v = self.decompress(v_rec[idx.reshape(-1)], torch.float32).view(*idx.shape, -1)
        wk = top.values / top.values.sum(-1, keepdim=True)
        return (wk.unsqueeze(-1) * v).sum(-2)


class TurboQuantCache:
    """Per-layer K/V store for HF-style decoding: the most recent `window` tokens stay
    in full precision, older ones are kept as TurboQuant records and decompressed on
    read.  update(k, v, layer) appends [B, H, T, D] states and returns the full K / V.

    Works with transformers' Cache protocol through `as_hf_cache()`."""

    def __init__(self, head_dim: int = 128, window: int = 128, bits_per_angle: int = 3, seed: int = 0):
        self.comp = KVCacheCompressor(head_dim, bits_per_angle, seed=seed)
        self.window = window
        self.recent: Dict[int, List[torch.Tensor]] = {}
        self.packed: Dict[int, List[Optional[torch.Tensor]]] = {}

    def update(self, k: torch.Tensor, v: torch.Tensor, layer: int) -> Tuple[torch.Tensor, torch.Tensor]:
        if self.comp.signs.device != k.device:
            self.comp.to(k.device)
        rk, rv = self.recent.get(layer, [None, None])
        rk = k if rk is None else torch.cat([rk, k], dim=-2)
        rv = v if rv is None else torch.cat([rv, v], dim=-2)
        pk, pv = self.packed.get(layer, [None, None])
        over = rk.shape[-2] - self.window
        if over > 0:
            ck, cv = self.comp.compress(rk[..., :over, :]), self.comp.compress(rv[..., :over, :])
            pk = ck if pk is None else torch.cat([pk, ck], dim=-2)
            pv = cv if pv is None else torch.cat([pv, cv], dim=-2)
            rk, rv = rk[..., over:, :], rv[..., over:, :]
        self.recent[layer] = [rk, rv]
        self.packed[layer] = [pk, pv]
        if pk is None:
            return rk, rv
        dk = self.comp.decompress(pk, rk.dtype)
        dv = self.comp.decompress(pv, rv.dtype)
        return torch.cat([dk, rk], dim=-2), torch.cat([dv, rv], dim=-2)

    def get_seq_length(self, layer: int = 0) -> int:
        rk = self.recent.get(layer, [None])[0]
        pk = self.packed.get(layer, [None])[0]
        return (0 if rk is None else rk.shape[-2]) + (0 if pk is None else pk.shape[-2])

    def memory_bytes(self) -> Dict[str, int]:
        full = sum(t.numel() * t.element_size() for kv in self.recent.values() for t in kv if t is not None)
        comp = sum(t.numel() for kv in self.packed.values() for t in kv if t is not None)
        return {"full_precision": full, "compressed": comp}

    def reset(self) -> None:
        self.recent.clear()
        self.packed.clear()

    def as_hf_cache(self):
        """A transformers DynamicCache whose layers route through this store."""
        from transformers import DynamicCache

        store = self

        class _TQCache(DynamicCache):
            def update(self, key_states, value_states, layer_idx, cache_kwargs=None):
                return store.update(key_states, value_states, layer_idx)

            def get_seq_length(self, layer_idx=0):
                return store.get_seq_length(layer_idx)

        return _TQCache()

    @classmethod
    def from_model_config(cls, cfg, window: int = 128, bits_per_angle: int = 3) -> "TurboQuantCache":
        head_dim = getattr(cfg, "head_dim", None) or cfg.hidden_size // cfg.num_attention_heads
        return cls(head_dim, window, bits_per_angle)
