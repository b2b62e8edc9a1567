"""Operator layer: sm_100a kernels for CUDA tensors, PyTorch reference math for CPU.

Every op takes the same arguments on both devices.  CUDA tensors always go to the
native extension ``vramancer_b200._C`` (built by ``python setup.py build_ext
--inplace``); if it is missing on a machine with a GPU the op raises instead of
silently falling back.  CPU tensors run the plain-PyTorch reference of the same math,
which is the oracle the GPU tests compare against and the path used for CPU-only
execution (for example the split-vs-single parity check on two CPU devices).

Reference parity: these ops replace the reference's Triton kernels
(core/triton_fused_rmsnorm.py, core/triton_fused_rope.py, core/triton_sampling.py),
its paged attention kernel (csrc/paged_attention_kernel.cu) and the cuBLAS GEMMs of
its HF path.
"""
from __future__ import annotations

import importlib
import math
import os
from typing import Optional

import torch

_native = None
_native_err: Optional[BaseException] = None


LAUNCHES = [0]   # number of native kernel launches issued through this module


def native():
    """Returns the loaded extension module, raising a clear error if it is absent."""
    global _native, _native_err
    LAUNCHES[0] += 1
    if _native is not None:
        return _native
    try:
        _native = importlib.import_module("vramancer_b200._C")
    except BaseException as e:  # ImportError or a loader error
        _native_err = e
        raise RuntimeError(
            "vramancer_b200 native kernels are not built (run `python setup.py build_ext --inplace`): "
            f"{e!r}") from e
    return _native


def native_available() -> bool:
    try:
        _host_call()
        return True
    except RuntimeError:
        return False


EPI_NONE = 0
EPI_SILU_MUL = 1


# --------------------------------------------------------------------------- GEMM
def linear(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor] = None, *,
           out: Optional[torch.Tensor] = None, epilogue: int = EPI_NONE,
           residual: Optional[torch.Tensor] = None, force_splits: int = 0,
           ssq_out: Optional[torch.Tensor] = None, ssq_in: Optional[torch.Tensor] = None,
           ssq_parts: int = 0, norm_eps: float = 0.0) -> torch.Tensor:
    """y = x @ w.T (+ bias) (+ residual); with EPI_SILU_MUL, w rows are interleaved
    (gate_j, up_j) pairs and y[:, j] = silu(gate_j) * up_j.  `w` may be a quantised
    weight (quant.nvfp4.NVFP4Weight), which brings its own GEMM.

    Folded RMSNorm (decode, M <= 128): with `ssq_out` [parts, >= M] fp32 (needs
    `residual`), ssq_out[t, m] = sum over output features 128 t .. 128 t + 127 of
    bf16(y[m, n])^2; with `ssq_in`, x @ w.T is first scaled per row by
    rsqrt(sum_{t < ssq_parts} ssq_in[t, m] / K + norm_eps) (w carries the norm weight)."""
    if getattr(w, "_vrm_quant", None) is not None:
        if ssq_out is not None or ssq_in is not None:
            raise ValueError("the folded RMSNorm needs a bf16 weight")
        return w.linear(x, bias, out=out, epilogue=epilogue, residual=residual)
    if x.is_cuda:
        if out is None:
            n = w.shape[0] // 2 if epilogue == EPI_SILU_MUL else w.shape[0]
            out = torch.empty(x.shape[0], n, dtype=x.dtype, device=x.device)
        native().gemm_out(x, w, bias, out, force_splits, epilogue, residual, ssq_out, ssq_in, ssq_parts, norm_eps)
        return out
    y = x.float() @ w.float().t()
    if ssq_in is not None:
        sq = ssq_in[:ssq_parts, : x.shape[0]].sum(0)
        y = y * torch.rsqrt(sq / x.shape[1] + norm_eps)[:, None]
    if bias is not None:
        y = y + bias.float()
    if epilogue == EPI_SILU_MUL:
        g, u = y[:, 0::2], y[:, 1::2]
        y = torch.nn.functional.silu(g) * u
    if residual is not None:
        y = y + residual.float()
    y = y.to(x.dtype)
    if ssq_out is not None:
        M, N = y.shape
        parts = (N + 127) // 128
        yf = torch.nn.functional.pad(y.float(), (0, parts * 128 - N))
        ssq_out[:parts, :M] = (yf * yf).view(M, parts, 128).sum(-1).t()
    if out is not None:
        out.copy_(y)
        return out
    return y


# --------------------------------------------------------------------------- norms
def rmsnorm(x: torch.Tensor, w: torch.Tensor, eps: float, *, residual: Optional[torch.Tensor] = None,
            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """out = rmsnorm(x [+ residual]) * w; the sum is written back into residual."""
    if out is None:
        out = torch.empty_like(x)
    if x.is_cuda:
        native().rmsnorm(x, residual, w, out, eps)
        return out
    h = x.float()
    if residual is not None:
        h = (h + residual.float()).to(x.dtype)
        residual.copy_(h)
        h = h.float()
    y = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps) * w.float()
    out.copy_(y.to(out.dtype))
    return out


def layernorm(x: torch.Tensor, w: torch.Tensor, b: torch.Tensor, eps: float, *,
              residual: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty_like(x)
    if x.is_cuda:
        native().layernorm(x, residual, w, b, out, eps)
        return out
    h = x.float()
    if residual is not None:
        h = (h + residual.float()).to(x.dtype)
        residual.copy_(h)
        h = h.float()
    y = torch.nn.functional.layer_norm(h, (h.shape[-1],), w.float(), b.float(), eps)
    out.copy_(y.to(out.dtype))
    return out


# --------------------------------------------------------------------------- RoPE
def qk_rmsnorm(qkv: torch.Tensor, wq: torch.Tensor, wk: torch.Tensor, num_q_heads: int, num_kv_heads: int,
               head_dim: int, eps: float) -> None:
    """Per-head RMSNorm of the q and k heads of qkv [T, (Hq + 2 KH) * D] in place
    (Qwen3 q_norm / k_norm; v heads untouched)."""
    if qkv.is_cuda:
        native().qk_rmsnorm(qkv, wq, wk, num_q_heads, num_kv_heads, head_dim, eps)
        return
    T = qkv.shape[0]
    Hq, KH, D = num_q_heads, num_kv_heads, head_dim
    v = qkv.view(T, Hq + 2 * KH, D)
    for sl, w in ((slice(0, Hq), wq), (slice(Hq, Hq + KH), wk)):
        h = v[:, sl].float()
        y = h * torch.rsqrt(h.pow(2).mean(-1, keepdim=True) + eps) * w.float()
        v[:, sl] = y.to(qkv.dtype)


def rope_inv_freq(rot_dim: int, theta: float, scaling=None, max_pos: int = 0):
    """RoPE frequencies f_i = theta^(-2i/rot_dim), i < rot_dim/2, rescaled for long
    context, and the factor the cos / sin table is multiplied by.

    `scaling` is a mapping (or (key, value) pairs) of HF rope parameters:
      linear   f_i / factor (position interpolation)
      llama3   frequencies with wavelength above original_ctx / low_freq_factor divided
               by factor, below original_ctx / high_freq_factor kept, a linear blend of
               the two in between (the Llama 3.1 rule)
      yarn     NTK-by-parts (Peng et al., "YaRN", 2023): dimensions that turn fewer than
               beta_slow times over the original context are interpolated (f / factor),
               more than beta_fast times extrapolated (f), a linear ramp between; the
               table is scaled by 0.1 ln(factor) + 1 (or the mscale / mscale_all_dim
               ratio, or attention_factor)
      dynamic  the unscaled frequencies: NTK re-basing that depends on the current
               sequence length cannot live in one static table; exact while sequences
               stay within original_max_position_embeddings
    Returns (float64 tensor [rot_dim / 2], float table factor)."""
    i2 = torch.arange(0, rot_dim, 2, dtype=torch.float64) / rot_dim
    inv = 1.0 / (theta ** i2)
    sc = dict(scaling or {})
    kind = sc.get("rope_type", sc.get("type", "default"))
    if kind in ("default", "dynamic", None):
        return inv, 1.0
    factor = float(sc.get("factor", 1.0))
    if kind == "linear":
        return inv / factor, 1.0
    orig = float(sc.get("original_max_position_embeddings") or max_pos)
    if kind == "llama3":
        lo, hi = float(sc.get("low_freq_factor", 1.0)), float(sc.get("high_freq_factor", 4.0))
        wavelen = 2 * math.pi / inv
        smooth = ((orig / wavelen - lo) / (hi - lo)).clamp(0.0, 1.0)
        blended = (1 - smooth) * inv / factor + smooth * inv
        return torch.where(wavelen > orig / lo, inv / factor, torch.where(wavelen < orig / hi, inv, blended)), 1.0
    if kind == "yarn":
        if "factor" not in sc and max_pos and orig:
            factor = max_pos / orig
        beta_fast, beta_slow = float(sc.get("beta_fast", 32.0)), float(sc.get("beta_slow", 1.0))

        def dim_of(turns):      # dimension index whose frequency turns `turns` times over orig
            return rot_dim * math.log(orig / (turns * 2 * math.pi)) / (2 * math.log(theta))

        lo = max(math.floor(dim_of(beta_fast)), 0)
        hi = min(math.ceil(dim_of(beta_slow)), rot_dim - 1)
        if hi == lo:
            hi += 0.001
        ramp = ((torch.arange(rot_dim // 2, dtype=torch.float64) - lo) / (hi - lo)).clamp(0.0, 1.0)
        inv = (inv / factor) * ramp + inv * (1 - ramp)

        def mscale(s, m=1.0):
            return 1.0 if s <= 1 else 0.1 * m * math.log(s) + 1.0

        att = sc.get("attention_factor")
        if att is None:
            if sc.get("mscale") and sc.get("mscale_all_dim"):
                att = mscale(factor, float(sc["mscale"])) / mscale(factor, float(sc["mscale_all_dim"]))
            else:
                att = mscale(factor)
        return inv, float(att)
    raise ValueError(f"unsupported rope scaling {kind!r} (linear, llama3, yarn, dynamic)")


def rope_cos_sin(max_pos: int, rot_dim: int, theta: float, device=None, scaling=None) -> torch.Tensor:
    """[max_pos, rot_dim] fp32 table = [cos(p * f_i) | sin(p * f_i)] x table factor, with
    the frequencies and factor of `rope_inv_freq` (f_i = theta^(-2i/rot_dim) unscaled)."""
    inv, att = rope_inv_freq(rot_dim, theta, scaling, max_pos)
    p = torch.arange(max_pos, dtype=torch.float64)
    ang = torch.outer(p, inv)
    return (torch.cat([ang.cos(), ang.sin()], dim=1) * att).to(torch.float32).to(device)


def _fp8_dtype():
    return torch.float8_e4m3fn


def rope_kv_write(qkv: torch.Tensor, positions: Optional[torch.Tensor], cos_sin: Optional[torch.Tensor],
                  cache: torch.Tensor, slot_mapping: Optional[torch.Tensor], kv_scale: Optional[torch.Tensor],
                  layer: int, num_q_heads: int, num_kv_heads: int, head_dim: int) -> None:
    """Rotates q/k of qkv [T, (Hq+2KH)*D] in place and stores k/v rows into the paged cache
    [pages, layers, 2, KH, page_size, row] at slot_mapping (bf16, fp8 e4m3 / kv_scale, or
    four-bit rows in a uint8 cache: `kv.q4`)."""
    if qkv.is_cuda:
        native().rope_kv_write(qkv, positions, cos_sin, cache, slot_mapping, kv_scale, layer,
                               num_q_heads, num_kv_heads, head_dim)
        return
    T = qkv.shape[0]
    Hq, KH, D = num_q_heads, num_kv_heads, head_dim
    v = qkv.view(T, Hq + 2 * KH, D)
    if cos_sin is not None and T > 0:
        rot = cos_sin.shape[1]
        half = rot // 2
        cs = cos_sin[positions.long()]
        c, s = cs[:, None, :half], cs[:, None, half:]
        qk = v[:, :Hq + KH, :].float()
        x1, x2 = qk[..., :half].clone(), qk[..., half:rot].clone()
        qk[..., :half] = x1 * c - x2 * s
        qk[..., half:rot] = x2 * c + x1 * s
        v[:, :Hq + KH, :] = qk.to(qkv.dtype)
    if slot_mapping is None or T == 0:
        return
    ps = cache.shape[4]
    slots = slot_mapping.long()
    valid = slots >= 0
    if not bool(valid.any()):
        return
    idx = torch.nonzero(valid).flatten()
    page, off = slots[idx] // ps, slots[idx] % ps
    k = v[idx, Hq:Hq + KH, :]
    vv = v[idx, Hq + KH:, :]
    if cache.dtype == torch.uint8:
        from ..kv import q4
        cache[page, layer, 0, :, off, :] = q4.quantize(k.float())
        cache[page, layer, 1, :, off, :] = q4.quantize(vv.float())
    elif cache.dtype == torch.float8_e4m3fn:
        sk = kv_scale[layer, 0].view(1, KH, 1)
        sv = kv_scale[layer, 1].view(1, KH, 1)
        kq = (k.float() / sk).clamp(-448, 448).to(torch.float8_e4m3fn)
        vq = (vv.float() / sv).clamp(-448, 448).to(torch.float8_e4m3fn)
        cache[page, layer, 0, :, off, :] = kq
        cache[page, layer, 1, :, off, :] = vq
    else:
        cache[page, layer, 0, :, off, :] = k.to(cache.dtype)
        cache[page, layer, 1, :, off, :] = vv.to(cache.dtype)


# --------------------------------------------------------------------------- TurboQuant KV pages
def tq_kv_write(qkv: torch.Tensor, slot_mapping: torch.Tensor, pool: torch.Tensor, layer: int,
                num_q_heads: int, num_kv_heads: int, comp) -> None:
    """The (rotated) k / v rows of qkv [T, (Hq + 2 KH) * 128] as 64-byte TurboQuant records
    into pool int8 [pages, layers, 2, KH, 16, 64] at slot_mapping (< 0 skips); comp is
    the pool's kv.turboquant.KVCacheCompressor (rotation signs, JL matrix)."""
    if qkv.is_cuda:
        native().tq_kv_write(qkv, slot_mapping, pool, layer, num_q_heads, num_kv_heads, comp.signs, comp.jl)
        return
    T = qkv.shape[0]
    Hq, KH = num_q_heads, num_kv_heads
    v = qkv.view(T, Hq + 2 * KH, 128)
    slots = slot_mapping.long()
    idx = torch.nonzero(slots >= 0).flatten()
    if idx.numel() == 0:
        return
    rec = comp.compress(torch.stack([v[idx, Hq:Hq + KH], v[idx, Hq + KH:]], 1).float())   # [n, 2, KH, 64]
    pool[slots[idx] // 16, layer, :, :, slots[idx] % 16] = rec.view(torch.int8)


def tq_paged_decode(q: torch.Tensor, pool: torch.Tensor, layer: int, block_tables: torch.Tensor,
                    context_lens: torch.Tensor, comp, sm_scale: float, num_q_heads: int,
                    out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Decode attention scored straight from TurboQuant K records (asymmetric QJL
    estimator) with values from their polar decodes; q [B, >= Hq * 128] -> [B, Hq * 128]."""
    B = q.shape[0]
    if out is None:
        out = torch.empty(B, num_q_heads * 128, dtype=q.dtype, device=q.device)
    if q.is_cuda:
        native().tq_paged_decode(q, pool, layer, block_tables, context_lens, comp.signs, comp.jl, sm_scale, out,
                                 num_q_heads)
        return out
    KH = pool.shape[3]
    G = num_q_heads // KH
    for b in range(B):
        n = int(context_lens[b])
        pages = block_tables[b, : (n + 15) // 16].long()
        rec = pool[pages, layer].view(torch.uint8)                      # [P, 2, KH, 16, 64]
        rec = rec.permute(1, 2, 0, 3, 4).reshape(2, KH, -1, 64)[:, :, :n]
        qb = q[b, : num_q_heads * 128].float().view(KH, G, 128)
        for h in range(KH):
            s = comp.attention_score(qb[h], rec[0, h]) * sm_scale
            w = torch.softmax(s, dim=-1)
            vv = comp.decompress(rec[1, h], torch.float32)
            out[b, h * G * 128:(h + 1) * G * 128] = (w @ vv).reshape(-1).to(out.dtype)
    return out


def tq_decompress_pool(pool: torch.Tensor, layer: int, pages: torch.Tensor, comp) -> torch.Tensor:
    """bf16 pages [len(pages), 1, 2, KH, 16, 128] decoded from a TurboQuant pool's layer."""
    rec = pool[pages.long(), layer].contiguous()                          # [n, 2, KH, 16, 64]
    n, _, KH = rec.shape[0], rec.shape[1], rec.shape[2]
    dec = comp.decompress(rec.view(torch.uint8).reshape(-1, 64), torch.bfloat16)
    return dec.view(n, 1, 2, KH, 16, 128)


# --------------------------------------------------------------------------- attention
def cache_head_dim(cache: torch.Tensor) -> int:
    """Head dim of a KV pool [pages, layers, 2, KH, page_size, row] (uint8 = four-bit rows)."""
    return cache.shape[5] * 8 // 5 if cache.dtype == torch.uint8 else cache.shape[5]


def _gather_kv(cache: torch.Tensor, layer: int, pages: torch.Tensor, n: int,
               kv_scale: Optional[torch.Tensor]):
    """[n, KH, D] float K and V of one sequence from its page list."""
    k = cache[pages, layer, 0]  # [P, KH, ps, D]
    v = cache[pages, layer, 1]
    KH, ps, D = k.shape[1], k.shape[2], k.shape[3]
    k = k.permute(0, 2, 1, 3).reshape(-1, KH, D)[:n]
    v = v.permute(0, 2, 1, 3).reshape(-1, KH, D)[:n]
    if cache.dtype == torch.uint8:
        from ..kv import q4
        return q4.dequantize(k), q4.dequantize(v)
    k, v = k.float(), v.float()
    if kv_scale is not None and cache.dtype == torch.float8_e4m3fn:
        k = k * kv_scale[layer, 0].view(1, KH, 1)
        v = v * kv_scale[layer, 1].view(1, KH, 1)
    return k, v


def paged_attention_decode(q: torch.Tensor, cache: torch.Tensor, layer: int, block_tables: torch.Tensor,
                           context_lens: torch.Tensor, kv_scale: Optional[torch.Tensor], sm_scale: float,
                           num_q_heads: int, *, out: Optional[torch.Tensor] = None,
                           num_splits: int = 0, positions: Optional[torch.Tensor] = None,
                           cos_sin: Optional[torch.Tensor] = None,
                           slot_mapping: Optional[torch.Tensor] = None,
                           l2_prefetch: Optional[torch.Tensor] = None) -> torch.Tensor:
    """One query token per sequence: q [B, >=Hq*D] -> out [B, Hq*D].

    With `positions` (and `slot_mapping`) q is the unrotated qkv row and the kernel also
    does this step's RoPE (cos_sin, rotate-half over all head dims; None = no rotation)
    and writes the token's k / v into the cache: the work of `rope_kv_write`, fused.
    `l2_prefetch` (a contiguous tensor, e.g. the next projection's weights) is brought
    into L2 by the kernel's CTAs while attention runs (GPU only; no effect on results)."""
    B = q.shape[0]
    D = cache_head_dim(cache)
    if out is None:
        out = torch.empty(B, num_q_heads * D, dtype=q.dtype, device=q.device)
    if q.is_cuda:
        native().paged_attention_decode(q, cache, layer, block_tables, context_lens, kv_scale, sm_scale, out,
                                        num_splits, num_q_heads, positions, cos_sin, slot_mapping, l2_prefetch)
        return out
    if positions is not None:
        rope_kv_write(q, positions, cos_sin, cache, slot_mapping, kv_scale, layer, num_q_heads, cache.shape[3], D)
    KH = cache.shape[3]
    G = num_q_heads // KH
    ps = cache.shape[4]
    for b in range(B):
        n = int(context_lens[b])
        if n == 0:
            out[b].zero_()
            continue
        pages = block_tables[b, : (n + ps - 1) // ps].long()
        k, v = _gather_kv(cache, layer, pages, n, kv_scale)
        qb = q[b, : num_q_heads * D].float().view(KH, G, D)
        s = torch.einsum("kgd,nkd->kgn", qb, k) * sm_scale
        p = torch.softmax(s, dim=-1)
        o = torch.einsum("kgn,nkd->kgd", p, v)
        out[b] = o.reshape(-1).to(out.dtype)
    return out


def paged_attention_prefill(q: torch.Tensor, cache: torch.Tensor, layer: int, block_tables: torch.Tensor,
                            cu_q: torch.Tensor, context_lens: torch.Tensor, kv_scale: Optional[torch.Tensor],
                            sm_scale: float, num_q_heads: int, max_q_len: int, *,
                            out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Causal attention of new tokens (rows of q, grouped by cu_q) over their sequence's
    cached prefix plus themselves; keys/values are read from the paged cache."""
    T = q.shape[0]
    D = cache_head_dim(cache)
    if out is None:
        out = torch.empty(T, num_q_heads * D, dtype=q.dtype, device=q.device)
    if q.is_cuda:
        native().paged_attention_prefill(q, cache, layer, block_tables, cu_q, context_lens, kv_scale, sm_scale,
                                         out, max_q_len, num_q_heads)
        return out
    KH = cache.shape[3]
    G = num_q_heads // KH
    ps = cache.shape[4]
    B = cu_q.numel() - 1
    for b in range(B):
        s0, s1 = int(cu_q[b]), int(cu_q[b + 1])
        ql = s1 - s0
        if ql == 0:
            continue
        n = int(context_lens[b])
        pages = block_tables[b, : (n + ps - 1) // ps].long()
        k, v = _gather_kv(cache, layer, pages, n, kv_scale)
        qb = q[s0:s1, : num_q_heads * D].float().view(ql, KH, G, D)
        s = torch.einsum("qkgd,nkd->kgqn", qb, k) * sm_scale
        qpos = torch.arange(n - ql, n).view(ql, 1)
        kpos = torch.arange(n).view(1, n)
        s = s.masked_fill(kpos > qpos, float("-inf"))
        p = torch.softmax(s, dim=-1)
        o = torch.einsum("kgqn,nkd->qkgd", p, v)
        out[s0:s1] = o.reshape(ql, -1).to(out.dtype)
    return out


# --------------------------------------------------------------------------- elementwise
def silu_mul(x: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """[T, 2I] (gate | up) -> silu(gate) * up."""
    I = x.shape[1] // 2
    if out is None:
        out = torch.empty(x.shape[0], I, dtype=x.dtype, device=x.device)
    if x.is_cuda:
        native().silu_mul(x, out)
        return out
    out.copy_((torch.nn.functional.silu(x[:, :I].float()) * x[:, I:].float()).to(out.dtype))
    return out


def gelu_tanh_(x: torch.Tensor) -> torch.Tensor:
    if x.is_cuda:
        native().gelu_tanh_(x)
        return x
    x.copy_(torch.nn.functional.gelu(x.float(), approximate="tanh").to(x.dtype))
    return x


def embedding(ids: torch.Tensor, table: torch.Tensor, *, positions: Optional[torch.Tensor] = None,
              pos_table: Optional[torch.Tensor] = None, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(ids.numel(), table.shape[1], dtype=table.dtype, device=table.device)
    if table.is_cuda:
        native().embedding(ids, table, positions, pos_table, out)
        return out
    y = table[ids.long()]
    if pos_table is not None:
        y = (y.float() + pos_table[positions.long()].float()).to(table.dtype)
    out.copy_(y)
    return out


def add_(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    if a.is_cuda:
        native().add_(a, b)
        return a
    a.copy_((a.float() + b.float()).to(a.dtype))
    return a


# --------------------------------------------------------------------------- sampling
def argmax(logits: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    if logits.is_cuda:
        native().argmax(logits, out)
        return out
    out.copy_(torch.argmax(logits.float(), dim=-1).to(torch.int32))
    return out


def sample(logits: torch.Tensor, temperature: torch.Tensor, top_k: torch.Tensor, top_p: torch.Tensor,
           seed: int, steps: torch.Tensor, out: Optional[torch.Tensor] = None) -> torch.Tensor:
    """Temperature / top-k / top-p sampling (temperature <= 0 -> greedy)."""
    if out is None:
        out = torch.empty(logits.shape[0], dtype=torch.int32, device=logits.device)
    if logits.is_cuda:
        native().sample(logits, temperature, top_k, top_p, seed, steps, out)
        return out
    g = torch.Generator().manual_seed(int(seed))
    for r in range(logits.shape[0]):
        x = logits[r].float()
        t = float(temperature[r])
        if t <= 0:
            out[r] = int(torch.argmax(x))
            continue
        z = x / t
        k = int(top_k[r])
        if 0 < k < z.numel():
            thr = torch.topk(z, k).values[-1]
            z = z.masked_fill(z < thr, float("-inf"))
        p = float(top_p[r])
        if p < 1.0:
            probs = torch.softmax(z, -1)
            sp, si = torch.sort(probs, descending=True)
            keep = torch.cumsum(sp, 0) - sp < p
            mask = torch.zeros_like(probs, dtype=torch.bool)
            mask[si[keep]] = True
            z = z.masked_fill(~mask, float("-inf"))
        out[r] = int(torch.multinomial(torch.softmax(z, -1), 1, generator=g))
    return out


# Vocabulary-parallel sampling (sampling.cu): candidates per row and rank, and the
# largest top-k served from candidates.
VP_KC, VP_KMAX = 256, 128


def vp_sampling_ok(temperature, top_k, top_p, vocab: int, kmax: int = VP_KMAX) -> bool:
    """True when every row can be sampled from per-rank candidates: greedy, plain
    temperature, or top-k <= kmax (with any top-p).  Top-p without top-k needs the whole
    distribution, so such steps gather the full logits."""
    for t, k, p in zip(temperature, top_k, top_p):
        if t > 0 and not ((k <= 0 or k >= vocab) and p >= 1.0) and not (0 < k <= kmax):
            return False
    return True


def sample_vocab_parallel(logits: torch.Tensor, v_off: int, vocab: int, temperature: torch.Tensor,
                          top_k: torch.Tensor, top_p: torch.Tensor, seed: int, steps: torch.Tensor,
                          gather, out: Optional[torch.Tensor] = None, kc: int = VP_KC,
                          kmax: int = VP_KMAX) -> torch.Tensor:
    """Samples rows of a vocabulary that is split over tensor-parallel ranks.

    logits: this rank's bf16 shard [B, Vs] of columns [v_off, v_off + Vs); gather(t)
    returns every rank's t stacked ([ranks, ...]).  Each rank reduces its shard to kc
    candidates per row, one all-gather moves B x kc x 8 bytes per rank, and every rank
    picks the same ids -- for greedy rows, plain-temperature rows and rows with
    top-k <= kmax, the ids the full-vocabulary sampler gives (same Gumbel keys)."""
    B = logits.shape[0]
    if out is None:
        out = torch.empty(B, dtype=torch.int32, device=logits.device)
    cand = torch.empty(2, B, kc, dtype=torch.int32, device=logits.device)
    native().sample_vp_local(logits, int(v_off), int(vocab), temperature, top_k, top_p, int(seed), steps, kmax, cand)
    native().sample_vp_combine(gather(cand), int(vocab), temperature, top_k, top_p, int(seed), steps, kmax, out)
    return out


def _host_call():
    m = native()
    LAUNCHES[0] -= 1
    return m


def reserve_workspace(nbytes: int) -> None:
    _host_call().reserve_workspace(int(nbytes))


def read_and_clear_errors() -> int:
    """Error bits raised by bounded device-side waits since the last call (0 = none)."""
    return int(_host_call().read_and_clear_errors())


def decode_attention_splits(batch: int, kv_heads: int, max_pages: int) -> int:
    return int(_host_call().decode_attention_splits(batch, kv_heads, max_pages))
