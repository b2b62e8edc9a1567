"""Kernel microbenchmarks with CUDA-event timing (also the small cases for ncu).

    python -m vramancer_b200.ops.microbench gemm --m 1 --n 5120 --k 13824
    python -m vramancer_b200.ops.microbench decode-attn --batch 32 --ctx 768
    python -m vramancer_b200.ops.microbench all

Reports achieved bandwidth / FLOP rate against MEASURED_PEAKS.json when present
(copy bandwidth and cuBLAS bf16 throughput measured on this GPU type), otherwise
against 6.65 TB/s and 1.59 PFLOP/s.

Reference parity: core/layer_profiler.py:182-611 (GPU GFLOPS / bandwidth
microbenchmarks) and core/benchmark.py.
"""
from __future__ import annotations

import argparse
import json
import math
import os

import torch

from . import (argmax, linear, native, paged_attention_decode, paged_attention_prefill, rmsnorm, rope_cos_sin,
               rope_kv_write, sample)

ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return d["hbm_gbs"] / 1000.0, d["bf16_tflops"], "measured"
    return 6.65, 1590.0, "fallback"


def time_it(fn, iters=50, warm=5, graph=True):
    """Per-call device time.  With graph=True the `iters` calls are captured in one CUDA
    graph and replayed, so host launch overhead is excluded (as in the decode graph)."""
    for _ in range(warm):
        fn()
    torch.cuda.synchronize()
    if graph:
        g = torch.cuda.CUDAGraph()
        s = torch.cuda.Stream()
        s.wait_stream(torch.cuda.current_stream())
        with torch.cuda.stream(s):
            fn()
        torch.cuda.current_stream().wait_stream(s)
        torch.cuda.synchronize()
        with torch.cuda.graph(g):
            for _ in range(iters):
                fn()
        g.replay()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record()
        g.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / iters * 1000.0
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(iters):
        fn()
    e1.record()
    torch.cuda.synchronize()
    return e0.elapsed_time(e1) / iters * 1000.0  # us


def bench_gemm(m, n, k, iters=50, copies=None, residual=False, fold=None):
    """Rotates over enough weight copies to exceed L2 so every launch streams from HBM.
    fold="producer": residual GEMM that also stores the per-token norm sums;
    fold="consumer": GEMM scaled by the folded RMSNorm (norm sums read per call)."""
    hbm, tflops, src = peaks()
    wbytes = n * k * 2
    if copies is None:
        copies = max(1, math.ceil(3 * 126e6 / wbytes))
    ws = [torch.randn(n, k, device="cuda", dtype=torch.bfloat16) * 0.02 for _ in range(copies)]
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    state = [0]

    ssq = torch.ones(64, 128, device="cuda") if fold else None
    parts = (k + 127) // 128
    if fold == "producer":
        residual = True

    def fn():
        # residual=True: the in-place residual update of the decode step (out += x W^T)
        if fold == "consumer":
            linear(x, ws[state[0] % copies], out=out, ssq_in=ssq, ssq_parts=parts, norm_eps=1e-6)
        else:
            linear(x, ws[state[0] % copies], out=out, residual=out if residual else None,
                   ssq_out=ssq if fold == "producer" else None)
        state[0] += 1

    us = time_it(fn, iters)
    byts = wbytes + m * k * 2 + m * n * 2 * (2 if residual else 1)
    flops = 2.0 * m * n * k
    r = {"kernel": "gemm", "m": m, "n": n, "k": k, "residual": residual, "fold": fold, "us": round(us, 2),
         "tb_s": round(byts / us / 1e6, 3), "frac_hbm": round(byts / us / 1e6 / hbm, 3),
         "tflops": round(flops / us / 1e6, 1), "frac_tc": round(flops / us / 1e6 / tflops, 3),
         "peaks": src}
    if m >= 256 and not residual:
        # the library GEMM on the same operands, for comparison only
        wt = [w.t() for w in ws]
        st2 = [0]

        def lib():
            torch.matmul(x, wt[st2[0] % copies], out=out)
            st2[0] += 1

        lus = time_it(lib, iters)
        r["cublas_us"] = round(lus, 2)
        r["vs_cublas"] = round(lus / us, 3)
    return r


def bench_nvfp4(m, n, k, iters=50, copies=None):
    """W4A16 NVFP4 GEMM; bytes = packed weights + block scales + activations + output."""
    from ..quant.nvfp4 import quantize
    hbm, tflops, src = peaks()
    wbytes = n * k // 2 + n * k // 16
    if copies is None:
        copies = max(1, math.ceil(3 * 126e6 / wbytes))
    base = torch.randn(n, k, device="cuda", dtype=torch.bfloat16) * 0.02
    ws = [quantize(base * (1 + 0.01 * i)) for i in range(copies)]
    del base
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(m, n, device="cuda", dtype=torch.bfloat16)
    state = [0]

    def fn():
        linear(x, ws[state[0] % copies], out=out)
        state[0] += 1

    us = time_it(fn, iters)
    byts = wbytes + m * k * 2 + m * n * 2
    return {"kernel": "nvfp4_gemm", "m": m, "n": n, "k": k, "us": round(us, 2),
            "tb_s": round(byts / us / 1e6, 3), "frac_hbm": round(byts / us / 1e6 / hbm, 3),
            "bf16_equiv_tb_s": round(n * k * 2 / us / 1e6, 3), "peaks": src}


def _kv_cache(shape, fp8, q4):
    """Random KV pool of one page format (bf16, fp8 e4m3, or four-bit rows in uint8)."""
    x = torch.randn(*shape, device="cuda")
    if q4:
        from ..kv import q4 as q4fmt
        return q4fmt.quantize(x)
    return x.to(torch.float8_e4m3fn if fp8 else torch.bfloat16)


def bench_decode_attn(batch, ctx, kv_heads=8, q_heads=40, head_dim=128, layers=4, fp8=False, iters=50,
                      splits=0, fused=False, q4=False):
    """splits > 0 forces the split count; fused runs the model's path (RoPE on q and the
    step's K/V written into its page inside the kernel); q4 reads four-bit pages."""
    hbm, _, src = peaks()
    ps = 16
    pages = (ctx + ps - 1) // ps
    P = batch * pages
    cache = _kv_cache((P, layers, 2, kv_heads, ps, head_dim), fp8, q4)
    bt = torch.arange(P, dtype=torch.int32, device="cuda").view(batch, pages)
    cl = torch.full((batch,), ctx, dtype=torch.int32, device="cuda")
    q = torch.randn(batch, (q_heads + (2 * kv_heads if fused else 0)) * head_dim, device="cuda",
                    dtype=torch.bfloat16)
    out = torch.empty(batch, q_heads * head_dim, device="cuda", dtype=torch.bfloat16)
    scale = torch.ones(layers, 2, kv_heads, device="cuda") if fp8 else None
    state = [0]
    kw = {}
    if fused:
        pos = torch.full((batch,), ctx - 1, dtype=torch.int32, device="cuda")
        slots = bt[:, (ctx - 1) // ps] * ps + (ctx - 1) % ps
        kw = dict(positions=pos, cos_sin=rope_cos_sin(ctx + 16, head_dim, 1e6, "cuda"), slot_mapping=slots.int())

    def fn():
        paged_attention_decode(q, cache, state[0] % layers, bt, cl, scale, 1 / math.sqrt(head_dim), q_heads, out=out,
                               num_splits=splits, **kw)
        state[0] += 1

    us = time_it(fn, iters)
    byts = batch * ctx * kv_heads * 2 * cache.shape[5] * cache.element_size()
    return {"kernel": "decode_attn", "batch": batch, "ctx": ctx, "fp8": fp8, "q4": q4, "kv_heads": kv_heads,
            "q_heads": q_heads, "splits": splits or "auto", "fused": fused, "us": round(us, 2),
            "tb_s": round(byts / us / 1e6, 3), "frac_hbm": round(byts / us / 1e6 / hbm, 3), "peaks": src}


def bench_tq_decode(batch, ctx, kv_heads=8, q_heads=40, layers=4, iters=50):
    """Decode attention straight from TurboQuant KV pages (64-byte records per row)."""
    from ..kv.pool import KVPool, KVPoolSpec
    from . import tq_kv_write, tq_paged_decode
    hbm, _, src = peaks()
    ps, D = 16, 128
    pages = (ctx + ps - 1) // ps
    P = batch * pages
    pool = KVPool(KVPoolSpec(P, layers, kv_heads, D, dtype=torch.int8), device="cuda")
    bt = torch.arange(P, dtype=torch.int32, device="cuda").view(batch, pages)
    cl = torch.full((batch,), ctx, dtype=torch.int32, device="cuda")
    slots = torch.arange(P * ps, dtype=torch.int32, device="cuda")
    qkv = torch.randn(P * ps, (q_heads + 2 * kv_heads) * D, device="cuda", dtype=torch.bfloat16)
    for layer in range(layers):
        tq_kv_write(qkv, slots, pool.cache, layer, q_heads, kv_heads, pool.tq)
    q = torch.randn(batch, q_heads * D, device="cuda", dtype=torch.bfloat16)
    out = torch.empty_like(q)
    state = [0]

    def fn():
        tq_paged_decode(q, pool.cache, state[0] % layers, bt, cl, pool.tq, 1 / math.sqrt(D), q_heads, out=out)
        state[0] += 1

    us = time_it(fn, iters)
    byts = batch * ctx * kv_heads * 2 * 64
    return {"kernel": "tq_paged_decode", "batch": batch, "ctx": ctx, "us": round(us, 2),
            "tb_s": round(byts / us / 1e6, 3), "frac_hbm": round(byts / us / 1e6 / hbm, 3), "peaks": src}


def bench_nvfp4_prefill(m, n, k, iters=20):
    """Prefill-sized GEMM three ways: bf16 tcgen05 GEMM, NVFP4 W4A4 block-scaled tcgen05
    GEMM (codes already quantised), and W4A4 including the activation quantisation."""
    from ..quant import nvfp4 as nv
    _, tflops, src = peaks()
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    w = torch.randn(n, k, device="cuda", dtype=torch.bfloat16) * 0.02
    qw = nv.quantize(w)
    mp = (m + 127) // 128 * 128
    qa, sfa, gsa = native().nvfp4_rows_quantize(x, mp, None)
    flop = 2.0 * m * n * k
    t_bf16 = time_it(lambda: linear(x, w), iters)
    t_gemm = time_it(lambda: native().nvfp4_bs_gemm(qa, sfa, gsa, m, qw.q_rows, qw.s_atoms, qw.gs), iters)
    t_full = time_it(lambda: linear(x, qw), iters)
    r = {"kernel": "nvfp4_prefill", "m": m, "n": n, "k": k, "bf16_us": round(t_bf16, 2),
         "bf16_tflops": round(flop / t_bf16 / 1e6, 1), "w4a4_gemm_us": round(t_gemm, 2),
         "w4a4_gemm_tflops": round(flop / t_gemm / 1e6, 1), "w4a4_with_act_quant_us": round(t_full, 2),
         "w4a4_with_act_quant_tflops": round(flop / t_full / 1e6, 1), "peaks": src,
         "bf16_frac_of_measured": round(flop / t_bf16 / 1e6 / tflops, 3)}
    return r


def bench_rmsnorm(tokens, hidden=5120, iters=50):
    """Residual add + RMSNorm over [tokens, hidden] bf16 (the decode step's norm)."""
    hbm, _, src = peaks()
    n = max(2, math.ceil(3 * 126e6 / (tokens * hidden * 2 * 3)))
    xs = [torch.randn(tokens, hidden, device="cuda", dtype=torch.bfloat16) for _ in range(n)]
    rs = [torch.randn(tokens, hidden, device="cuda", dtype=torch.bfloat16) for _ in range(n)]
    w = torch.randn(hidden, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(tokens, hidden, device="cuda", dtype=torch.bfloat16)
    state = [0]

    def fn():
        i = state[0] % n
        rmsnorm(xs[i], w, 1e-6, residual=rs[i], out=out)
        state[0] += 1

    us = time_it(fn, iters)
    byts = tokens * hidden * 2 * 4   # read x, residual; write residual, out
    return {"kernel": "rmsnorm_residual", "tokens": tokens, "hidden": hidden, "us": round(us, 2),
            "tb_s": round(byts / us / 1e6, 3), "frac_hbm": round(byts / us / 1e6 / hbm, 3), "peaks": src}


def bench_rope_kv(tokens, q_heads=40, kv_heads=8, head_dim=128, fp8=False, iters=50):
    """RoPE on q/k + K/V rows written into 16-token pages (bf16, or fp8 with per-head scales)."""
    hbm, _, src = peaks()
    ps, layers = 16, 4
    width = (q_heads + 2 * kv_heads) * head_dim
    qkv = torch.randn(tokens, width, device="cuda", dtype=torch.bfloat16)
    pages = (tokens + ps - 1) // ps + 1
    dt = torch.float8_e4m3fn if fp8 else torch.bfloat16
    cache = torch.zeros(pages, layers, 2, kv_heads, ps, head_dim, device="cuda", dtype=dt)
    cs = rope_cos_sin(8192, head_dim, 1e6, device="cuda")
    pos = torch.randint(0, 8192, (tokens,), device="cuda", dtype=torch.int32)
    slots = torch.randperm(pages * ps, device="cuda")[:tokens].to(torch.int32)
    scale = torch.full((layers, 2, kv_heads), 0.05, device="cuda") if fp8 else None
    state = [0]

    def fn():
        rope_kv_write(qkv, pos, cs, cache, slots, scale, state[0] % layers, q_heads, kv_heads, head_dim)
        state[0] += 1

    us = time_it(fn, iters)
    byts = tokens * (width * 2 + (q_heads + kv_heads) * head_dim * 2 + 2 * kv_heads * head_dim * cache.element_size())
    return {"kernel": "rope_kv_write", "tokens": tokens, "fp8": fp8, "us": round(us, 2),
            "tb_s": round(byts / us / 1e6, 3), "frac_hbm": round(byts / us / 1e6 / hbm, 3), "peaks": src}


def bench_prefill_attn(batch, seq, q_heads=40, kv_heads=8, head_dim=128, fp8=False, iters=10, q4=False):
    """Causal paged prefill attention of `batch` sequences of `seq` new tokens (no prefix)."""
    _, tflops, src = peaks()
    ps, layers = 16, 1
    pages = (seq + ps - 1) // ps
    P = batch * pages
    cache = _kv_cache((P, layers, 2, kv_heads, ps, head_dim), fp8, q4)
    bt = torch.arange(P, dtype=torch.int32, device="cuda").view(batch, pages)
    cl = torch.full((batch,), seq, dtype=torch.int32, device="cuda")
    cu = torch.arange(0, (batch + 1) * seq, seq, dtype=torch.int32, device="cuda")
    q = torch.randn(batch * seq, q_heads * head_dim, device="cuda", dtype=torch.bfloat16)
    out = torch.empty_like(q)
    scale = torch.ones(layers, 2, kv_heads, device="cuda") if fp8 else None

    def fn():
        paged_attention_prefill(q, cache, 0, bt, cu, cl, scale, 1 / math.sqrt(head_dim), q_heads, seq, out=out)

    us = time_it(fn, iters)
    flop = batch * q_heads * 4.0 * head_dim * seq * (seq + 1) / 2   # causal QK^T + PV
    return {"kernel": "prefill_attn", "batch": batch, "seq": seq, "fp8": fp8, "q4": q4, "us": round(us, 2),
            "tflops": round(flop / us / 1e6, 1), "frac_of_measured_bf16": round(flop / us / 1e6 / tflops, 3),
            "peaks": src}


def bench_sample(batch, vocab=152064, greedy=False, iters=50):
    """Sampler over bf16 logits [batch, vocab]: argmax, or temperature / top-k / top-p."""
    hbm, _, src = peaks()
    logits = torch.randn(batch, vocab, device="cuda", dtype=torch.bfloat16)
    out = torch.empty(batch, dtype=torch.int32, device="cuda")
    temp = torch.full((batch,), 0.8, device="cuda")
    topk = torch.full((batch,), 50, dtype=torch.int32, device="cuda")
    topp = torch.full((batch,), 0.9, device="cuda")
    steps = torch.zeros(batch, dtype=torch.int32, device="cuda")
    if greedy:
        fn = lambda: argmax(logits, out)   # noqa: E731
    else:
        fn = lambda: sample(logits, temp, topk, topp, 1234, steps, out)   # noqa: E731
    us = time_it(fn, iters)
    byts = batch * vocab * 2
    return {"kernel": "argmax" if greedy else "sample_topk_topp", "batch": batch, "vocab": vocab,
            "us": round(us, 2), "tb_s": round(byts / us / 1e6, 3), "frac_hbm": round(byts / us / 1e6 / hbm, 3),
            "peaks": src}


def bench_turboquant(vectors, head_dim=128, iters=20):
    """TurboQuant record compress / decompress of `vectors` head_dim vectors (bf16)."""
    from ..kv.turboquant import KVCacheCompressor
    hbm, _, src = peaks()
    comp = KVCacheCompressor(head_dim=head_dim).to("cuda")
    x = torch.randn(vectors, head_dim, device="cuda", dtype=torch.bfloat16)
    rec = comp.compress(x)
    t_c = time_it(lambda: comp.compress(x), iters, graph=False)
    t_d = time_it(lambda: comp.decompress(rec), iters, graph=False)
    rb = rec.numel() * rec.element_size()
    xb = x.numel() * 2
    return {"kernel": "turboquant", "vectors": vectors, "record_bytes": rec.shape[-1],
            "compress_us": round(t_c, 2), "compress_tb_s": round((xb + rb) / t_c / 1e6, 3),
            "decompress_us": round(t_d, 2), "decompress_tb_s": round((xb + rb) / t_d / 1e6, 3),
            "frac_hbm_decompress": round((xb + rb) / t_d / 1e6 / hbm, 3), "peaks": src}


def bench_act_quant(tokens, hidden=5120, iters=50):
    """Per-token activation quantisers feeding the low-precision GEMMs: fp8 e4m3 rows
    (per-token scale) and NVFP4 rows (per-token scale, e4m3 scale per 16, e2m1 codes)."""
    hbm, _, src = peaks()
    x = torch.randn(tokens, hidden, device="cuda", dtype=torch.bfloat16)
    mp = (tokens + 127) // 128 * 128
    t8 = time_it(lambda: native().fp8_rows_quantize(x), iters)
    t4 = time_it(lambda: native().nvfp4_rows_quantize(x, mp, None), iters)
    b8 = tokens * hidden * 3
    b4 = tokens * hidden * 2 + tokens * hidden // 2 + tokens * hidden // 16
    return {"kernel": "act_quant", "tokens": tokens, "hidden": hidden,
            "fp8_us": round(t8, 2), "fp8_frac_hbm": round(b8 / t8 / 1e6 / hbm, 3),
            "nvfp4_us": round(t4, 2), "nvfp4_frac_hbm": round(b4 / t4 / 1e6 / hbm, 3), "peaks": src}


def bench_fp8(m, n, k, iters=50):
    """FP8 W8A8 GEMM (per-channel weight scales, per-token activation scales, activation
    quantisation included) against the bf16 GEMM on the same shape; weights rotated past
    L2."""
    from ..quant import fp8 as f8
    hbm, tflops, src = peaks()
    copies = max(1, math.ceil(3 * 126e6 / (n * k)))
    ws = [(torch.randn(n, k, device="cuda") * 0.02).bfloat16() for _ in range(copies)]
    qs = [f8.quantize(w) for w in ws]
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    st = [0, 0]

    def f():
        linear(x, qs[st[0] % copies])
        st[0] += 1

    def b():
        linear(x, ws[st[1] % copies])
        st[1] += 1

    t8 = time_it(f, iters)
    t16 = time_it(b, iters)
    flop = 2.0 * m * n * k
    wb8, wb16 = n * k, 2 * n * k
    return {"kernel": "fp8_w8a8_gemm", "m": m, "n": n, "k": k, "fp8_us": round(t8, 2), "bf16_us": round(t16, 2),
            "speedup": round(t16 / t8, 3), "fp8_weight_tb_s": round(wb8 / t8 / 1e6, 3),
            "fp8_frac_hbm": round(wb8 / t8 / 1e6 / hbm, 3), "fp8_tflops": round(flop / t8 / 1e6, 1),
            "bf16_frac_hbm": round(wb16 / t16 / 1e6 / hbm, 3), "peaks": src}


def trace_gemm(m, n, k):
    """Per-CTA timelines of two back-to-back stream-K decode GEMM launches on cold
    weights (us from the first launch's earliest CTA entry)."""
    copies = max(2, math.ceil(3 * 126e6 / (n * k * 2)))
    ws = [torch.randn(n, k, device="cuda", dtype=torch.bfloat16) * 0.02 for _ in range(copies)]
    x = torch.randn(m, k, device="cuda", dtype=torch.bfloat16)
    bufs = [torch.zeros(1024, 8, dtype=torch.int64, device="cuda") for _ in range(2)]
    for w in ws:
        linear(x, w)
    torch.cuda.synchronize()
    native().gemm_set_trace(bufs[0])
    linear(x, ws[0])
    native().gemm_set_trace(bufs[1])
    linear(x, ws[1])
    torch.cuda.synchronize()
    native().gemm_set_trace(None)
    names = ["entry", "setup", "pdl_wait", "first_stage", "last_mma", "epi_done"]
    t0 = bufs[0][bufs[0][:, 0] > 0][:, 0].double().min()
    out = {"kernel": "gemm_trace", "m": m, "n": n, "k": k}
    for i, b in enumerate(bufs):
        t = b[b[:, 0] > 0].double()
        rel = (t[:, :6] - t0) / 1000.0
        out[f"launch{i}"] = {"ctas": int(t.shape[0]),
                             "median": dict(zip(names, [round(v, 2) for v in rel.median(0).values.tolist()])),
                             "min": dict(zip(names, [round(v, 2) for v in rel.min(0).values.tolist()])),
                             "max": dict(zip(names, [round(v, 2) for v in rel.max(0).values.tolist()]))}
    return out


QWEN14B_DECODE = [("qkv", 7168, 5120), ("o_proj", 5120, 5120), ("gate_up", 27648, 5120), ("down", 5120, 13824),
                  ("lm_head", 152064, 5120)]


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("what", choices=["gemm", "nvfp4", "nvfp4-prefill", "fp8", "decode-attn", "all", "trace", "rmsnorm",
                                     "rope-kv", "prefill-attn", "sample", "turboquant", "act-quant", "others", "tq-decode"])
    ap.add_argument("--tokens", type=int, default=None)
    ap.add_argument("--kv-heads", type=int, default=8)
    ap.add_argument("--q-heads", type=int, default=40)
    ap.add_argument("--splits", type=int, default=0)
    ap.add_argument("--fused", action="store_true", help="decode-attn: RoPE + KV write inside the kernel")
    ap.add_argument("--seq", type=int, default=2048)
    ap.add_argument("--greedy", action="store_true")
    ap.add_argument("--m", type=int, default=1)
    ap.add_argument("--n", type=int, default=5120)
    ap.add_argument("--k", type=int, default=13824)
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--ctx", type=int, default=768)
    ap.add_argument("--fp8", action="store_true")
    ap.add_argument("--q4", action="store_true", help="decode-attn / prefill-attn: four-bit KV pages")
    ap.add_argument("--iters", type=int, default=50)
    ap.add_argument("--residual", action="store_true")
    ap.add_argument("--fold", action="store_true", help="gemm: also the folded-norm producer / consumer modes")
    a = ap.parse_args(argv)
    native()
    if a.what == "trace":
        shapes = QWEN14B_DECODE[:4] if (a.n, a.k) == (5120, 13824) else [("custom", a.n, a.k)]
        for name, n, k in shapes:
            r = trace_gemm(a.m, n, k)
            r["name"] = name
            print(json.dumps(r))
    elif a.what == "gemm" and a.fold:
        for m in (1, 32):
            for name, n, k in QWEN14B_DECODE[:4]:
                for mode in ((None, "consumer") if name in ("qkv", "gate_up") else (None, "producer")):
                    r = bench_gemm(m, n, k, a.iters, residual=(mode is None and name in ("o_proj", "down")),
                                   fold=mode)
                    r["name"] = name
                    print(json.dumps(r))
    elif a.what == "gemm":
        print(json.dumps(bench_gemm(a.m, a.n, a.k, a.iters, residual=a.residual)))
    elif a.what == "nvfp4":
        shapes = [(a.n, a.k)] if a.n != 5120 or a.k != 13824 else [(n, k) for _, n, k in QWEN14B_DECODE[:4]]
        for m in ((a.m,) if a.m != 1 else (1, 8, 32)):
            for n, k in shapes:
                print(json.dumps(bench_nvfp4(m, n, k, a.iters)))
    elif a.what == "nvfp4-prefill":
        for n, k in ([(a.n, a.k)] if a.n != 5120 or a.k != 13824 else [(27648, 5120), (5120, 13824), (7168, 5120)]):
            print(json.dumps(bench_nvfp4_prefill(a.m if a.m != 1 else 4096, n, k, a.iters)))
    elif a.what == "tq-decode":
        print(json.dumps(bench_tq_decode(a.batch, a.ctx, kv_heads=a.kv_heads, q_heads=a.q_heads, iters=a.iters)))
    elif a.what == "decode-attn":
        print(json.dumps(bench_decode_attn(a.batch, a.ctx, kv_heads=a.kv_heads, q_heads=a.q_heads, fp8=a.fp8,
                                           iters=a.iters, splits=a.splits, fused=a.fused, q4=a.q4)))
    elif a.what == "fp8":
        for m in ((a.m,) if a.m != 1 else (1, 32, 4096)):
            for name, n, k in QWEN14B_DECODE[:4]:
                r = bench_fp8(m, n, k, a.iters if m < 1024 else 10)
                r["name"] = name
                print(json.dumps(r))
    elif a.what == "rmsnorm":
        print(json.dumps(bench_rmsnorm(a.tokens or a.batch, iters=a.iters)))
    elif a.what == "rope-kv":
        print(json.dumps(bench_rope_kv(a.tokens or a.batch, fp8=a.fp8, iters=a.iters)))
    elif a.what == "prefill-attn":
        print(json.dumps(bench_prefill_attn(a.batch, a.seq, fp8=a.fp8, iters=a.iters, q4=a.q4)))
    elif a.what == "sample":
        print(json.dumps(bench_sample(a.batch, greedy=a.greedy, iters=a.iters)))
    elif a.what == "turboquant":
        print(json.dumps(bench_turboquant(a.tokens or 65536, iters=a.iters)))
    elif a.what == "act-quant":
        print(json.dumps(bench_act_quant(a.tokens or 4096, iters=a.iters)))
    elif a.what == "others":
        for t in (1, 32, 4096):
            print(json.dumps(bench_rmsnorm(t, iters=a.iters)))
        for t in (32, 4096):
            for fp8 in (False, True):
                print(json.dumps(bench_rope_kv(t, fp8=fp8, iters=a.iters)))
        for b, s in ((1, 4096), (4, 2048)):
            for fp8 in (False, True):
                print(json.dumps(bench_prefill_attn(b, s, fp8=fp8, iters=10)))
        for b in (1, 32):
            print(json.dumps(bench_sample(b, greedy=True, iters=a.iters)))
            print(json.dumps(bench_sample(b, iters=a.iters)))
        print(json.dumps(bench_turboquant(65536, iters=20)))
        for t in (32, 4096):
            print(json.dumps(bench_act_quant(t, iters=a.iters)))
    else:
        for m in (1, 32, 512):
            for name, n, k in QWEN14B_DECODE:
                r = bench_gemm(m, n, k, a.iters)
                r["name"] = name
                print(json.dumps(r))
                if name in ("o_proj", "down"):     # the decode step adds the residual in place
                    r = bench_gemm(m, n, k, a.iters, residual=True)
                    r["name"] = name + "+residual"
                    print(json.dumps(r))
        for b in (1, 32):
            for fp8 in (False, True):
                print(json.dumps(bench_decode_attn(b, a.ctx, fp8=fp8, iters=a.iters)))


if __name__ == "__main__":
    main()
