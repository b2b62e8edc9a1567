"""Numerics of every CUDA kernel against the fp32 PyTorch reference of the same op
(the CPU path of vramancer_b200.ops)."""
import math

import pytest
import torch

from vramancer_b200 import ops

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _close(a, b, rtol=2e-2, atol=2e-2):
    a, b = a.float().cpu(), b.float().cpu()
    err = (a - b).abs()
    tol = atol + rtol * b.abs()
    bad = (err > tol).sum().item()
    assert bad == 0, f"{bad} / {a.numel()} out of tolerance, max err {err.max().item():.4g}"


# ------------------------------------------------------------------------- GEMM
@pytest.mark.parametrize("M", [1, 5, 16, 32, 33, 64, 100, 128, 129, 300, 512])
@pytest.mark.parametrize("N,K", [(256, 128), (384, 512), (1000, 320), (2048, 1024)])
def test_gemm(M, N, K, cuda_errors_clean):
    torch.manual_seed(M * 7 + N + K)
    x = torch.randn(M, K) * 0.5
    w = torch.randn(N, K) * 0.05
    b = torch.randn(N) * 0.1
    xg, wg, bg = x.bfloat16().to(DEV), w.bfloat16().to(DEV), b.bfloat16().to(DEV)
    y = ops.linear(xg, wg, bg)
    ref = ops.linear(x.bfloat16(), w.bfloat16(), b.bfloat16())
    _close(y, ref)


@pytest.mark.parametrize("mode", [0, 1, 3, 4, 5])
@pytest.mark.parametrize("M,N,K", [(129, 512, 320), (512, 5120, 1024), (300, 2304, 5120), (1000, 1536, 640),
                                   (2048, 16384, 256), (384, 2560, 8192), (640, 768, 12800)])
def test_gemm_prefill_modes(mode, M, N, K, cuda_errors_clean):
    """Every prefill GEMM kernel (tiled, stream-K, persistent 128- and 256-wide, tiled
    only) against the fp32 reference, with bias + residual and with the SiLU-mul
    epilogue.  Shapes leave partial tiles; in the persistent kernel they give whole-tile
    rounds plus stream-K remainders whose tiles collect 2 to 6 partials (the last two
    shapes), or whole tiles only; the (2048, 16384) and (512, 5120) shapes take the
    default mode's automatic 256-wide persistent kernel."""
    torch.manual_seed(M + N + K + mode)
    x = (torch.randn(M, K) * 0.5).bfloat16()
    w = (torch.randn(N, K) * 0.05).bfloat16()
    b = (torch.randn(N) * 0.1).bfloat16()
    r = torch.randn(M, N).bfloat16()
    ref = ops.linear(x, w, b, residual=r)
    ref_silu = ops.linear(x, w, b, epilogue=ops.EPI_SILU_MUL)
    nat = ops.native()
    nat.gemm_set_prefill_mode(mode)
    try:
        xg, wg, bg = x.to(DEV), w.to(DEV), b.to(DEV)
        y = ops.linear(xg, wg, bg, residual=r.to(DEV))
        y2 = ops.linear(xg, wg, bg, epilogue=ops.EPI_SILU_MUL)
        y3 = ops.linear(xg, wg, bg, residual=r.to(DEV))
    finally:
        nat.gemm_set_prefill_mode(0)
    _close(y, ref)
    _close(y2, ref_silu)
    assert torch.equal(y, y3)      # split tails sum in split order: deterministic


@pytest.mark.parametrize("M", [1, 32, 256])
@pytest.mark.parametrize("splits", [1, 2, 5])
def test_gemm_splitk_deterministic(M, splits, cuda_errors_clean):
    torch.manual_seed(0)
    x = (torch.randn(M, 1280) * 0.5).bfloat16()
    w = (torch.randn(640, 1280) * 0.05).bfloat16()
    ref = ops.linear(x, w)
    y1 = ops.linear(x.to(DEV), w.to(DEV), force_splits=splits)
    y2 = ops.linear(x.to(DEV), w.to(DEV), force_splits=splits)
    _close(y1, ref)
    assert torch.equal(y1, y2), "split-K reduction must be deterministic"


@pytest.mark.parametrize("M", [1, 20, 200])
def test_gemm_silu_and_residual_epilogues(M, cuda_errors_clean):
    torch.manual_seed(1)
    K, I = 512, 384
    x = (torch.randn(M, K) * 0.5).bfloat16()
    wgu = (torch.randn(2 * I, K) * 0.05).bfloat16()
    ref = ops.linear(x, wgu, epilogue=ops.EPI_SILU_MUL)
    y = ops.linear(x.to(DEV), wgu.to(DEV), epilogue=ops.EPI_SILU_MUL)
    _close(y, ref)
    y2 = ops.linear(x.to(DEV), wgu.to(DEV), epilogue=ops.EPI_SILU_MUL, force_splits=3)
    _close(y2, ref)
    w = (torch.randn(K, K) * 0.05).bfloat16()
    r = (torch.randn(M, K)).bfloat16()
    ref_r = ops.linear(x, w, residual=r)
    rg = r.to(DEV)
    ops.linear(x.to(DEV), w.to(DEV), residual=rg, out=rg)   # in-place residual stream update
    _close(rg, ref_r)


@pytest.mark.parametrize("M", [1, 32])
@pytest.mark.parametrize("N,K,epi", [(896, 5120, "bias"), (3456, 5120, "silu"), (5120, 640, "residual"),
                                     (5120, 1728, "ssq")])
def test_gemm_tp_shard_shapes(M, N, K, epi, cuda_errors_clean):
    """Decode GEMMs of tensor-parallel shard shapes, whose tiles split over 2..8 CTAs of
    one thread-block cluster (fixup through distributed shared memory): every epilogue
    kind against the fp32 reference, and bitwise the same on a second call."""
    torch.manual_seed(M + N + K)
    x = (torch.randn(M, K) * 0.5).bfloat16()
    w = (torch.randn(N, K) * 0.05).bfloat16()
    b = (torch.randn(N) * 0.1).bfloat16()
    xg, wg, bg = x.to(DEV), w.to(DEV), b.to(DEV)
    if epi == "bias":
        ref, got = ops.linear(x, w, b), [ops.linear(xg, wg, bg) for _ in range(2)]
    elif epi == "silu":
        ref = ops.linear(x, w, epilogue=ops.EPI_SILU_MUL)
        got = [ops.linear(xg, wg, epilogue=ops.EPI_SILU_MUL) for _ in range(2)]
    else:
        r = torch.randn(M, N).bfloat16()
        ref = ops.linear(x, w, residual=r)
        got = []
        for _ in range(2):
            rg = r.to(DEV)
            buf = torch.zeros((N + 127) // 128, 128, device=DEV) if epi == "ssq" else None
            ops.linear(xg, wg, residual=rg, out=rg, ssq_out=buf)
            got.append(rg)
            if buf is not None:
                want = (rg.float() ** 2).view(M, -1, 128).sum(-1).t()
                _close(buf[:, :M], want, rtol=1e-5, atol=1e-3)
    _close(got[0], ref)
    assert torch.equal(got[0], got[1])


# ------------------------------------------------------------------------- norms
@pytest.mark.parametrize("H", [128, 768, 3584, 5120])
@pytest.mark.parametrize("with_res", [False, True])
def test_rmsnorm_layernorm(H, with_res, cuda_errors_clean):
    torch.manual_seed(H)
    x = torch.randn(7, H).bfloat16()
    r = torch.randn(7, H).bfloat16() if with_res else None
    w = (1 + 0.1 * torch.randn(H)).bfloat16()
    b = (0.1 * torch.randn(H)).bfloat16()
    rc = r.clone() if r is not None else None
    ref = ops.rmsnorm(x, w, 1e-6, residual=rc)
    rg = r.to(DEV) if r is not None else None
    y = ops.rmsnorm(x.to(DEV), w.to(DEV), 1e-6, residual=rg)
    _close(y, ref)
    if r is not None:
        _close(rg, rc, rtol=1e-2, atol=1e-2)
    rc2 = r.clone() if r is not None else None
    ref2 = ops.layernorm(x, w, b, 1e-5, residual=rc2)
    rg2 = r.to(DEV) if r is not None else None
    y2 = ops.layernorm(x.to(DEV), w.to(DEV), b.to(DEV), 1e-5, residual=rg2)
    _close(y2, ref2)


# ------------------------------------------------------------------------- rope + kv write
@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("D", [64, 128])
def test_rope_kv_write(fp8, D, cuda_errors_clean):
    torch.manual_seed(D)
    T, Hq, KH, L, P = 9, 6, 2, 3, 8
    qkv = torch.randn(T, (Hq + 2 * KH) * D).bfloat16()
    pos = torch.randint(0, 500, (T,), dtype=torch.int32)
    cs = ops.rope_cos_sin(512, D, 10000.0)
    slots = torch.randperm(P * 16)[:T].to(torch.int32)
    slots[3] = -1
    dt = torch.float8_e4m3fn if fp8 else torch.bfloat16
    scale = (torch.rand(L, 2, KH) + 0.5) / 100 if fp8 else None
    cache_c = torch.zeros(P, L, 2, KH, 16, D, dtype=dt)
    q_c = qkv.clone()
    ops.rope_kv_write(q_c, pos, cs, cache_c, slots, scale, 1, Hq, KH, D)
    cache_g = cache_c.clone().zero_().to(DEV)
    q_g = qkv.to(DEV)
    ops.rope_kv_write(q_g, pos.to(DEV), cs.to(DEV), cache_g, slots.to(DEV),
                      scale.to(DEV) if scale is not None else None, 1, Hq, KH, D)
    _close(q_g, q_c)
    _close(cache_g.float(), cache_c.float(), rtol=7e-2, atol=2e-2)


@pytest.mark.parametrize("M", [1, 7, 32, 100])
def test_gemm_folded_norm_producer(M, cuda_errors_clean):
    """A residual GEMM that also stores per-(128-feature tile, token) sums of squares of
    its bf16 output: same output bits as without, sums equal to the fp32 reference."""
    torch.manual_seed(M)
    K, N = 512, 640
    x = torch.randn(M, K, device=DEV).bfloat16()
    w = (torch.randn(N, K, device=DEV) * 0.05).bfloat16()
    r = torch.randn(M, N, device=DEV).bfloat16()
    ref = r.clone()
    ops.linear(x, w, residual=ref, out=ref)
    out = r.clone()
    buf = torch.full((8, 128), -1.0, device=DEV)
    ops.linear(x, w, residual=out, out=out, ssq_out=buf)
    torch.cuda.synchronize()
    assert torch.equal(out, ref)
    want = (out.float() ** 2).view(M, 5, 128).sum(-1).t()
    _close(buf[:5, :M], want, rtol=1e-5, atol=1e-4)


@pytest.mark.parametrize("M", [1, 16, 48, 128])
@pytest.mark.parametrize("silu", [False, True])
def test_gemm_folded_norm_consumer(M, silu, cuda_errors_clean):
    """GEMM on the raw residual stream scaled per token by rsqrt(mean of squares + eps)
    from partial sums (the folded RMSNorm) against the fp32 reference."""
    torch.manual_seed(M + 3 * silu)
    K, N = 640, 768
    h = (torch.randn(M, K) * 2).bfloat16()
    w = (torch.randn(N, K) * 0.05).bfloat16()
    b = None if silu else (torch.randn(N) * 0.1).bfloat16()
    buf = torch.zeros(8, 128)
    buf[:5, :M] = (h.float() ** 2).view(M, 5, 128).sum(-1).t()
    epi = ops.EPI_SILU_MUL if silu else ops.EPI_NONE
    ref = ops.linear(h, w, b, epilogue=epi, ssq_in=buf, ssq_parts=5, norm_eps=1e-6)
    got = ops.linear(h.to(DEV), w.to(DEV), b.to(DEV) if b is not None else None, epilogue=epi,
                     ssq_in=buf.to(DEV), ssq_parts=5, norm_eps=1e-6)
    _close(got, ref)
    # the same as RMSNorm (weight 1) followed by the plain GEMM
    xn = ops.rmsnorm(h.to(DEV), torch.ones(K, device=DEV).bfloat16(), 1e-6)
    _close(got, ops.linear(xn, w.to(DEV), b.to(DEV) if b is not None else None, epilogue=epi))


def test_folded_norm_decode_logits(cuda_errors_clean):
    """A model whose RMSNorms run inside the decode GEMMs (folded weights, norm sums
    from the residual GEMMs) gives the logits of the same model with standalone norm
    kernels: prefill (norms without weight + folded weights) and a decode step."""
    from vramancer_b200.kv.pool import KVPool, KVPoolSpec
    from vramancer_b200.models.config import PRESETS
    from vramancer_b200.models.transformer import DecoderModel, ForwardBatch
    from vramancer_b200.models.weights import random_weights
    cfg = PRESETS["tiny-qwen2-d128"]
    lens = [5, 20, 33]
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in lens]
    i32 = lambda v: torch.tensor(v, dtype=torch.int32, device=DEV)   # noqa: E731

    def run(fold):
        w = random_weights(cfg, device=DEV, dtype=torch.bfloat16, seed=11)
        model = DecoderModel(cfg, w, device=DEV, dtype=torch.bfloat16)
        if fold:
            assert model.fold_norms()
        pool = KVPool(KVPoolSpec(16, cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, dtype=torch.bfloat16), DEV)
        bt = [[4 * b + j for j in range(4)] for b in range(3)]
        ids, pos, slots, cu = [], [], [], [0]
        for b, p in enumerate(prompts):
            ids += p
            pos += list(range(len(p)))
            slots += [bt[b][t // 16] * 16 + t % 16 for t in range(len(p))]
            cu.append(cu[-1] + len(p))
        pre = ForwardBatch(input_ids=i32(ids), positions=i32(pos), slot_mapping=i32(slots), block_tables=i32(bt),
                           context_lens=i32(lens), is_decode=False, cu_q=i32(cu), max_q_len=max(lens),
                           logits_rows=torch.tensor([c - 1 for c in cu[1:]], device=DEV))
        lp = model.forward(pre, pool).float()
        dec = ForwardBatch(input_ids=i32([7, 8, 9]), positions=i32(lens),
                           slot_mapping=i32([bt[b][n // 16] * 16 + n % 16 for b, n in enumerate(lens)]),
                           block_tables=i32(bt), context_lens=i32([n + 1 for n in lens]), is_decode=True,
                           attn_splits=0)
        ld = model.forward(dec, pool).float()
        return lp, ld, model.folded

    lp0, ld0, f0 = run(False)
    lp1, ld1, f1 = run(True)
    assert not f0 and f1
    scale = ld0.abs().max().item()
    _close(lp1, lp0, rtol=0.0, atol=0.03 * scale)
    _close(ld1, ld0, rtol=0.0, atol=0.03 * scale)
    assert (ld1 - ld0).abs().mean().item() < 0.005 * scale


# ------------------------------------------------------------------------- attention
def _make_cache(lens, L, KH, D, dt, layer, seed=0):
    torch.manual_seed(seed)
    ps = 16
    pages_per = [(n + ps - 1) // ps for n in lens]
    P = sum(pages_per) + 3
    perm = torch.randperm(P)
    bt = torch.zeros(len(lens), max(pages_per) + 1, dtype=torch.int32)
    k = 0
    for b, n in enumerate(pages_per):
        bt[b, :n] = perm[k:k + n].to(torch.int32)
        k += n
    cache = (torch.randn(P, L, 2, KH, ps, D) * 1.5)
    scale = None
    if dt == torch.float8_e4m3fn:
        scale = (torch.rand(L, 2, KH) + 0.5) / 50
        cache = (cache / scale.view(1, L, 2, KH, 1, 1)).clamp(-448, 448).to(dt)
    else:
        cache = cache.to(dt)
    return cache, bt, scale


@pytest.mark.parametrize("D,Hq,KH", [(128, 40, 8), (128, 28, 4), (64, 12, 12), (128, 32, 4)])
@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("splits", [0, 1, 3])
def test_paged_decode(D, Hq, KH, fp8, splits, cuda_errors_clean):
    lens = [1, 17, 300, 64, 1033]
    L, layer = 2, 1
    dt = torch.float8_e4m3fn if fp8 else torch.bfloat16
    cache, bt, scale = _make_cache(lens, L, KH, D, dt, layer, seed=D + Hq)
    B = len(lens)
    q = torch.randn(B, (Hq + 2 * KH) * D).bfloat16()     # q is a strided view of qkv rows
    cl = torch.tensor(lens, dtype=torch.int32)
    sm = 1.0 / math.sqrt(D)
    ref = ops.paged_attention_decode(q, cache, layer, bt, cl, scale, sm, Hq)
    out = ops.paged_attention_decode(q.to(DEV), cache.to(DEV), layer, bt.to(DEV), cl.to(DEV),
                                     scale.to(DEV) if scale is not None else None, sm, Hq, num_splits=splits)
    _close(out, ref, rtol=3e-2, atol=3e-2)


@pytest.mark.parametrize("D,Hq,KH,rope", [(128, 40, 8, True), (128, 28, 4, True), (64, 12, 12, False)])
@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("splits", [0, 1, 3])
def test_paged_decode_fused_rope_kv_write(D, Hq, KH, rope, fp8, splits, cuda_errors_clean):
    """Decode attention that also rotates q / k and writes this step's k / v into the
    cache gives the same bits (output and cache) as the standalone RoPE + KV write
    kernel followed by decode attention.  Row 2 is a padded row (no context, slot -1)."""
    lens = [1, 17, 0, 300, 64, 1033]
    L, layer = 2, 1
    dt = torch.float8_e4m3fn if fp8 else torch.bfloat16
    cache, bt, scale = _make_cache([max(n, 1) for n in lens], L, KH, D, dt, layer, seed=D + Hq + 7)
    B = len(lens)
    g = torch.Generator().manual_seed(splits)
    qkv = torch.randn(B, (Hq + 2 * KH) * D, generator=g).bfloat16()
    cl = torch.tensor(lens, dtype=torch.int32)
    pos = torch.tensor([max(n - 1, 0) for n in lens], dtype=torch.int32)
    slots = torch.tensor([int(bt[b, (n - 1) // 16]) * 16 + (n - 1) % 16 if n > 0 else -1
                          for b, n in enumerate(lens)], dtype=torch.int32)
    cs = ops.rope_cos_sin(2048, D, 1e6, device=DEV) if rope else None
    sm = 1.0 / math.sqrt(D)
    d = lambda t: t.to(DEV) if t is not None else None   # noqa: E731
    # standalone kernels
    c1, q1 = d(cache).clone(), d(qkv).clone()
    ops.rope_kv_write(q1, d(pos), cs, c1, d(slots), d(scale), layer, Hq, KH, D)
    o1 = ops.paged_attention_decode(q1, c1, layer, d(bt), d(cl), d(scale), sm, Hq, num_splits=splits)
    # fused
    c2, q2 = d(cache).clone(), d(qkv).clone()
    o2 = ops.paged_attention_decode(q2, c2, layer, d(bt), d(cl), d(scale), sm, Hq, num_splits=splits,
                                    positions=d(pos), cos_sin=cs, slot_mapping=d(slots))
    torch.cuda.synchronize()
    assert torch.equal(c1.view(torch.uint8), c2.view(torch.uint8))
    assert torch.equal(o1[[0, 1, 3, 4, 5]], o2[[0, 1, 3, 4, 5]])
    assert torch.equal(q2, d(qkv))            # the fused kernel leaves the qkv rows as they were


@pytest.mark.parametrize("splits", [0, 2, 7])
@pytest.mark.parametrize("tma", [False, True])
def test_paged_decode_many_sequences(splits, tma, cuda_errors_clean):
    """Many sequences; with the persistent TMA kernel many (sequence, head, chunk) items
    per CTA: its page ring runs across item boundaries and chunks of one sequence land
    on different CTAs."""
    ops.native().set_decode_tma(tma)
    try:
        _many_sequences(splits)
    finally:
        ops.native().set_decode_tma(False)


def _many_sequences(splits):
    g = torch.Generator().manual_seed(splits)
    lens = torch.randint(1, 700, (70,), generator=g).tolist()
    D, Hq, KH, L, layer = 128, 40, 8, 2, 0
    cache, bt, scale = _make_cache(lens, L, KH, D, torch.bfloat16, layer, seed=3)
    B = len(lens)
    q = torch.randn(B, (Hq + 2 * KH) * D, generator=g).bfloat16()
    cl = torch.tensor(lens, dtype=torch.int32)
    sm = 1.0 / math.sqrt(D)
    ref = ops.paged_attention_decode(q, cache, layer, bt, cl, scale, sm, Hq)
    dq, dc, dbt, dcl = q.to(DEV), cache.to(DEV), bt.to(DEV), cl.to(DEV)
    if splits == 2:
        # also the small-batch shapes (bs 1 and 8) through the same kernel
        for nb in (1, 8):
            r1 = ops.paged_attention_decode(q[:nb], cache, layer, bt[:nb], cl[:nb], scale, sm, Hq)
            o1 = ops.paged_attention_decode(dq[:nb], dc, layer, dbt[:nb], dcl[:nb], None, sm, Hq)
            _close(o1, r1, rtol=3e-2, atol=3e-2)
    out = ops.paged_attention_decode(dq, dc, layer, dbt, dcl, None, sm, Hq, num_splits=splits)
    _close(out, ref, rtol=3e-2, atol=3e-2)
    again = ops.paged_attention_decode(dq, dc, layer, dbt, dcl, None, sm, Hq, num_splits=splits)
    assert torch.equal(out, again)     # chunk merges are in chunk order: deterministic


@pytest.mark.parametrize("D,Hq,KH", [(128, 40, 8), (64, 12, 12)])
@pytest.mark.parametrize("fp8", [False, True])
def test_paged_prefill(D, Hq, KH, fp8, cuda_errors_clean):
    # (new tokens, total context) per sequence: plain prefill and chunked prefill with prefix
    specs = [(5, 5), (64, 64), (70, 200), (130, 130), (1, 40)]
    L, layer = 2, 0
    dt = torch.float8_e4m3fn if fp8 else torch.bfloat16
    cache, bt, scale = _make_cache([s[1] for s in specs], L, KH, D, dt, layer, seed=D)
    cu = [0]
    for ql, _ in specs:
        cu.append(cu[-1] + ql)
    T = cu[-1]
    q = torch.randn(T, Hq * D).bfloat16()
    cu_q = torch.tensor(cu, dtype=torch.int32)
    cl = torch.tensor([s[1] for s in specs], dtype=torch.int32)
    sm = 1.0 / math.sqrt(D)
    mq = max(s[0] for s in specs)
    ref = ops.paged_attention_prefill(q, cache, layer, bt, cu_q, cl, scale, sm, Hq, mq)
    out = ops.paged_attention_prefill(q.to(DEV), cache.to(DEV), layer, bt.to(DEV), cu_q.to(DEV), cl.to(DEV),
                                      scale.to(DEV) if scale is not None else None, sm, Hq, mq)
    _close(out, ref, rtol=3e-2, atol=3e-2)


@pytest.mark.parametrize("D,Hq,KH", [(128, 40, 8), (128, 16, 16), (64, 12, 4)])
def test_paged_prefill_tc_matches_warp_mma(D, Hq, KH, cuda_errors_clean):
    """The tcgen05 prefill kernel (bf16 pages) against the fp32 reference and the
    warp-MMA kernel: multi-block causal rows, chunked prefill behind a cached prefix,
    partial tiles and pages, GQA groups."""
    specs = [(300, 300), (1, 700), (129, 129), (200, 1000), (64, 64), (513, 600)]
    L, layer = 2, 1
    cache, bt, _ = _make_cache([s[1] for s in specs], L, KH, D, torch.bfloat16, layer, seed=D + Hq)
    cu = [0]
    for ql, _ in specs:
        cu.append(cu[-1] + ql)
    q = torch.randn(cu[-1], (Hq + 2 * KH) * D).bfloat16()      # q rows of a qkv buffer (strided)
    cu_q = torch.tensor(cu, dtype=torch.int32)
    cl = torch.tensor([s[1] for s in specs], dtype=torch.int32)
    sm = 1.0 / math.sqrt(D)
    mq = max(s[0] for s in specs)
    ref = ops.paged_attention_prefill(q, cache, layer, bt, cu_q, cl, None, sm, Hq, mq)
    args = (q.to(DEV), cache.to(DEV), layer, bt.to(DEV), cu_q.to(DEV), cl.to(DEV), None, sm, Hq, mq)
    nat = ops.native()
    nat.set_prefill_tc(True)
    try:
        tc = ops.paged_attention_prefill(*args)
    finally:
        nat.set_prefill_tc(False)
    mma = ops.paged_attention_prefill(*args)
    _close(tc, ref, rtol=3e-2, atol=3e-2)
    _close(tc, mma, rtol=3e-2, atol=3e-2)


# ------------------------------------------------------------------------- elementwise + sampling
def test_elementwise(cuda_errors_clean):
    torch.manual_seed(3)
    x = torch.randn(5, 2 * 264).bfloat16()
    _close(ops.silu_mul(x.to(DEV)), ops.silu_mul(x))
    g = torch.randn(1000).bfloat16()
    _close(ops.gelu_tanh_(g.clone().to(DEV)), ops.gelu_tanh_(g.clone()))
    table = torch.randn(100, 64).bfloat16()
    pt = torch.randn(50, 64).bfloat16()
    ids = torch.randint(0, 100, (9,), dtype=torch.int32)
    pos = torch.randint(0, 50, (9,), dtype=torch.int32)
    ref = ops.embedding(ids, table, positions=pos, pos_table=pt)
    out = ops.embedding(ids.to(DEV), table.to(DEV), positions=pos.to(DEV), pos_table=pt.to(DEV))
    _close(out, ref)


@pytest.mark.parametrize("V", [500, 50257, 152064])
def test_argmax_and_sampling(V, cuda_errors_clean):
    torch.manual_seed(V)
    B = 6
    logits = (torch.randn(B, V) * 3).bfloat16()
    ref = torch.argmax(logits.float(), -1).to(torch.int32)
    lg = logits.to(DEV)
    assert torch.equal(ops.argmax(lg).cpu(), ref)
    z = torch.zeros(B, dtype=torch.float32, device=DEV)
    k0 = torch.zeros(B, dtype=torch.int32, device=DEV)
    p1 = torch.ones(B, dtype=torch.float32, device=DEV)
    st = torch.arange(B, dtype=torch.int32, device=DEV)
    assert torch.equal(ops.sample(lg, z, k0, p1, 1, st).cpu(), ref)          # T=0 -> greedy
    t1 = torch.ones(B, device=DEV)
    assert torch.equal(ops.sample(lg, t1, torch.ones(B, dtype=torch.int32, device=DEV), p1, 7, st).cpu(), ref)
    # top-k = 5: every draw must be one of the 5 largest logits
    k5 = torch.full((B,), 5, dtype=torch.int32, device=DEV)
    top5 = torch.topk(logits.float(), 5, dim=-1).indices
    for s in range(20):
        ids = ops.sample(lg, t1, k5, p1, 100 + s, st).cpu()
        for b in range(B):
            assert int(ids[b]) in top5[b].tolist()
    # top-p = tiny: nucleus is the argmax
    pp = torch.full((B,), 1e-4, dtype=torch.float32, device=DEV)
    assert torch.equal(ops.sample(lg, t1, k0, pp, 3, st).cpu(), ref)
    # unrestricted sampling frequencies follow softmax on a small vocabulary
    if V == 500:
        lg1 = torch.zeros(1, 500)
        lg1[0, :4] = torch.tensor([2.0, 1.0, 0.5, 0.0])
        lg1[0, 4:] = -30
        lgd = lg1.bfloat16().to(DEV)
        counts = torch.zeros(4)
        for s in range(2000):
            i = int(ops.sample(lgd, t1[:1], k0[:1], p1[:1], 1000 + s, st[:1]))
            counts[i] += 1
        freq = counts / counts.sum()
        pref = torch.softmax(torch.tensor([2.0, 1.0, 0.5, 0.0]), 0)
        assert (freq - pref).abs().max() < 0.04


# ------------------------------------------------------------------------- MoE (device path)
def _moe_fp32_reference(x, ids, w, gu, dn, add=None):
    """Plain fp32 MoE over given routing: sum_k w[t,k] * down_e(silu(gate_e x) * up_e x)."""
    T, H = x.shape
    out = torch.zeros(T, H)
    for t in range(T):
        for k in range(ids.shape[1]):
            e = int(ids[t, k])
            y = gu[e] @ x[t]
            h = torch.nn.functional.silu(y[0::2]) * y[1::2]
            out[t] += float(w[t, k]) * (dn[e] @ h)
    return out if add is None else out + add


@pytest.mark.parametrize("T,E,topk,BN", [(7, 128, 8, 16), (64, 16, 4, 32), (300, 8, 2, 128), (1, 4, 1, 16)])
def test_moe_plan(T, E, topk, BN, cuda_errors_clean):
    g = torch.Generator().manual_seed(T)
    ids = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(T)]).to(DEV)
    counts, offsets, row_of, tok, blocks, nblk = ops.native().moe_plan(ids, E, BN)
    flat = ids.flatten().cpu()
    c_ref = torch.bincount(flat, minlength=E)
    off_ref = torch.cat([torch.zeros(1, dtype=torch.long), c_ref.cumsum(0)])
    assert torch.equal(counts.cpu().long(), c_ref) and torch.equal(offsets.cpu().long(), off_ref)
    ro, tk = row_of.cpu().long(), tok.cpu().long()
    assert sorted(ro.tolist()) == list(range(T * topk))
    for p in range(T * topk):
        assert off_ref[flat[p]] <= ro[p] < off_ref[flat[p] + 1] and tk[ro[p]] == p // topk
    want = [[e, int(off_ref[e]) + r0, min(BN, int(c_ref[e]) - r0)] for e in range(E) for r0 in range(0, int(c_ref[e]), BN)]
    assert blocks.cpu()[:int(nblk.item()), :3].tolist() == want


@pytest.mark.parametrize("T,E,topk", [(1, 8, 2), (128, 128, 8), (300, 64, 4), (77, 256, 8), (5, 1000, 3),
                                      (129, 16, 1)])
def test_moe_route_matches_torch(T, E, topk, cuda_errors_clean):
    """Device softmax / top-k / renormalisation (fused with the plan up to 128 tokens)
    against torch in fp32 on the same bf16 logits."""
    g = torch.Generator().manual_seed(T * E)
    logits = (torch.randn(T, E, generator=g) * 2).to(DEV, torch.bfloat16)
    ids, w, counts, offsets, row_of, tok, blocks, nblk = ops.native().moe_route(logits, topk, True, 16)
    probs = torch.softmax(logits.float(), -1)
    rw, rids = torch.topk(probs, topk, dim=-1)
    rw = rw / rw.sum(-1, keepdim=True)
    same = ids == rids
    if not bool(same.all()):
        # only exact ties (bf16 logits) may order differently
        pv = probs.gather(1, ids)
        assert torch.allclose(pv, probs.gather(1, rids), rtol=0, atol=1e-7)
    torch.testing.assert_close(w.sort(-1).values, rw.sort(-1).values, rtol=1e-5, atol=1e-6)
    c_ref = torch.bincount(ids.flatten().cpu(), minlength=E)
    assert torch.equal(counts.cpu().long(), c_ref)
    ro = row_of.cpu().long()
    assert sorted(ro.tolist()) == list(range(T * topk))
    assert torch.equal(tok.cpu().long()[ro], torch.arange(T * topk) // topk)
    off = torch.cat([torch.zeros(1, dtype=torch.long), c_ref.cumsum(0)])
    want = [[e, int(off[e]) + r0, min(16, int(c_ref[e]) - r0)] for e in range(E) for r0 in range(0, int(c_ref[e]), 16)]
    assert blocks.cpu()[:int(nblk.item()), :3].tolist() == want


def test_moe_layer_fused_residual_norm(cuda_errors_clean):
    """r += MoE(x) in place and the next RMSNorm, fused into the combine."""
    from vramancer_b200.models.config import get_config
    from vramancer_b200.parallel import moe
    T, E, topk, H, I = 48, 32, 4, 1024, 256
    cfg = get_config("tiny-moe").with_(hidden_size=H, num_experts=E, experts_per_token=topk,
                                       expert_intermediate_size=I)
    g = torch.Generator().manual_seed(5)
    bf = lambda t: t.to(DEV, torch.bfloat16)  # noqa: E731
    x, router = bf(torch.randn(T, H, generator=g) * 0.5), bf(torch.randn(E, H, generator=g) * 0.05)
    gu, dn = bf(torch.randn(E, 2 * I, H, generator=g) * 0.03), bf(torch.randn(E, H, I, generator=g) * 0.03)
    r0, nw = bf(torch.randn(T, H, generator=g)), bf(torch.rand(H, generator=g) + 0.5)
    y = moe.moe_forward(cfg, x, router, gu, dn).float()
    r = r0.clone()
    xn = moe.moe_forward(cfg, x, router, gu, dn, residual=r, norm_w=nw)
    r_ref = r0.float() + y
    _close(r, r_ref, rtol=2e-2, atol=2e-2)
    rr = r.float()
    xn_ref = rr * torch.rsqrt(rr.pow(2).mean(-1, keepdim=True) + cfg.norm_eps) * nw.float()
    _close(xn, xn_ref, rtol=2e-2, atol=2e-2)
    r2 = r0.clone()
    assert moe.moe_forward(cfg, x, router, gu, dn, residual=r2) is None
    assert torch.equal(r2, r)


@pytest.mark.parametrize("epi", [0, 1])
def test_moe_grouped_linear(epi, cuda_errors_clean):
    """The grouped GEMM over a plan against a per-row fp32 product with that row's expert."""
    T, E, topk, H, N, BN = 40, 16, 4, 512, 384, 16
    g = torch.Generator().manual_seed(3)
    ids = torch.stack([torch.randperm(E, generator=g)[:topk] for _ in range(T)]).to(DEV)
    _, offsets, _, _, blocks, nblk = ops.native().moe_plan(ids, E, BN)
    P = T * topk
    xp = (torch.randn(P + BN, H, generator=g) * 0.5).to(DEV, torch.bfloat16)
    w = (torch.randn(E, N, H, generator=g) * 0.05).to(DEV, torch.bfloat16)
    out = ops.native().moe_grouped_linear(xp, w, blocks, nblk, BN, epi)
    off = offsets.cpu().tolist()
    for e in range(E):
        y = xp[off[e]:off[e + 1]].float() @ w[e].float().t()
        if epi == 1:
            y = torch.nn.functional.silu(y[:, 0::2]) * y[:, 1::2]
        _close(out[off[e]:off[e + 1]], y, rtol=2e-2, atol=2e-2)


@pytest.mark.parametrize("T,E,topk,H,I", [(1, 8, 2, 256, 128), (32, 64, 8, 1024, 384), (200, 16, 4, 512, 256),
                                         (7, 128, 8, 2048, 768)])
def test_moe_device_matches_fp32(T, E, topk, H, I, cuda_errors_clean):
    from vramancer_b200.models.config import get_config
    from vramancer_b200.parallel import moe
    cfg = get_config("tiny-moe").with_(hidden_size=H, num_experts=E, experts_per_token=topk,
                                       expert_intermediate_size=I)
    torch.manual_seed(T + E)
    bf = lambda t: t.bfloat16().to(DEV)  # noqa: E731
    x, router = bf(torch.randn(T, H) * 0.5), bf(torch.randn(E, H) * 0.05)
    gu, dn = bf(torch.randn(E, 2 * I, H) * 0.03), bf(torch.randn(E, H, I) * 0.03)
    sgu, sdn, sg = bf(torch.randn(2 * I, H) * 0.03), bf(torch.randn(H, I) * 0.03), bf(torch.randn(1, H) * 0.05)
    w, ids = moe.route(cfg, x, router)
    assert bool(((ids >= 0) & (ids < E)).all())
    c = lambda t: t.float().cpu()  # noqa: E731
    got = moe.moe_forward(cfg, x, router, gu, dn)
    torch.cuda.synchronize()
    ref = _moe_fp32_reference(c(x), c(ids), c(w), c(gu), c(dn))
    _close(got, ref, rtol=3e-2, atol=3e-2)
    # with the gated shared expert folded into the combine
    shared = moe.expert_mlp(x, sgu, sdn).float() * torch.sigmoid(ops.linear(x, sg).float())
    got_s = moe.moe_forward(cfg, x, router, gu, dn, shared_gate_up=sgu, shared_down=sdn, shared_gate=sg)
    _close(got_s, ref + c(shared), rtol=3e-2, atol=3e-2)
    # repeated calls give identical bits (grouped row order may vary, the sums do not)
    assert torch.equal(moe.moe_forward(cfg, x, router, gu, dn), got)


def test_moe_back_to_back_calls(cuda_errors_clean):
    """Many MoE layers of changing shapes back to back, no synchronisation between them:
    the plan is read up to four kernels after it is written by grids launched early
    (programmatic dependent launch), which must still see the finished plan."""
    from vramancer_b200.models.config import get_config
    from vramancer_b200.parallel import moe
    g = torch.Generator().manual_seed(11)
    outs = []
    for i, (T, E, topk, H, I) in enumerate([(7, 128, 8, 1024, 768), (7, 128, 8, 2048, 384), (33, 64, 4, 512, 256),
                                            (1, 128, 8, 1024, 384), (96, 16, 2, 512, 128)] * 3):
        cfg = get_config("tiny-moe").with_(hidden_size=H, num_experts=E, experts_per_token=topk,
                                           expert_intermediate_size=I)
        x = (torch.randn(T, H, generator=g) * 0.5).to(DEV, torch.bfloat16)
        router = (torch.randn(E, H, generator=g) * 0.05).to(DEV, torch.bfloat16)
        gu = (torch.randn(E, 2 * I, H, generator=g) * 0.03).to(DEV, torch.bfloat16)
        dn = (torch.randn(E, H, I, generator=g) * 0.03).to(DEV, torch.bfloat16)
        w, ids = moe.route(cfg, x, router)
        outs.append((moe.moe_forward(cfg, x, router, gu, dn), x, ids, w, gu, dn))
    torch.cuda.synchronize()
    for got, x, ids, w, gu, dn in outs:
        y = torch.einsum("tkoh,th->tko", gu[ids].float(), x.float())
        h = torch.nn.functional.silu(y[..., 0::2]) * y[..., 1::2]
        ref = (torch.einsum("tkhi,tki->tkh", dn[ids].float(), h) * w.unsqueeze(-1)).sum(1)
        _close(got, ref, rtol=3e-2, atol=3e-2)


def test_moe_model_decodes_under_cuda_graphs(cuda_errors_clean):
    from vramancer_b200.engine.engine import SamplingParams
    from vramancer_b200.llm import LLM
    kw = dict(device="cuda:0", max_batch=4, max_model_len=128, kv_pages=64, seed=2)
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (5, 23, 40)]
    eager = LLM("tiny-moe", use_cuda_graph=False, **kw)
    want = [o.output_ids for o in eager.generate(prompts, SamplingParams(max_tokens=8))]
    graph = LLM("tiny-moe", use_cuda_graph=True, **kw)
    assert graph.runner.use_graph
    got = [o.output_ids for o in graph.generate(prompts, SamplingParams(max_tokens=8))]
    assert got == want
    graph.runner.release_graphs()
