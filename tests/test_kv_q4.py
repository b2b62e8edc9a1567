"""Four-bit KV pages: the row format's host oracle, the CPU paths of the KV write and
attention over a uint8 pool, the engine on a four-bit pool, and (GPU) the CUDA kernels
against the fp32 reference over the same stored rows."""
import math

import pytest
import torch

from vramancer_b200 import ops
from vramancer_b200.engine.engine import SamplingParams
from vramancer_b200.kv import q4
from vramancer_b200.kv.pool import KVPool, KVPoolSpec, kv_dtype_from_str
from vramancer_b200.llm import LLM
from vramancer_b200.models.config import PRESETS
from vramancer_b200.models.transformer import DecoderModel, ForwardBatch
from vramancer_b200.models.weights import random_weights

DEV = "cuda"


# ------------------------------------------------------------------------- format (CPU)
@pytest.mark.parametrize("D", [64, 128])
def test_q4_roundtrip_error_bound(D):
    g = torch.Generator().manual_seed(D)
    x = torch.randn(7, 3, D, generator=g) * 4 + 1
    rows = q4.quantize(x)
    assert rows.dtype == torch.uint8 and rows.shape == (7, 3, q4.row_bytes(D))
    y = q4.dequantize(rows)
    grp = x.view(7, 3, D // 32, 32)
    step = (grp.amax(-1) - grp.amin(-1)) / 15
    err = (y - x).abs().view(7, 3, D // 32, 32).amax(-1)
    # half a step, plus the fp16 rounding of scale and min
    assert bool((err <= 0.5 * step * 1.01 + 1e-3 * grp.abs().amax(-1)).all())


def test_q4_layout():
    """Element 2i in the low nibble of byte i; the group's fp16 (scale, min) after the codes."""
    x = torch.arange(64, dtype=torch.float32).view(1, 64)   # group 0: 0..31, group 1: 32..63
    r = q4.quantize(x)[0]
    sm = r[32:].view(torch.float16).float()
    s = float(torch.tensor(31 / 15).half())
    assert sm.tolist() == [s, 0.0, s, 32.0]
    assert int(r[0]) & 15 == 0 and int(r[15]) >> 4 == 15     # codes of x = 0 and x = 31
    const = q4.dequantize(q4.quantize(torch.full((2, 128), -3.25)))
    assert torch.equal(const, torch.full((2, 128), -3.25))


def test_pool_spec_q4():
    assert kv_dtype_from_str("q4") == torch.uint8
    spec = KVPoolSpec(4, 48, 8, 128, dtype=torch.uint8)
    bf = KVPoolSpec(4, 48, 8, 128, dtype=torch.bfloat16)
    assert spec.row == 80 and spec.bytes_per_page * 16 == bf.bytes_per_page * 5
    pool = KVPool(spec)
    assert pool.cache.shape == (4, 48, 2, 8, 16, 80) and pool.kv_scale is None
    assert ops.cache_head_dim(pool.cache) == 128


def test_q4_cpu_write_and_decode_match_dequantized_pool():
    """rope_kv_write into a uint8 pool then decode attention equals decode attention over
    the dequantised pool (the same values in fp32)."""
    torch.manual_seed(0)
    D, Hq, KH, L, P, T = 64, 4, 2, 2, 6, 37
    qkv = torch.randn(T, (Hq + 2 * KH) * D)
    pos = torch.arange(T, dtype=torch.int32)
    cs = ops.rope_cos_sin(64, D, 10000.0)
    slots = torch.arange(T, dtype=torch.int32)
    cache = KVPool(KVPoolSpec(P, L, KH, D, dtype=torch.uint8)).cache
    ops.rope_kv_write(qkv, pos, cs, cache, slots, None, 1, Hq, KH, D)
    deq = q4.dequantize(cache)
    bt = torch.arange(P, dtype=torch.int32).view(1, P)
    cl = torch.tensor([T], dtype=torch.int32)
    q = qkv[-1:].clone()
    a = ops.paged_attention_decode(q, cache, 1, bt, cl, None, 1 / math.sqrt(D), Hq)
    b = ops.paged_attention_decode(q, deq, 1, bt, cl, None, 1 / math.sqrt(D), Hq)
    assert torch.allclose(a, b, atol=1e-5)
    # the stored k rows are the rotated k rows, quantised
    k_rot = qkv[:, Hq * D:(Hq + KH) * D].view(T, KH, D)
    k_back = deq[:, 1, 0].permute(0, 2, 1, 3).reshape(-1, KH, D)[:T]
    step = (k_rot.view(T, KH, 2, 32).amax(-1) - k_rot.view(T, KH, 2, 32).amin(-1)).amax() / 15
    assert (k_back - k_rot).abs().max() <= 0.51 * step + 1e-3


def _recompute_greedy_q4(cfg, weights, prompt, n_new):
    model = DecoderModel(cfg, weights, device="cpu", dtype=torch.float32)
    seq = list(prompt)
    for _ in range(n_new):
        T = len(seq)
        pages = (T + 15) // 16
        pool = KVPool(KVPoolSpec(pages, cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, dtype=torch.uint8))
        i32 = lambda v: torch.tensor(v, dtype=torch.int32)   # noqa: E731
        b = ForwardBatch(input_ids=i32(seq), positions=i32(list(range(T))), slot_mapping=i32(list(range(T))),
                         block_tables=i32([list(range(pages))]), context_lens=i32([T]), is_decode=False,
                         cu_q=i32([0, T]), max_q_len=T, logits_rows=torch.tensor([T - 1]))
        logits = model.forward(b, pool)
        seq.append(int(torch.argmax(logits[0].float())))
    return seq[len(prompt):]


def test_engine_q4_pool_matches_recompute():
    """Continuous batching over a four-bit pool gives the tokens of a full recompute over
    a four-bit pool (every token's K/V is quantised once, per row)."""
    cfg = PRESETS["tiny-qwen2"]
    w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=3, std=0.2)
    llm = LLM(cfg, device="cpu", dtype=torch.float32, kv_cache_dtype="q4", weights=w, max_batch=8,
              max_model_len=256, kv_pages=64)
    assert llm.pool.cache.dtype == torch.uint8
    g = torch.Generator().manual_seed(5)
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (5, 21)]
    reqs = llm.generate(prompts, SamplingParams(max_tokens=6))
    for p, r in zip(prompts, reqs):
        assert r.output_ids == _recompute_greedy_q4(cfg, w, p, 6)


# ------------------------------------------------------------------------- kernels (GPU)
def _q4_cache(lens, L, KH, D, seed=0):
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
    cache = q4.quantize(torch.randn(P, L, 2, KH, ps, D) * 1.5 + 0.3)
    return cache, bt


def _close(a, b, rtol=3e-2, atol=3e-2):
    a, b = a.float().cpu(), b.float().cpu()
    err = (a - b).abs()
    bad = (err > atol + rtol * b.abs()).sum().item()
    assert bad == 0, f"{bad} / {a.numel()} out of tolerance, max err {err.max().item():.4g}"


@pytest.mark.gpu
@pytest.mark.parametrize("D", [64, 128])
def test_q4_rope_kv_write_gpu(D, cuda_errors_clean):
    """The CUDA KV write stores the same four-bit rows as the host oracle (codes, scales
    and minima), from the same rotated bf16 k / v."""
    torch.manual_seed(D)
    T, Hq, KH, L, P = 9, 6, 2, 3, 8
    qkv = torch.randn(T, (Hq + 2 * KH) * D).bfloat16()
    pos = torch.randint(0, 500, (T,), dtype=torch.int32)
    cs = ops.rope_cos_sin(512, D, 10000.0)
    slots = torch.randperm(P * 16)[:T].to(torch.int32)
    slots[3] = -1
    cache_c = torch.zeros(P, L, 2, KH, 16, q4.row_bytes(D), dtype=torch.uint8)
    q_c = qkv.clone()
    ops.rope_kv_write(q_c, pos, cs, cache_c, slots, None, 1, Hq, KH, D)
    cache_g = torch.zeros_like(cache_c).to(DEV)
    q_g = qkv.to(DEV)
    ops.rope_kv_write(q_g, pos.to(DEV), cs.to(DEV), cache_g, slots.to(DEV), None, 1, Hq, KH, D)
    assert torch.equal(q_g.cpu(), q_c)
    assert torch.equal(cache_g.cpu(), cache_c)


@pytest.mark.gpu
@pytest.mark.parametrize("D,Hq,KH", [(128, 40, 8), (128, 28, 4), (64, 12, 12)])
@pytest.mark.parametrize("splits", [0, 1, 3, 16])
def test_q4_paged_decode_gpu(D, Hq, KH, splits, cuda_errors_clean):
    lens = [1, 17, 300, 64, 1033]
    L, layer = 2, 1
    cache, bt = _q4_cache(lens, L, KH, D, seed=D + Hq)
    B = len(lens)
    q = torch.randn(B, (Hq + 2 * KH) * D).bfloat16()
    cl = torch.tensor(lens, dtype=torch.int32)
    sm = 1.0 / math.sqrt(D)
    ref = ops.paged_attention_decode(q, cache, layer, bt, cl, None, sm, Hq)     # fp32 over dequantised rows
    out = ops.paged_attention_decode(q.to(DEV), cache.to(DEV), layer, bt.to(DEV), cl.to(DEV), None, sm, Hq,
                                     num_splits=splits)
    _close(out, ref)


@pytest.mark.gpu
@pytest.mark.parametrize("D,Hq,KH,rope", [(128, 40, 8, True), (64, 12, 12, False)])
@pytest.mark.parametrize("splits", [0, 1, 3])
def test_q4_paged_decode_fused_write_gpu(D, Hq, KH, rope, splits, cuda_errors_clean):
    """Decode attention with the fused RoPE + four-bit KV write gives the same bits
    (cache and output) as the standalone write followed by decode attention."""
    lens = [1, 17, 0, 300, 64, 1033]
    L, layer = 2, 1
    cache, bt = _q4_cache([max(n, 1) for n in lens], L, KH, D, seed=D + 7)
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
    c1, q1 = d(cache).clone(), d(qkv).clone()
    ops.rope_kv_write(q1, d(pos), cs, c1, d(slots), None, layer, Hq, KH, D)
    o1 = ops.paged_attention_decode(q1, c1, layer, d(bt), d(cl), None, sm, Hq, num_splits=splits)
    c2, q2 = d(cache).clone(), d(qkv).clone()
    o2 = ops.paged_attention_decode(q2, c2, layer, d(bt), d(cl), None, sm, Hq, num_splits=splits,
                                    positions=d(pos), cos_sin=cs, slot_mapping=d(slots))
    torch.cuda.synchronize()
    assert torch.equal(c1, c2)
    assert torch.equal(o1[[0, 1, 3, 4, 5]], o2[[0, 1, 3, 4, 5]])


@pytest.mark.gpu
@pytest.mark.parametrize("D,Hq,KH", [(128, 40, 8), (64, 12, 12)])
def test_q4_paged_prefill_gpu(D, Hq, KH, cuda_errors_clean):
    specs = [(5, 5), (64, 64), (70, 200), (130, 130), (1, 40)]
    L, layer = 2, 0
    cache, bt = _q4_cache([s[1] for s in specs], L, KH, D, seed=D)
    cu = [0]
    for ql, _ in specs:
        cu.append(cu[-1] + ql)
    q = torch.randn(cu[-1], Hq * D).bfloat16()
    cu_q = torch.tensor(cu, dtype=torch.int32)
    cl = torch.tensor([s[1] for s in specs], dtype=torch.int32)
    sm = 1.0 / math.sqrt(D)
    mq = max(s[0] for s in specs)
    ref = ops.paged_attention_prefill(q, cache, layer, bt, cu_q, cl, None, sm, Hq, mq)
    out = ops.paged_attention_prefill(q.to(DEV), cache.to(DEV), layer, bt.to(DEV), cu_q.to(DEV), cl.to(DEV),
                                      None, sm, Hq, mq)
    _close(out, ref)


@pytest.mark.gpu
def test_q4_engine_gpu(cuda_errors_clean):
    """A bf16 model over a four-bit pool on the GPU: generation runs through the CUDA
    graphs with the fused decode write, the pool is 5/16 of the bf16 pool's bytes, and
    the logits after a 70-token context stay close to those over a bf16 pool (random
    weights give near-flat logits, so greedy tokens are not compared)."""
    from vramancer_b200.engine.speculative import _full_logits
    cfg = PRESETS["tiny-qwen2-d128"]
    w = random_weights(cfg, device=DEV, dtype=torch.bfloat16, seed=3, std=0.02)
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 40, 70)]
    sizes, logits = [], []
    for kv in ("bf16", "q4"):
        llm = LLM(cfg, device=DEV, dtype=torch.bfloat16, kv_cache_dtype=kv, weights=w, max_batch=4,
                  max_model_len=256, kv_pages=64)
        reqs = llm.generate(prompts, SamplingParams(max_tokens=12))
        assert [len(r.output_ids) for r in reqs] == [12, 12, 12]
        sizes.append(llm.pool.nbytes())
        logits.append(_full_logits(llm, prompts[2])[0].float().cpu())
        del llm
    assert sizes[1] * 16 == sizes[0] * 5
    cos = torch.nn.functional.cosine_similarity(logits[0], logits[1], dim=0).item()
    assert cos >= 0.98, cos
