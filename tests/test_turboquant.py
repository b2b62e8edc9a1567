"""TurboQuant KV records: oracle properties on CPU; CUDA compress / decompress
against the oracle on a B200."""
import math

import pytest
import torch

from vramancer_b200.kv.turboquant import KVCacheCompressor, TurboQuantCache


def test_record_layout_and_round_trip_cpu():
    c = KVCacheCompressor(128)
    assert c.record_bytes == 64 and c.bits_per_dim == 4.0
    x = torch.randn(256, 128)
    rec = c.compress(x)
    assert rec.shape == (256, 64) and rec.dtype == torch.uint8
    assert torch.all(rec[:, 60:] == 0)
    xd = c.decompress(rec, torch.float32)
    rel = ((xd - x).norm(dim=-1) / x.norm(dim=-1)).mean()
    assert rel < 0.3                                  # 3-bit angles
    # the radius is the vector norm (rotation is orthonormal)
    _, rad, _, _ = c._fields(rec)
    assert torch.allclose(rad.float(), x.norm(dim=-1), rtol=2e-3)


def test_qjl_reduces_score_error_and_is_unbiased():
    c = KVCacheCompressor(128, seed=3)
    g = torch.Generator().manual_seed(0)
    k = torch.randn(2000, 128, generator=g)
    q = torch.randn(16, 128, generator=g)
    rec = c.compress(k)
    true = q @ k.t()
    e0 = (c.attention_score(q, rec, qjl=False) - true)
    e1 = (c.attention_score(q, rec, qjl=True) - true)
    assert e1.pow(2).mean() < e0.pow(2).mean()
    assert abs(e1.mean()) < 0.05 * true.std()


def test_sparse_v_attention_on_peaked_scores():
    c = KVCacheCompressor(128, seed=1)
    g = torch.Generator().manual_seed(1)
    k = torch.randn(512, 128, generator=g)
    v = torch.randn(512, 128, generator=g)
    q = 4 * k[:4] + 0.1 * torch.randn(4, 128, generator=g)       # each query matches one key
    out = c.sparse_v_attend(q, c.compress(k), c.compress(v), 1 / math.sqrt(128), keep=0.05)
    ref = torch.softmax(q @ k.t() / math.sqrt(128), -1) @ v
    assert ((out - ref).norm() / ref.norm()) < 0.35


def test_turboquant_cache_window():
    cache = TurboQuantCache(head_dim=128, window=8)
    k = torch.randn(1, 2, 5, 128)
    v = torch.randn(1, 2, 5, 128)
    K, V = cache.update(k, v, 0)
    assert K.shape == (1, 2, 5, 128) and torch.equal(K, k)
    K, V = cache.update(torch.randn(1, 2, 6, 128), torch.randn(1, 2, 6, 128), 0)
    assert K.shape == (1, 2, 11, 128) and cache.get_seq_length(0) == 11
    mem = cache.memory_bytes()
    assert mem["compressed"] == 2 * 1 * 2 * 3 * 64     # 3 tokens moved out of the window, K and V
    assert torch.allclose(K[..., :3, :], cache.comp.decompress(cache.packed[0][0], K.dtype))


@pytest.mark.gpu
def test_cuda_records_match_oracle():
    c = KVCacheCompressor(128, seed=5)
    g = torch.Generator().manual_seed(2)
    x = (torch.randn(4096, 128, generator=g) * 3).to(torch.bfloat16)
    ref = c.compress(x.float())
    got = c.to("cuda").compress(x.cuda()).cpu()
    ia, ra, sa, na = c.to("cpu")._fields(ref)
    ib, rb, sb, nb = c._fields(got)
    assert (ia == ib).float().mean() > 0.99
    assert torch.allclose(ra.float(), rb.float(), rtol=1e-3)
    assert (sa == sb).float().mean() > 0.97
    assert torch.all(got[:, 60:] == 0)
    # decompression of the same records: kernel vs oracle
    dk = c.to("cuda").decompress(ref.cuda(), torch.float32).cpu()
    do = c.to("cpu").decompress(ref, torch.float32)
    assert (dk - do).abs().max() <= 0.02 * do.abs().max()


@pytest.mark.gpu
def test_cuda_round_trip_fp32_input():
    c = KVCacheCompressor(128).to("cuda")
    x = torch.randn(10000, 128, device="cuda")
    xd = c.decompress(c.compress(x), torch.float32)
    rel = ((xd - x).norm(dim=-1) / x.norm(dim=-1)).mean()
    assert rel < 0.3


# ---------------------------------------------------------------- TurboQuant KV pages
def _tq_pool_case(B=3, KH=2, G=3, L=2, lens=(5, 40, 77), seed=0, device="cpu"):
    from vramancer_b200.kv.pool import KVPool, KVPoolSpec
    g = torch.Generator().manual_seed(seed)
    P = sum((n + 15) // 16 for n in lens) + 2
    pool = KVPool(KVPoolSpec(P, L, KH, 128, dtype=torch.int8), device=device)
    perm = torch.randperm(P, generator=g)
    bt = torch.zeros(B, max((n + 15) // 16 for n in lens), dtype=torch.int32)
    k = 0
    slots = []
    for b, n in enumerate(lens):
        np_ = (n + 15) // 16
        bt[b, :np_] = perm[k:k + np_].to(torch.int32)
        k += np_
        slots += [int(bt[b, t // 16]) * 16 + t % 16 for t in range(n)]
    Hq = KH * G
    qkv = (torch.randn(len(slots), (Hq + 2 * KH) * 128, generator=g) * 2).bfloat16()
    return pool, bt, torch.tensor(slots, dtype=torch.int32), qkv, Hq, KH


def test_tq_pages_cpu_write_and_decode():
    """Records written into a TurboQuant pool decode (CPU path) to the oracle's attention
    over the same records, and the pool is a quarter of a bf16 pool."""
    from vramancer_b200 import ops
    from vramancer_b200.kv.pool import KVPoolSpec
    pool, bt, slots, qkv, Hq, KH = _tq_pool_case()
    assert KVPoolSpec(4, 2, 2, 128, dtype=torch.int8).bytes_per_page * 4 == \
        KVPoolSpec(4, 2, 2, 128, dtype=torch.bfloat16).bytes_per_page
    ops.tq_kv_write(qkv, slots, pool.cache, 1, Hq, KH, pool.tq)
    lens = [5, 40, 77]
    cl = torch.tensor(lens, dtype=torch.int32)
    q = (torch.randn(3, Hq * 128) * 2).bfloat16()
    out = ops.tq_paged_decode(q, pool.cache, 1, bt, cl, pool.tq, 1 / math.sqrt(128), Hq)
    # oracle: the same math on records gathered per sequence
    off = 0
    G = Hq // KH
    for b, n in enumerate(lens):
        v = qkv[off:off + n].view(n, Hq + 2 * KH, 128)
        off += n
        for h in range(KH):
            krec = pool.tq.compress(v[:, Hq + h].float())
            vrec = pool.tq.compress(v[:, Hq + KH + h].float())
            s = pool.tq.attention_score(q[b, h * G * 128:(h + 1) * G * 128].float().view(G, 128), krec)
            w = torch.softmax(s / math.sqrt(128), -1)
            ref = w @ pool.tq.decompress(vrec, torch.float32)
            assert torch.allclose(out[b, h * G * 128:(h + 1) * G * 128].float().view(G, 128), ref, atol=2e-2,
                                  rtol=2e-2)


def test_tq_engine_cpu():
    """An engine over a TurboQuant pool generates, and its logits stay near those of an
    fp32 pool (records are ~4 bits per value)."""
    from vramancer_b200.engine.engine import SamplingParams
    from vramancer_b200.engine.speculative import _full_logits
    from vramancer_b200.llm import LLM
    from vramancer_b200.models.config import PRESETS
    from vramancer_b200.models.weights import random_weights
    cfg = PRESETS["tiny-qwen2-d128"]
    w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=3, std=0.02)
    g = torch.Generator().manual_seed(9)
    seq = torch.randint(0, cfg.vocab_size, (50,), generator=g).tolist()
    logits = []
    for kv in ("fp32", "tq"):
        llm = LLM(cfg, device="cpu", dtype=torch.float32, kv_cache_dtype=kv, weights=w, max_batch=4,
                  max_model_len=256, kv_pages=64)
        r = llm.generate([seq[:20]], SamplingParams(max_tokens=6))[0]
        assert len(r.output_ids) == 6
        logits.append(_full_logits(llm, seq)[0])
    cos = torch.nn.functional.cosine_similarity(logits[0], logits[1], dim=0).item()
    assert cos > 0.9, cos


@pytest.mark.gpu
def test_tq_pages_gpu_match_cpu(cuda_errors_clean):
    """The CUDA record writer and the decode attention over TurboQuant pages against the
    CPU path (the oracle): records agree as the compressor test allows, outputs within
    the estimator's tolerance."""
    from vramancer_b200 import ops
    pool_c, bt, slots, qkv, Hq, KH = _tq_pool_case(B=3, KH=4, G=5, lens=(5, 140, 300), seed=4)
    pool_g, *_ = _tq_pool_case(B=3, KH=4, G=5, lens=(5, 140, 300), seed=4, device="cuda")
    ops.tq_kv_write(qkv, slots, pool_c.cache, 1, Hq, KH, pool_c.tq)
    ops.tq_kv_write(qkv.cuda(), slots.cuda(), pool_g.cache, 1, Hq, KH, pool_g.tq)
    torch.cuda.synchronize()
    rg = pool_g.cache.cpu().view(torch.uint8)
    rc = pool_c.cache.view(torch.uint8)
    ia, ra, _, _ = pool_c.tq._fields(rc.reshape(-1, 64).clone())
    ib, rb, _, _ = pool_c.tq._fields(rg.reshape(-1, 64).clone())
    assert (ia == ib).float().mean() > 0.99
    assert torch.allclose(ra.float(), rb.float(), rtol=1e-3, atol=1e-3)
    cl = torch.tensor([5, 140, 300], dtype=torch.int32)
    q = (torch.randn(3, Hq * 128) * 2).bfloat16()
    ref = ops.tq_paged_decode(q, pool_c.cache, 1, bt, cl, pool_c.tq, 1 / math.sqrt(128), Hq)
    # the kernel on the oracle's records (same inputs, so only the kernel's arithmetic differs)
    pool_g.cache.copy_(pool_c.cache.cuda())
    out = ops.tq_paged_decode(q.cuda(), pool_g.cache, 1, bt.cuda(), cl.cuda(), pool_g.tq, 1 / math.sqrt(128), Hq)
    torch.cuda.synchronize()
    err = (out.float().cpu() - ref.float()).abs().max().item()
    assert err <= 3e-2 * ref.float().abs().max().item() + 2e-2, err


@pytest.mark.gpu
def test_tq_engine_gpu(cuda_errors_clean):
    """A bf16 model over a TurboQuant pool on the GPU: graph-replayed decode through the
    record writer and the record attention; logits close to a bf16 pool's."""
    from vramancer_b200.engine.engine import SamplingParams
    from vramancer_b200.engine.speculative import _full_logits
    from vramancer_b200.llm import LLM
    from vramancer_b200.models.config import PRESETS
    from vramancer_b200.models.weights import random_weights
    cfg = PRESETS["tiny-qwen2-d128"]
    w = random_weights(cfg, device="cuda", dtype=torch.bfloat16, seed=3, std=0.02)
    g = torch.Generator().manual_seed(9)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 40, 70)]
    logits = []
    for kv in ("bf16", "tq"):
        llm = LLM(cfg, device="cuda", dtype=torch.bfloat16, kv_cache_dtype=kv, weights=w, max_batch=4,
                  max_model_len=256, kv_pages=64)
        reqs = llm.generate(prompts, SamplingParams(max_tokens=12))
        assert [len(r.output_ids) for r in reqs] == [12, 12, 12]
        logits.append(_full_logits(llm, prompts[2])[0].float().cpu())
        del llm
    cos = torch.nn.functional.cosine_similarity(logits[0], logits[1], dim=0).item()
    assert cos > 0.9, cos
