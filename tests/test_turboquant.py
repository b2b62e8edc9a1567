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
