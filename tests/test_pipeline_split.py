"""GPT-2 124M architecture, random-init fp32, layers split 6/6 across
two CPU devices by the model splitter; batch 1, a 32-token prompt drawn uniformly from
the vocabulary with a fixed seed, greedy decode of 64 tokens; the split run must match
the single-device run token for token."""
import torch

from vramancer_b200.engine.engine import LLMEngine, SamplingParams
from vramancer_b200.engine.runner import ModelRunner
from vramancer_b200.kv.paged import PagedKVCacheManager
from vramancer_b200.kv.pool import KVPool, KVPoolSpec
from vramancer_b200.models.config import PRESETS
from vramancer_b200.models.transformer import DecoderModel
from vramancer_b200.models.weights import random_weights
from vramancer_b200.parallel.pipeline import build_local_pipeline
from vramancer_b200.parallel.placement import (compute_optimal_placement, split_layers,
                                               split_model_into_blocks)


def _engine(model, pool, pages):
    runner = ModelRunner(model, pool, max_batch=1, max_model_len=256, use_cuda_graph=False)
    return LLMEngine(runner, PagedKVCacheManager(pages, enable_prefix_cache=False))


def test_gpt2_split_6_6_matches_single_device():
    cfg = PRESETS["gpt2"]
    g = torch.Generator().manual_seed(1234)
    prompt = torch.randint(0, cfg.vocab_size, (32,), generator=g).tolist()
    pages = 8
    w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=0)
    single = DecoderModel(cfg, w, device="cpu", dtype=torch.float32)
    pool = KVPool(KVPoolSpec(pages, cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, dtype=torch.float32))
    ref = _engine(single, pool, pages).generate([prompt], SamplingParams(max_tokens=64, ignore_eos=True))[0]

    blocks = split_model_into_blocks(cfg, ["cpu", "cpu"])          # the splitter picks 6/6
    assert [(b.start, b.end) for b in blocks] == [(0, 6), (6, 12)]
    pipe = build_local_pipeline(cfg, blocks, num_pages=pages, dtype=torch.float32, seed=0)
    out = _engine(pipe, None, pages).generate([prompt], SamplingParams(max_tokens=64, ignore_eos=True))[0]
    assert len(out.output_ids) == 64
    assert out.output_ids == ref.output_ids
    assert pipe.hops > 0


def test_split_helpers():
    assert split_layers(12, [1, 1]) == [6, 6]
    assert split_layers(48, [3, 1]) == [36, 12]
    assert sum(split_layers(28, [0.3, 0.5, 0.2])) == 28
    # bottleneck DP: twice-as-fast GPU gets about twice the layers
    r = compute_optimal_placement([1.0] * 12, [1.0] * 12, [2.0, 1.0], [100, 100])
    assert r == [(0, 8), (8, 12)]
    # memory constraint forces a split
    r = compute_optimal_placement([1.0] * 10, [1.0] * 10, [10.0, 1.0], [6, 100])
    assert r[0] == (0, 6)
