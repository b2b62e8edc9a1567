"""Recompute preemption: with a KV pool too small for every running sequence, the
engine gives the most recently admitted sequences' pages back, re-prefills them later
(prompt + generated tokens) and finishes every request with exactly the tokens of an
engine whose pool is large enough (greedy, fp32 CPU reference ops)."""
import torch

from vramancer_b200.engine.engine import SamplingParams
from vramancer_b200.llm import LLM
from vramancer_b200.models.config import PRESETS
from vramancer_b200.models.weights import random_weights


def _run(kv_pages, lookahead=True, prefix=True):
    cfg = PRESETS["tiny-qwen2"]
    w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=7, std=0.2)
    llm = LLM(cfg, device="cpu", dtype=torch.float32, kv_cache_dtype="fp32", weights=w, max_batch=6,
              max_model_len=160, kv_pages=kv_pages, enable_prefix_cache=prefix)
    llm.engine.lookahead = lookahead
    g = torch.Generator().manual_seed(3)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (9, 30, 17, 44, 5)]
    reqs = llm.generate(prompts, SamplingParams(max_tokens=40))
    return [r.output_ids for r in reqs], [r.finish_reason for r in reqs], llm.engine.stats["preempted"]


def test_preemption_matches_unconstrained_pool():
    want, reasons, pre = _run(96)
    assert pre == 0 and all(len(t) == 40 for t in want)
    for lookahead in (True, False):
        for prefix in (True, False):
            got, reasons, pre = _run(14, lookahead, prefix)
            assert pre > 0, (lookahead, prefix)
            assert got == want, (lookahead, prefix)
            assert all(r == "length" for r in reasons)


def test_sequence_larger_than_pool_ends_instead_of_failing():
    cfg = PRESETS["tiny-qwen2"]
    w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=7, std=0.2)
    llm = LLM(cfg, device="cpu", dtype=torch.float32, kv_cache_dtype="fp32", weights=w, max_batch=2,
              max_model_len=160, kv_pages=3)
    r = llm.generate([[1, 2, 3, 4, 5]], SamplingParams(max_tokens=100))[0]
    assert r.finished and r.finish_reason == "length" and 0 < len(r.output_ids) < 100


def test_speculation_with_a_small_pool():
    """Prompt-lookup speculation on a pool too small for every verify step: drafts are
    skipped when their pages are missing, preemption makes room, and the greedy tokens
    equal those of an unconstrained engine."""
    cfg = PRESETS["tiny-qwen2"]
    outs = []
    for pages in (96, 9):
        w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=0)   # repetitive output: drafts hit
        llm = LLM(cfg, device="cpu", dtype=torch.float32, kv_cache_dtype="fp32", weights=w, max_batch=4,
                  max_model_len=200, kv_pages=pages, spec_num_draft=6, spec_ngram=2)
        g = torch.Generator().manual_seed(5)
        prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (30, 20, 12)]
        reqs = llm.generate(prompts, SamplingParams(max_tokens=40))
        outs.append([r.output_ids for r in reqs])
        assert llm.engine.spec_stats.proposed > 0
        if pages == 9:
            assert llm.engine.stats["preempted"] > 0
    assert outs[0] == outs[1]
