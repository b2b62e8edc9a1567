"""Speculative decoding must reproduce plain greedy decoding exactly (CPU reference ops)."""
import torch

from vramancer_b200.engine.engine import SamplingParams
from vramancer_b200.engine.speculative import PromptLookupDecoder, accept_greedy, find_draft
from vramancer_b200.llm import LLM
from vramancer_b200.models.config import PRESETS
from vramancer_b200.models.weights import random_weights


def test_find_draft_and_accept():
    seq = [5, 6, 7, 8, 9, 1, 2, 5, 6, 7]
    assert find_draft(seq, 3, 4) == [8, 9, 1, 2]
    assert find_draft([1, 2, 3], 3, 4) == []
    assert accept_greedy([8, 9, 4], [8, 9, 1, 3]) == ([8, 9, 1], 2)
    assert accept_greedy([8], [0, 5]) == ([0], 0)


def _llm(**kw):
    cfg = PRESETS["tiny-qwen2"]
    w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=5, std=0.2)
    return LLM(cfg, device="cpu", dtype=torch.float32, kv_cache_dtype="fp32", weights=w, max_batch=4,
               max_model_len=512, kv_pages=128, **kw), cfg


def test_prompt_lookup_engine_matches_plain_greedy():
    g = torch.Generator().manual_seed(3)
    span = torch.randint(0, 512, (16,), generator=g).tolist()
    prompts = [span * 4, torch.randint(0, 512, (20,), generator=g).tolist()]
    plain, _ = _llm()
    ref = [r.output_ids for r in plain.generate(prompts, SamplingParams(max_tokens=24))]
    spec, _ = _llm(spec_num_draft=8, spec_ngram=3)
    out = [r.output_ids for r in spec.generate(prompts, SamplingParams(max_tokens=24))]
    assert out == ref


def test_prompt_lookup_decoder_standalone():
    g = torch.Generator().manual_seed(4)
    p = torch.randint(0, 512, (12,), generator=g).tolist() * 3
    plain, _ = _llm()
    ref = plain.generate([p], SamplingParams(max_tokens=16))[0].output_ids
    llm, _ = _llm()
    dec = PromptLookupDecoder(llm, num_draft=8, ngram=3)
    assert dec.generate(p, 16) == ref


def test_draft_model_accepts_self_drafts_and_matches_greedy():
    from vramancer_b200.engine.speculative import DraftModelDecoder
    g = torch.Generator().manual_seed(9)
    p = torch.randint(0, 512, (10,), generator=g).tolist()
    plain, _ = _llm()
    ref = plain.generate([p], SamplingParams(max_tokens=20))[0].output_ids
    target, _ = _llm()
    drafter, _ = _llm()                      # identical weights: every draft is right
    dec = DraftModelDecoder(target, drafter, gamma=4, adaptive=True)
    assert dec.generate(p, 20) == ref
    assert dec.stats.acceptance == 1.0 and dec.stats.proposed > 0


def test_wrong_drafts_are_rejected_without_changing_output():
    from vramancer_b200.engine.speculative import speculative_decode_step
    g = torch.Generator().manual_seed(11)
    p = torch.randint(0, 512, (9,), generator=g).tolist()
    plain, _ = _llm()
    ref = plain.generate([p], SamplingParams(max_tokens=6))[0].output_ids
    llm, _ = _llm()
    eng = llm.engine
    req = eng.add_request(p, SamplingParams(max_tokens=6))
    eng.step()                                # prefill + first token (+ one decode)
    while not req.finished:
        bad = [(t + 1) % 512 for t in ref[len(req.output_ids):len(req.output_ids) + 3]]
        toks = speculative_decode_step(eng, [req], 0, 0, eng.spec_stats, drafts=[bad])[0]
        for t in toks:
            eng._emit(req, t)
            if req.finished:
                break
    assert req.output_ids == ref
