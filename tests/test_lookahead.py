"""Overlapped decode (step n+1 launched on step n's device-resident tokens before the
host reads them) must emit exactly what the synchronous engine emits: greedy and
sampled requests, staggered arrivals, stop tokens, length limits, aborts, page
boundaries.  Runs the host logic on CPU; the GPU tests run the same engine on CUDA."""
import pytest
import torch

from vramancer_b200.engine.engine import SamplingParams
from vramancer_b200.llm import LLM
from vramancer_b200.models.config import PRESETS
from vramancer_b200.models.weights import random_weights


def _llm(lookahead: bool, eos=None):
    cfg = PRESETS["tiny-qwen2"]
    w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=5, std=0.2)
    llm = LLM(cfg, device="cpu", dtype=torch.float32, kv_cache_dtype="fp32", weights=w, max_batch=8,
              max_model_len=128, kv_pages=96, eos_token_id=eos)
    llm.engine.lookahead = lookahead
    return llm


def _run(llm, script):
    """script: list of (step index, prompt, params) arrivals; aborts: (step, k-th request)."""
    eng = llm.engine
    reqs = []
    arrivals, aborts = script
    step = 0
    while step < 400 and (eng.has_unfinished() or any(s >= step for s, _, _ in arrivals)):
        for s, p, sp in arrivals:
            if s == step:
                reqs.append(eng.add_request(p, sp))
        for s, k in aborts:
            if s == step and k < len(reqs):
                eng.abort(reqs[k].request_id)
        eng.step()
        step += 1
    eng.flush()
    return [(list(r.output_ids), r.finish_reason) for r in reqs]


def _script(vocab, seed):
    g = torch.Generator().manual_seed(seed)
    rnd = lambda n: torch.randint(0, vocab, (n,), generator=g).tolist()   # noqa: E731
    arrivals = [
        (0, rnd(5), SamplingParams(max_tokens=20)),
        (0, rnd(16), SamplingParams(max_tokens=7)),
        (2, rnd(31), SamplingParams(max_tokens=25, temperature=0.9, top_k=20)),
        (5, rnd(3), SamplingParams(max_tokens=1)),
        (6, rnd(9), SamplingParams(max_tokens=30, temperature=0.7, top_p=0.8)),
        (9, rnd(40), SamplingParams(max_tokens=12)),
    ]
    aborts = [(14, 2)]
    return arrivals, aborts


def _same(a, b):
    """Equal outputs, except that an aborted request may have one token fewer with
    lookahead (its last step was still in flight when the abort came)."""
    assert len(a) == len(b)
    for (ta, ra), (tb, rb) in zip(a, b):
        assert ra == rb
        if ra == "abort":
            n = min(len(ta), len(tb))
            assert ta[:n] == tb[:n] and abs(len(ta) - len(tb)) <= 1
        else:
            assert ta == tb


def test_lookahead_matches_synchronous_engine():
    a = _run(_llm(False), _script(512, 0))
    b = _run(_llm(True), _script(512, 0))
    _same(a, b)
    assert any(r == "abort" for _, r in a) and any(r == "length" for _, r in a)


def test_lookahead_with_stop_tokens():
    # an EOS that greedy decoding actually emits: take a token from a plain run
    base = _run(_llm(False), _script(512, 1))
    eos = base[0][0][3]
    a = _run(_llm(False, eos=eos), _script(512, 1))
    b = _run(_llm(True, eos=eos), _script(512, 1))
    _same(a, b)
    assert any(r == "stop" for _, r in a)


def test_lookahead_chains_steps():
    llm = _llm(True)
    calls = {"chained": 0, "plain": 0}
    orig = llm.runner.launch_decode

    def spy(*args, ids_on_device=False, **kw):
        calls["chained" if ids_on_device else "plain"] += 1
        return orig(*args, ids_on_device=ids_on_device, **kw)

    llm.runner.launch_decode = spy
    reqs = llm.generate([[1, 2, 3], [4, 5, 6, 7]], SamplingParams(max_tokens=16))
    assert all(len(r.output_ids) == 16 for r in reqs)
    assert calls["chained"] >= 10


@pytest.mark.gpu
def test_lookahead_matches_synchronous_engine_on_gpu(cuda_errors_clean):
    """Graph-replayed decode on the GPU: overlapped and synchronous engines agree token
    for token (the chained step's ids come from the device copy of the sampled ids)."""
    cfg = PRESETS["tiny-qwen2-d128"]
    w = random_weights(cfg, device="cuda", dtype=torch.bfloat16, seed=5)
    outs = []
    for la in (False, True):
        llm = LLM(cfg, device="cuda", weights=w, max_batch=8, max_model_len=160, kv_pages=96)
        llm.engine.lookahead = la
        outs.append(_run(llm, _script(cfg.vocab_size, 2)))
    _same(outs[0], outs[1])
