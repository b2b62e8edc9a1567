"""Engine correctness on CPU: paged-KV continuous batching must produce exactly the
tokens of a no-cache full-recompute greedy decode (the CPU reference ops)."""
import torch

from vramancer_b200 import ops
from vramancer_b200.engine.engine import SamplingParams
from vramancer_b200.kv.pool import KVPool, KVPoolSpec
from vramancer_b200.llm import LLM
from vramancer_b200.models.config import PRESETS
from vramancer_b200.models.transformer import DecoderModel, ForwardBatch
from vramancer_b200.models.weights import random_weights


def recompute_greedy(cfg, weights, prompt, n_new, dtype=torch.float32):
    """Greedy decode that re-runs the whole sequence each step (no KV reuse)."""
    model = DecoderModel(cfg, weights, device="cpu", dtype=dtype)
    seq = list(prompt)
    for _ in range(n_new):
        T = len(seq)
        pages = (T + 15) // 16
        pool = KVPool(KVPoolSpec(pages, cfg.num_layers, cfg.num_kv_heads, cfg.head_dim, dtype=dtype))
        i32 = lambda v: torch.tensor(v, dtype=torch.int32)
        b = ForwardBatch(input_ids=i32(seq), positions=i32(list(range(T))), slot_mapping=i32(list(range(T))),
                         block_tables=i32([list(range(pages))]), context_lens=i32([T]), is_decode=False,
                         cu_q=i32([0, T]), max_q_len=T, logits_rows=torch.tensor([T - 1]))
        logits = model.forward(b, pool)
        seq.append(int(torch.argmax(logits[0].float())))
    return seq[len(prompt):]


def _check(preset, prompts, n_new=8, kv="fp32", **kw):
    cfg = PRESETS[preset]
    w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=3, std=0.2)
    llm = LLM(cfg, device="cpu", dtype=torch.float32, kv_cache_dtype=kv, weights=w, max_batch=8,
              max_model_len=256, kv_pages=128, **kw)
    reqs = llm.generate(prompts, SamplingParams(max_tokens=n_new))
    for p, r in zip(prompts, reqs):
        assert r.output_ids == recompute_greedy(cfg, w, p, n_new), (preset, p)
    return llm


def test_engine_matches_recompute_qwen2():
    g = torch.Generator().manual_seed(0)
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (5, 17, 33)]
    _check("tiny-qwen2", prompts)


def test_engine_matches_recompute_gpt2():
    g = torch.Generator().manual_seed(1)
    prompts = [torch.randint(0, 500, (n,), generator=g).tolist() for n in (3, 20)]
    _check("tiny-gpt2", prompts)


def test_engine_chunked_prefill_and_prefix_cache():
    g = torch.Generator().manual_seed(2)
    base = torch.randint(0, 512, (40,), generator=g).tolist()
    llm = _check("tiny-qwen2", [base + [7, 8, 9]], max_prefill_tokens=16)
    # a later request with the same 40-token prefix reuses its 2 full pages
    p2 = base + [1, 2]
    r = llm.generate([p2], SamplingParams(max_tokens=8))[0]
    assert llm.kv.stats()["prefix_hits"] >= 1 and r.cached_tokens == 32
    cfg = PRESETS["tiny-qwen2"]
    w = llm.weights
    assert r.output_ids == recompute_greedy(cfg, w, p2, 8)


def test_engine_moe():
    g = torch.Generator().manual_seed(4)
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (6, 19)]
    _check("tiny-moe", prompts, n_new=5)
