"""Many client threads against one serving pipeline (CPU, tiny model): concurrent
submits, sampled and greedy requests, streaming, aborts and a small KV pool (so
preemption happens) -- every request completes, greedy results equal the ones of the
same prompts run one at a time, and the engine ends idle with every KV page free."""
import random
import threading

import torch

from vramancer_b200.pipeline import InferencePipeline


def test_many_threads_one_pipeline():
    pipe = InferencePipeline(enable_metrics=True).load("tiny-qwen2", device="cpu", max_model_len=160, max_batch=8,
                                                       kv_pages=20)
    eng = pipe.engine
    eng.eos_token_id = None
    rng = random.Random(0)
    prompts = [[rng.randrange(1, 500) for _ in range(rng.randint(4, 60))] for _ in range(40)]
    # one at a time first (the reference result of every greedy prompt)
    want = {i: pipe.generate(p, max_new_tokens=12, return_ids=True) for i, p in enumerate(prompts[:20])}

    errors, results = [], {}

    def client(k):
        try:
            r = random.Random(k)
            for j in range(2):
                i = (k * 2 + j) % len(prompts)
                if i < 20:
                    results[i] = pipe.generate(prompts[i], max_new_tokens=12, return_ids=True)
                elif r.random() < 0.5:
                    out = pipe.generate(prompts[i], max_new_tokens=10, temperature=0.8, top_k=30, return_ids=True)
                    assert len(out) == 10
                else:
                    toks = list(pipe.generate_stream(prompts[i], max_new_tokens=8))
                    assert len(toks) >= 1
        except Exception as e:   # surfaced below
            errors.append(repr(e))

    threads = [threading.Thread(target=client, args=(k,)) for k in range(20)]
    for t in threads:
        t.start()
    for t in threads:
        t.join(timeout=300)
    assert not any(t.is_alive() for t in threads)
    assert not errors, errors[:3]
    for i, out in results.items():
        assert out == want[i], i
    assert not eng.has_unfinished()
    assert eng.stats["preempted"] > 0          # the small pool forced recompute preemption
    eng.flush()
    assert eng.kv.num_free_pages() == eng.kv.num_pages
    pipe.shutdown()
