"""Request-level resume after a failed engine step (fault injected on the host: the
runner raises): running requests re-prefill their prompt + generated tokens and finish
with exactly the tokens of an undisturbed run; a request that keeps failing ends with
an error after its retries."""
import pytest
import torch

from vramancer_b200.pipeline import InferencePipeline


def _pipe():
    return InferencePipeline(enable_metrics=False).load("tiny-qwen2", device="cpu", max_model_len=128, max_batch=4,
                                                        kv_pages=64)


def test_resume_after_transient_failures():
    prompts = [[5, 6, 7, 8, 9], list(range(100, 130)), [42] * 9]
    ref = _pipe()
    want = [ref.generate(p, max_new_tokens=16, return_ids=True) for p in prompts]
    ref.shutdown()

    pipe = _pipe()
    runner = pipe.engine.runner
    orig = runner.launch_decode
    calls = {"n": 0}

    def flaky(*a, **k):
        calls["n"] += 1
        if calls["n"] in (4, 9):          # two injected failures mid-decode
            raise RuntimeError("injected device error")
        return orig(*a, **k)

    runner.launch_decode = flaky
    futs = [pipe.submit(p, 16) for p in prompts]
    got = [f.result(timeout=120).output_ids for f in futs]
    assert got == want
    assert calls["n"] > 9
    pipe.shutdown()


def test_persistent_failure_ends_with_error():
    pipe = _pipe()

    def broken(*a, **k):
        raise RuntimeError("device gone")

    pipe.engine.runner.launch_decode = broken
    fut = pipe.submit([1, 2, 3], 8)
    with pytest.raises(RuntimeError):
        fut.result(timeout=120)
    assert not pipe.engine.has_unfinished()
    assert pipe.engine.kv.num_free_pages() == pipe.engine.kv.num_pages
    pipe.shutdown()
