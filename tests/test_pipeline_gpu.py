"""Conductor on the GPU: single device, and a 2-GPU in-process pipeline that must match it."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_pipeline_single_and_pp_match():
    from vramancer_b200.pipeline import InferencePipeline
    p1 = InferencePipeline(enable_metrics=False).load("tiny-qwen2-d128", num_gpus=1, max_model_len=256, max_batch=4)
    prompt = list(range(3, 40))
    a = p1.generate(prompt, max_new_tokens=12, return_ids=True)
    assert len(a) == 12
    out = p1.generate_batch(["abc", "defg"], max_new_tokens=4)
    assert len(out) == 2
    w = p1.llm.weights
    p1.shutdown()
    if torch.cuda.device_count() < 2:
        return
    p2 = InferencePipeline(enable_metrics=False).load("tiny-qwen2-d128", num_gpus=2, max_model_len=256,
                                                       max_batch=4)
    assert p2.mode == "pp2"
    b = p2.generate(prompt, max_new_tokens=12, return_ids=True)
    p2.shutdown()
    # same random-init weights on both paths (per-tensor seeds): bf16 tokens agree
    assert b[:4] == a[:4]
