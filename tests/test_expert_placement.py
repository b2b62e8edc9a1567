"""Expert usage histogram, hot/cold split and load-balancing permutation (CPU)."""
import pytest
import torch

from vramancer_b200.models.config import get_config
from vramancer_b200.models.weights import random_weights
from vramancer_b200.parallel import moe
from vramancer_b200.parallel.expert_placement import (ExpertUsage, apply_expert_permutation, balanced_permutation,
                                                      hot_cold, rank_loads)


def test_permutation_preserves_the_layer():
    cfg = get_config("tiny-moe")
    w = random_weights(cfg, seed=2, layers=[0], embed=False, head=False, dtype=torch.float32)
    x = torch.randn(9, cfg.hidden_size)
    args = lambda ww: (cfg, x, ww["layers.0.router_w"], ww["layers.0.experts_gate_up_w"],  # noqa: E731
                       ww["layers.0.experts_down_w"])
    want = moe.moe_forward(*args(w))
    perm = [3, 0, 7, 1, 6, 2, 5, 4]
    w2 = apply_expert_permutation(dict(w), cfg, perm, layers=[0])
    got = moe.moe_forward(*args(w2))
    torch.testing.assert_close(got, want, rtol=1e-5, atol=1e-6)
    with pytest.raises(ValueError):
        apply_expert_permutation(dict(w), cfg, [0, 0, 1, 2, 3, 4, 5, 6], layers=[0])


def test_usage_hook_and_balance():
    cfg = get_config("tiny-moe")
    usage = ExpertUsage(cfg)
    w = random_weights(cfg, seed=2, layers=[0, 1], embed=False, head=False, dtype=torch.float32)
    moe.set_usage_hook(usage)
    try:
        for layer in (0, 1):
            moe.moe_forward(cfg, torch.randn(20, cfg.hidden_size), w[f"layers.{layer}.router_w"],
                            w[f"layers.{layer}.experts_gate_up_w"], w[f"layers.{layer}.experts_down_w"])
    finally:
        moe.set_usage_hook(None)
    c = usage.counts()
    assert c.shape == (2, 8) and int(c[0].sum()) == 20 * 2 and int(c[1].sum()) == 40
    # a skewed histogram: contiguous ranges are badly unbalanced, the permutation fixes it
    skew = torch.tensor([100, 90, 80, 70, 5, 4, 3, 2])
    before = rank_loads(skew, 2)
    perm = balanced_permutation(skew, 2)
    after = rank_loads(skew, 2, perm)
    assert sorted(perm) == list(range(8))
    assert max(before) / min(before) > 10 and max(after) / min(after) < 1.1
    hot, cold = hot_cold(skew, 0.8)
    assert hot == [0, 1, 2, 3] and sorted(hot + cold) == list(range(8))
