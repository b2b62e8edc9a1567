"""Vocabulary-parallel sampling: per-rank candidates + one small all-gather give the ids
of the full-vocabulary sampler.  The GPU test emulates the ranks in one process (each
rank's shard through `sample_vp_local`, the stacked candidates through
`sample_vp_combine`) and compares with `sample` over the whole row."""
import pytest
import torch

from vramancer_b200 import ops


def test_vp_sampling_ok_modes():
    V = 1000
    assert ops.vp_sampling_ok([0.0, 0.0], [0, 0], [1.0, 0.5], V)          # greedy ignores top-p
    assert ops.vp_sampling_ok([0.7], [0], [1.0], V)                      # plain temperature
    assert ops.vp_sampling_ok([0.7], [50], [0.9], V)                     # top-k (+ top-p)
    assert ops.vp_sampling_ok([0.7], [ops.VP_KMAX], [1.0], V)
    assert not ops.vp_sampling_ok([0.7], [ops.VP_KMAX + 1], [1.0], V)
    assert not ops.vp_sampling_ok([0.7], [0], [0.9], V)                  # nucleus over everything
    assert ops.vp_sampling_ok([0.7], [V], [1.0], V)                      # top-k = vocab is no top-k


def _row_params(B):
    temps, ks, ps = [], [], []
    modes = [(0.0, 0, 1.0), (0.8, 0, 1.0), (0.7, 50, 0.9), (1.0, 128, 1.0), (1.2, 1, 1.0), (0.9, 20, 1.0),
             (0.6, 100, 0.5), (1.5, 0, 1.0)]
    for r in range(B):
        t, k, p = modes[r % len(modes)]
        temps.append(t)
        ks.append(k)
        ps.append(p)
    return temps, ks, ps


@pytest.mark.gpu
@pytest.mark.parametrize("tp", [2, 8])
@pytest.mark.parametrize("V", [152064, 4096])
def test_vocab_parallel_matches_full_row(tp, V, cuda_errors_clean):
    torch.manual_seed(tp + V)
    B = 24
    dev = "cuda"
    x = torch.randn(B, V, device=dev) * 3
    x[3] = torch.round(x[3] * 2) / 2          # a row with many tied logits
    logits = x.bfloat16()
    temps, ks, ps = _row_params(B)
    assert ops.vp_sampling_ok(temps, ks, ps, V)
    t = torch.tensor(temps, device=dev)
    k = torch.tensor(ks, dtype=torch.int32, device=dev)
    p = torch.tensor(ps, device=dev)
    steps = torch.randint(0, 1000, (B,), dtype=torch.int32, device=dev)
    seed = 1234
    full = ops.sample(logits, t, k, p, seed, steps)

    n = (V + tp - 1) // tp                    # lm_head rows per rank, the last shard padded
    padded = torch.cat([logits, torch.zeros(B, n * tp - V, dtype=logits.dtype, device=dev)], 1)
    nat = ops.native()
    cands = []
    for r in range(tp):
        c = torch.empty(2, B, ops.VP_KC, dtype=torch.int32, device=dev)
        nat.sample_vp_local(padded[:, r * n:(r + 1) * n].contiguous(), r * n, V, t, k, p, seed, steps,
                            ops.VP_KMAX, c)
        cands.append(c)
    gathered = torch.stack(cands)
    out = torch.empty(B, dtype=torch.int32, device=dev)
    nat.sample_vp_combine(gathered, V, t, k, p, seed, steps, ops.VP_KMAX, out)
    torch.cuda.synchronize()
    assert torch.equal(out, full), (out.tolist(), full.tolist())
    # the one-call wrapper with an emulated gather gives the same ids for rank 0's view
    out2 = ops.sample_vocab_parallel(padded[:, :n].contiguous(), 0, V, t, k, p, seed, steps,
                                     lambda c: torch.stack([c] + cands[1:]))
    assert torch.equal(out2, full)
