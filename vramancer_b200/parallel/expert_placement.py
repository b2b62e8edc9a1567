"""Expert usage statistics and placement for MoE models.

    usage = ExpertUsage(cfg)                  # per-layer routed-pair histogram (device)
    moe.set_usage_hook(usage)                 # every MoE layer call adds its routing
    ... run traffic ...
    perm = balanced_permutation(usage.counts(), world)   # experts -> EP ranks, by load
    apply_expert_permutation(weights, cfg, perm)         # same model, balanced ranks
    hot, cold = hot_cold(usage.counts()[layer], 0.8)     # experts carrying 80% of pairs

Expert parallelism gives rank r the contiguous experts [r E/W, (r+1) E/W).  When the
router favours some experts, the rank holding them does more of every layer's work and
the others wait at the combine.  Permuting the router's rows together with the expert
weights renames the experts without changing the layer's function (the softmax over
the router logits is permutation-equivariant), so a permutation that spreads the
measured load evenly over the contiguous ranges balances the ranks at no runtime cost.
`hot_cold` splits the experts of a layer by traffic for memory placement (hot experts
stay resident; cold ones are candidates for host memory).

Reference parity: core/expert_pinning.py:115-642 (hot/cold expert registry built from
an activation histogram; cold experts mirrored to a lender GPU and staged per call).
"""
from __future__ import annotations

from typing import Dict, List, Sequence, Tuple

import torch

from ..models.config import ModelConfig


class ExpertUsage:
    """Routed (token, k) pairs per expert and layer, accumulated on the device without
    host synchronisation (an index_add per MoE call)."""

    def __init__(self, cfg: ModelConfig, device=None):
        if not cfg.is_moe:
            raise ValueError("expert usage needs a MoE model")
        self.cfg = cfg
        self.device = torch.device(device) if device is not None else torch.device("cpu")
        self._counts = torch.zeros(cfg.num_layers, cfg.num_experts, dtype=torch.int64, device=self.device)
        self._layer = 0

    def observe(self, ids: torch.Tensor, layer: int = None) -> None:
        """ids: expert ids [T, k] of one MoE call (layer: which layer; default: the next one
        in call order, wrapping after the last)."""
        if layer is None:
            layer = self._layer
            self._layer = (self._layer + 1) % self.cfg.num_layers
        flat = ids.reshape(-1).to(self._counts.device, torch.int64)
        self._counts[layer].index_add_(0, flat, torch.ones_like(flat))

    def counts(self) -> torch.Tensor:
        return self._counts.cpu()

    def reset(self) -> None:
        self._counts.zero_()
        self._layer = 0


def hot_cold(counts: torch.Tensor, coverage: float = 0.8) -> Tuple[List[int], List[int]]:
    """(hot, cold) experts of one layer: the fewest experts carrying `coverage` of the
    routed pairs, most used first; the rest."""
    c = counts.reshape(-1).to(torch.float64)
    order = torch.argsort(c, descending=True).tolist()
    total = float(c.sum())
    hot, acc = [], 0.0
    for e in order:
        if total > 0 and acc >= coverage * total:
            break
        hot.append(e)
        acc += float(c[e])
    cold = [e for e in order if e not in set(hot)]
    return hot, cold


def balanced_permutation(counts: torch.Tensor, world: int) -> List[int]:
    """A permutation of the experts (new position -> old expert id) whose contiguous
    ranges of E / world hold nearly equal load.  `counts` is [E] or [layers, E] (summed:
    one permutation per model keeps the weights' layout uniform across layers; per-layer
    permutations are `balanced_permutation(counts[l], world)`).  Greedy longest-
    processing-time assignment under the equal-size constraint."""
    c = counts.to(torch.float64)
    if c.dim() == 2:
        c = c.sum(0)
    E = c.numel()
    if E % world:
        raise ValueError(f"{E} experts do not divide over {world} ranks")
    cap = E // world
    load = [0.0] * world
    bins: List[List[int]] = [[] for _ in range(world)]
    for e in torch.argsort(c, descending=True).tolist():
        r = min((i for i in range(world) if len(bins[i]) < cap), key=lambda i: load[i])
        bins[r].append(e)
        load[r] += float(c[e])
    return [e for b in bins for e in sorted(b)]


def rank_loads(counts: torch.Tensor, world: int, perm: Sequence[int] = None) -> List[float]:
    """Routed pairs per EP rank (contiguous expert ranges) under `perm`."""
    c = counts.to(torch.float64)
    if c.dim() == 2:
        c = c.sum(0)
    if perm is not None:
        c = c[torch.as_tensor(list(perm))]
    return [float(x) for x in c.view(world, -1).sum(1)]


def apply_expert_permutation(weights: Dict[str, torch.Tensor], cfg: ModelConfig, perm: Sequence[int],
                             layers: Sequence[int] = None) -> Dict[str, torch.Tensor]:
    """Renames the experts of every (or the given) MoE layer in place: new expert j is
    old expert perm[j] (router rows and both expert weight stacks move together)."""
    idx = torch.as_tensor(list(perm), dtype=torch.long)
    if sorted(idx.tolist()) != list(range(cfg.num_experts)):
        raise ValueError("perm must be a permutation of the experts")
    for i in (range(cfg.num_layers) if layers is None else layers):
        for name in ("router_w", "experts_gate_up_w", "experts_down_w"):
            key = f"layers.{i}.{name}"
            t = weights.get(key)
            if t is not None:
                weights[key] = t.index_select(0, idx.to(t.device)).contiguous()
    return weights
