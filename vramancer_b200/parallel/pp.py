"""Pipeline x tensor parallelism over processes: a PP x TP grid of ranks, one GPU each.

Ranks are stage-major (rank = stage * tp + tp_rank).  Each stage owns a contiguous
layer range (an even split, or `layer_split`), its own paged KV pool and its own CUDA
graphs; inside a stage the layers are tensor-parallel over the stage's TP group (the
fused NVLink all-reduce of parallel/symm.py).  Between stages the residual stream
crosses NCCL point-to-point (send / recv between ranks holding the same tp_rank).
The last stage samples; its sampled token ids are broadcast to every rank, so every
rank's engine takes the same scheduling decisions (lockstep, as under plain TP) and
the first stage embeds the right tokens next step.

Overlap.  A forward can be cut into `microbatches` groups of sequences: stage s sends
group m on and starts group m + 1 while stage s + 1 works on group m, so the stages
run concurrently within one forward.  That pays for prefill (compute-bound: the
pieces cost their share of the work); a decode step streams each stage's weights once
per group, so decode keeps one group by default (`decode_microbatches=1`).

Reference parity: core/backends.py:1314-1352 (accelerate device_map="auto" split) and
core/inference_pipeline.py:445-495 (activation hops by a patched send_to_device), one
process for all GPUs, no KV cache across the split in its manual path.  Here each stage
is a process with its own paged KV, and hops are NCCL p2p.
"""
from __future__ import annotations

from dataclasses import replace
from typing import List, Optional, Sequence, Tuple

import torch
import torch.distributed as dist

from ..models.transformer import DecoderModel, ForwardBatch


class PPGrid:
    """Stage / TP coordinates of this rank and the process groups of the grid."""

    def __init__(self, pp: int, tp: int, layer_split: Optional[Sequence[int]] = None, num_layers: int = 0):
        if not dist.is_initialized():
            raise RuntimeError("pipeline parallelism needs torch.distributed (torchrun)")
        world, rank = dist.get_world_size(), dist.get_rank()
        if pp * tp != world:
            raise ValueError(f"pp x tp = {pp} x {tp} != world size {world}")
        self.pp, self.tp, self.rank = pp, tp, rank
        self.stage, self.tp_rank = divmod(rank, tp)
        backend = dist.get_backend()
        self.tp_group = None
        for s in range(pp):      # every rank creates every group, in the same order
            g = dist.new_group(list(range(s * tp, (s + 1) * tp)), backend=backend) if tp > 1 else None
            if s == self.stage:
                self.tp_group = g
        self.prev = rank - tp if self.stage > 0 else None
        self.next = rank + tp if self.stage < pp - 1 else None
        self.sampler_root = (pp - 1) * tp          # broadcasts the sampled ids
        self.bounds = self._bounds(layer_split, num_layers) if num_layers else None

    def _bounds(self, layer_split, L: int) -> List[Tuple[int, int]]:
        if layer_split is None:
            cuts = [round(s * L / self.pp) for s in range(self.pp + 1)]
        else:
            if len(layer_split) != self.pp or sum(layer_split) != L:
                raise ValueError("layer_split must give every stage's layer count and sum to the layers")
            cuts = [0]
            for n in layer_split:
                cuts.append(cuts[-1] + n)
        return [(cuts[s], cuts[s + 1]) for s in range(self.pp)]

    @property
    def is_first(self) -> bool:
        return self.stage == 0

    @property
    def is_last(self) -> bool:
        return self.stage == self.pp - 1

    def layers(self, num_layers: int) -> Tuple[int, int]:
        if self.bounds is None:
            self.bounds = self._bounds(None, num_layers)
        return self.bounds[self.stage]


def split_batch(batch: ForwardBatch, groups: int) -> List[ForwardBatch]:
    """Cuts a forward into `groups` pieces by whole sequences (decode rows or prefill
    sequences); logits rows are renumbered within each piece."""
    if batch.is_decode:
        B = batch.num_tokens
        per = (B + groups - 1) // groups
        out = []
        for a in range(0, B, per):
            b = min(B, a + per)
            out.append(replace(batch, input_ids=batch.input_ids[a:b], positions=batch.positions[a:b],
                               slot_mapping=batch.slot_mapping[a:b], block_tables=batch.block_tables[a:b],
                               context_lens=batch.context_lens[a:b]))
        return out
    cu = batch.cu_q.tolist()
    S = len(cu) - 1
    per = (S + groups - 1) // groups
    rows = batch.logits_rows.tolist() if batch.logits_rows is not None else None
    out = []
    for s0 in range(0, S, per):
        s1 = min(S, s0 + per)
        t0, t1 = cu[s0], cu[s1]
        dev = batch.cu_q.device
        sub_cu = torch.tensor([c - t0 for c in cu[s0:s1 + 1]], dtype=batch.cu_q.dtype, device=dev)
        lr = None
        if rows is not None:
            lr = torch.tensor([r - t0 for r in rows if t0 <= r < t1], dtype=batch.logits_rows.dtype, device=dev)
        out.append(replace(batch, input_ids=batch.input_ids[t0:t1], positions=batch.positions[t0:t1],
                           slot_mapping=batch.slot_mapping[t0:t1], block_tables=batch.block_tables[s0:s1],
                           context_lens=batch.context_lens[s0:s1], cu_q=sub_cu,
                           max_q_len=max(cu[i + 1] - cu[i] for i in range(s0, s1)), logits_rows=lr))
    return out


class PPStageModel:
    """This rank's stage: the DecoderModel of its layers (TP-sharded over the stage's
    group) with the NCCL hops around it.  Same surface as DecoderModel for the model
    runner: forward() returns logits on the last stage and None elsewhere."""

    def __init__(self, cfg, weights, grid: PPGrid, *, device, dtype=torch.bfloat16, tp=None,
                 prefill_microbatches: int = 0, decode_microbatches: int = 1):
        first, last = grid.layers(cfg.num_layers)
        self.model = DecoderModel(cfg, weights, device=device, dtype=dtype, first_layer=first, last_layer=last,
                                  tp=tp)
        self.grid = grid
        self.cfg = cfg
        self.device = self.model.device
        self.dtype = dtype
        self.kvh = self.model.kvh
        self.tp = tp
        self.prefill_microbatches = prefill_microbatches or grid.pp
        self.decode_microbatches = max(1, decode_microbatches)
        self.hops = 0

    @property
    def num_local_layers(self) -> int:
        return self.model.num_local_layers

    @property
    def first_layer(self) -> int:
        return self.model.first_layer

    @property
    def last_layer(self) -> int:
        return self.model.last_layer

    def fold_norms(self) -> bool:
        return False

    @property
    def vocab_parallel(self) -> bool:
        return self.grid.is_last and self.model.vocab_parallel

    def set_vp_logits(self, on: bool) -> None:
        self.model.set_vp_logits(on)

    def sample_vocab_parallel(self, *a, **kw):
        return self.model.sample_vocab_parallel(*a, **kw)

    def _stage(self, batch: ForwardBatch, pool) -> Optional[torch.Tensor]:
        g = self.grid
        h = None
        if not g.is_first:
            h = torch.empty(batch.num_tokens, self.cfg.hidden_size, dtype=self.dtype, device=self.device)
            dist.recv(h, src=g.prev)
            self.hops += 1
        out = self.model.forward(batch, pool, hidden=h)
        if not g.is_last:
            dist.send(out.contiguous(), dst=g.next)
            return None
        return out

    def forward(self, batch: ForwardBatch, pool, hidden=None) -> Optional[torch.Tensor]:
        groups = self.decode_microbatches if batch.is_decode else self.prefill_microbatches
        nseq = batch.num_tokens if batch.is_decode else batch.cu_q.numel() - 1
        groups = max(1, min(groups, nseq))
        if groups == 1 or self.grid.pp == 1:
            return self._stage(batch, pool)
        outs = [self._stage(b, pool) for b in split_batch(batch, groups)]
        if not self.grid.is_last:
            return None
        outs = [o for o in outs if o is not None and o.shape[0] > 0]
        return torch.cat(outs, 0) if outs else None

    def share_sampled(self, ids: torch.Tensor) -> None:
        """Every rank gets the last stage's sampled ids (in place, int32 [n])."""
        if self.grid.pp > 1:
            dist.broadcast(ids, src=self.grid.sampler_root)
