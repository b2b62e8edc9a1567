"""One tensor-parallel rank's work on one GPU, without its peers.

    ctx = shard_context(8, "cuda:0")
    llm = LLM("qwen2.5-14b", tp=ctx)        # rank 0's shard of a TP=8 model

The context gives the model rank 0 of `size` ranks: weights are rank 0's shards, every
row-parallel projection runs the fused push GEMM + reduce/norm kernels with a one-rank
receive buffer (the same kernels and data volume on this GPU, no NVLink traffic), and
the vocabulary-parallel logits stay rank 0's slice (sampled from rank 0's candidates).  Timing a decode step on it gives a
TP rank's compute floor; a real TP=N run adds only the collectives' cost, so the two
together say where a TP=N step's time goes.  Outputs are not those of the full model.
"""
from __future__ import annotations

from typing import Optional

import torch

from ..models.transformer import TPContext


def shard_context(size: int, device: Optional[str] = None, fused: bool = True) -> TPContext:
    from .symm import FusedAllReduce
    dev = torch.device(device or f"cuda:{torch.cuda.current_device()}")
    far = FusedAllReduce(device=dev, local=True) if fused and dev.type == "cuda" else None
    return TPContext(0, size, lambda x: x, lambda x: x, fused_ar=far, all_gather_stack=lambda x: x.unsqueeze(0))
