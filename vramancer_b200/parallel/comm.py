"""Process-group plumbing: one process per GPU, torch.distributed over NCCL.

`init_distributed()` reads RANK / LOCAL_RANK / WORLD_SIZE / MASTER_* (torchrun) and
creates the default group with a short timeout, so that a rank that never arrives
ends its peers' next collective with an error instead of a hang.  `tp_context()`
builds the TPContext the model uses: all-reduce of row-parallel partial sums and
all-gather of vocab-parallel logits, NCCL-backed (capturable in CUDA graphs).

Reference parity: core/tensor_parallel.py:67-80 (single-process
torch.cuda.nccl.all_reduce with a CPU fallback), core/transfer_manager.py:343-380
(init_process_group only when MASTER_ADDR is set).
"""
from __future__ import annotations

import datetime
import os
from dataclasses import dataclass
from typing import Optional

import torch
import torch.distributed as dist

from ..models.transformer import TPContext


@dataclass
class DistInfo:
    rank: int = 0
    local_rank: int = 0
    world_size: int = 1
    backend: str = "none"

    @property
    def is_distributed(self) -> bool:
        return self.world_size > 1


def env_dist_info() -> DistInfo:
    return DistInfo(rank=int(os.environ.get("RANK", 0)), local_rank=int(os.environ.get("LOCAL_RANK", 0)),
                    world_size=int(os.environ.get("WORLD_SIZE", 1)))


def init_distributed(backend: Optional[str] = None, timeout_s: float = 120.0) -> DistInfo:
    info = env_dist_info()
    if info.world_size <= 1:
        return info
    if backend is None:
        backend = "nccl" if torch.cuda.is_available() else "gloo"
    if torch.cuda.is_available():
        torch.cuda.set_device(info.local_rank)
    if not dist.is_initialized():
        kw = {}
        if backend == "nccl":
            kw["device_id"] = torch.device("cuda", info.local_rank)
        dist.init_process_group(backend=backend, timeout=datetime.timedelta(seconds=timeout_s), **kw)
    info.backend = backend
    return info


def tp_context(group=None) -> Optional[TPContext]:
    if not dist.is_initialized():
        return None
    size = dist.get_world_size(group)
    if size == 1:
        return None
    rank = dist.get_rank(group)

    def all_reduce(x: torch.Tensor) -> torch.Tensor:
        dist.all_reduce(x, group=group)
        return x

    def all_gather_last(x: torch.Tensor) -> torch.Tensor:
        parts = [torch.empty_like(x) for _ in range(size)]
        dist.all_gather(parts, x.contiguous(), group=group)
        return torch.cat(parts, dim=-1)

    def all_gather_stack(x: torch.Tensor) -> torch.Tensor:
        out = torch.empty((size,) + tuple(x.shape), dtype=x.dtype, device=x.device)
        dist.all_gather_into_tensor(out, x.contiguous(), group=group)
        return out

    fused = None
    if torch.cuda.is_available() and dist.get_backend(group) == "nccl" and \
            os.environ.get("VRM_FUSED_AR", "1") not in ("0", "false"):
        from .symm import FusedAllReduce
        fused = FusedAllReduce(group, max_tokens=int(os.environ.get("VRM_FUSED_AR_MAX_TOKENS", "128")))
    return TPContext(rank, size, all_reduce, all_gather_last, fused_ar=fused, all_gather_stack=all_gather_stack)


def barrier() -> None:
    if dist.is_initialized():
        if dist.get_backend() == "nccl":
            dist.barrier(device_ids=[torch.cuda.current_device()])
        else:
            dist.barrier()


def max_over_ranks(v: float) -> float:
    if not dist.is_initialized() or dist.get_world_size() == 1:
        return v
    dev = torch.device("cuda", torch.cuda.current_device()) if dist.get_backend() == "nccl" else torch.device("cpu")
    t = torch.tensor([v], dtype=torch.float64, device=dev)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def destroy() -> None:
    if dist.is_initialized():
        dist.destroy_process_group()
