"""GPU resource scheduler: device discovery, memory-block bookkeeping, KV reservations,
next-layer prediction and block migration.

Blocks are accounted in MB per GPU (optionally backed by a tensor); allocation picks
the GPU with the most free memory after reservations unless one is requested; a
migration moves the backing tensor with the transfer manager.

Reference parity: core/scheduler.py:63-540 (AllocatedBlock, SimpleScheduler:
get_available_gpus, refresh_gpu_info, allocate_block, release_block,
predict_next_layers, find_alternate_gpu, migrate_block, total_allocated_mb,
estimate_kv_cache_mb, reserve_kv_cache, release_kv_cache, kv_cache_reserved_mb).
"""
from __future__ import annotations

import itertools
import threading
from dataclasses import dataclass, field
from typing import Any, Dict, List, Optional

import torch


@dataclass
class AllocatedBlock:
    id: int
    gpu_id: int
    size_mb: float
    priority: int = 5
    tensor: Optional[torch.Tensor] = None
    meta: Dict[str, Any] = field(default_factory=dict)


class Scheduler:
    def __init__(self, gpus: Optional[List[Dict[str, Any]]] = None, reserve_frac: float = 0.10):
        """gpus: [{"id", "name", "total_mb", "free_mb"}] (detected when None)."""
        self._gpus = gpus if gpus is not None else self._detect_gpus()
        self.reserve_frac = reserve_frac
        self._blocks: Dict[int, AllocatedBlock] = {}
        self._kv: Dict[int, float] = {}
        self._ids = itertools.count(1)
        self._lock = threading.RLock()
        self.transfer = None

    # ---------------------------------------------------------------- discovery
    @staticmethod
    def _detect_gpus() -> List[Dict[str, Any]]:
        out = []
        if not torch.cuda.is_available():
            return out
        for i in range(torch.cuda.device_count()):
            free, total = torch.cuda.mem_get_info(i)
            out.append({"id": i, "name": torch.cuda.get_device_name(i), "total_mb": total / 2**20,
                        "free_mb": free / 2**20})
        return out

    def refresh_gpu_info(self) -> None:
        if torch.cuda.is_available():
            self._gpus = self._detect_gpus()

    def get_available_gpus(self) -> List[Dict[str, Any]]:
        return [dict(g, usable_mb=self.usable_mb(g["id"])) for g in self._gpus]

    def _gpu(self, gid: int) -> Dict[str, Any]:
        for g in self._gpus:
            if g["id"] == gid:
                return g
        raise KeyError(f"no GPU {gid}")

    def usable_mb(self, gid: int) -> float:
        g = self._gpu(gid)
        return g["free_mb"] - g["total_mb"] * self.reserve_frac - self.total_allocated_mb(gid) - self._kv.get(gid, 0.0)

    # ---------------------------------------------------------------- blocks
    def _find_best_gpu(self, size_mb: float, exclude: Optional[int] = None) -> int:
        cands = [g["id"] for g in self._gpus if g["id"] != exclude and self.usable_mb(g["id"]) >= size_mb]
        if not cands:
            raise MemoryError(f"no GPU has {size_mb:.1f} MB free")
        return max(cands, key=self.usable_mb)

    def allocate_block(self, size_mb: float, priority: int = 5, gpu_id: Optional[int] = None,
                       materialize: bool = False, **meta) -> AllocatedBlock:
        with self._lock:
            gid = self._find_best_gpu(size_mb) if gpu_id is None else gpu_id
            if gpu_id is not None and self.usable_mb(gid) < size_mb:
                raise MemoryError(f"GPU {gid} has {self.usable_mb(gid):.1f} MB usable, {size_mb:.1f} requested")
            t = None
            if materialize:
                t = torch.empty(int(size_mb * 2**20), dtype=torch.uint8, device=f"cuda:{gid}")
            b = AllocatedBlock(next(self._ids), gid, size_mb, priority, t, meta)
            self._blocks[b.id] = b
            return b

    def release_block(self, block: AllocatedBlock) -> None:
        with self._lock:
            self._blocks.pop(block.id, None)
            block.tensor = None

    def find_alternate_gpu(self, exclude: Optional[int] = None, size_mb: float = 0.0) -> int:
        return self._find_best_gpu(size_mb, exclude=exclude)

    def migrate_block(self, block: AllocatedBlock, target_gpu: int) -> None:
        with self._lock:
            if self.usable_mb(target_gpu) < block.size_mb:
                raise MemoryError(f"GPU {target_gpu} cannot take {block.size_mb:.1f} MB")
            if block.tensor is not None and block.tensor.is_cuda:
                if self.transfer is None:
                    from .transfer import TransferManager
                    self.transfer = TransferManager()
                block.tensor = self.transfer.send_tensor(block.tensor, target_gpu)
            block.gpu_id = target_gpu

    @property
    def allocated_blocks(self) -> List[AllocatedBlock]:
        return list(self._blocks.values())

    def total_allocated_mb(self, gpu_id: Optional[int] = None) -> float:
        return sum(b.size_mb for b in self._blocks.values() if gpu_id is None or b.gpu_id == gpu_id)

    # ---------------------------------------------------------------- prediction
    @staticmethod
    def predict_next_layers(current_layers: List[int], num_layers: int, lookahead: int = 2) -> List[int]:
        """The layers after the highest one in use (decode walks layers in order and
        wraps to 0 for the next token)."""
        if not current_layers or num_layers <= 0:
            return list(range(min(lookahead, num_layers)))
        last = max(current_layers)
        return [(last + k) % num_layers for k in range(1, lookahead + 1)]

    # ---------------------------------------------------------------- KV reservations
    @staticmethod
    def estimate_kv_cache_mb(num_layers: int, num_kv_heads: int, head_dim: int, batch: int, seq_len: int,
                             dtype_bytes: int = 2) -> float:
        return 2 * num_layers * num_kv_heads * head_dim * batch * seq_len * dtype_bytes / 2**20

    def reserve_kv_cache(self, gpu_id: int, size_mb: float) -> None:
        with self._lock:
            if self.usable_mb(gpu_id) < size_mb:
                raise MemoryError(f"GPU {gpu_id}: cannot reserve {size_mb:.1f} MB of KV cache")
            self._kv[gpu_id] = self._kv.get(gpu_id, 0.0) + size_mb

    def release_kv_cache(self, gpu_id: int, size_mb: float) -> None:
        with self._lock:
            self._kv[gpu_id] = max(0.0, self._kv.get(gpu_id, 0.0) - size_mb)

    def kv_cache_reserved_mb(self, gpu_id: Optional[int] = None) -> float:
        return sum(v for k, v in self._kv.items() if gpu_id is None or k == gpu_id)
