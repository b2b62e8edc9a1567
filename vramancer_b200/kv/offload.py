"""Host tier for the prefix cache: KV pages evicted from VRAM are kept in pinned host
memory (and optionally behind it on NVMe through the hierarchical memory manager), and
a later request with the same prefix gets them back with one host-to-device copy
instead of recomputing the prefill.

The paged manager calls `on_evict` when it recycles a cached page (ref count 0, still
holding a prefix) and `restore` when a prefix misses in VRAM but hits here.  Copies
run on the current CUDA stream, so stream order places the eviction copy before any
later write of the recycled page and the restore copy before the kernels that read it.

Reference parity: core/paged_attention_offload.py:14-70 (evict cold pages to the
hierarchical memory manager, a DRAM dict) and the LRU eviction path of
core/paged_attention.py:1001-1103 (compress, parity, offload to L3).
"""
from __future__ import annotations

import threading
from collections import OrderedDict
from typing import Dict, List, Optional, Sequence, Tuple

import torch


class KVOffloader:
    def __init__(self, pools: Sequence[torch.Tensor], max_pages: int = 256, hierarchy=None):
        """pools: the KV cache tensors [pages, ...] of this rank (one per pipeline stage
        on this process); max_pages: host pages kept; hierarchy: optional
        HierarchicalMemoryManager that receives host pages pushed out of this store."""
        self.pools = list(pools)
        self.max_pages = max_pages
        self.hierarchy = hierarchy
        pin = any(p.is_cuda for p in self.pools) and torch.cuda.is_available()
        self.host = [torch.empty((max_pages,) + tuple(p.shape[1:]), dtype=p.dtype, pin_memory=pin)
                     for p in self.pools]
        self._free = list(range(max_pages - 1, -1, -1))
        self._index: "OrderedDict[bytes, Tuple[int, Tuple[int, ...]]]" = OrderedDict()
        self._spilled: Dict[bytes, Tuple[int, ...]] = {}
        self._lock = threading.Lock()
        self.stats = {"offloaded": 0, "restored": 0, "dropped": 0, "spilled": 0, "unspilled": 0}

    @property
    def page_bytes(self) -> int:
        return sum(h[0].numel() * h.element_size() for h in self.host)

    def __len__(self) -> int:
        return len(self._index)

    def _slot(self) -> int:
        if self._free:
            return self._free.pop()
        h, (slot, toks) = self._index.popitem(last=False)      # oldest host page
        if self.hierarchy is not None:
            from ..memory.hierarchy import MemoryBlock, Tier
            for i, hp in enumerate(self.host):
                bid = f"kv:{h.hex()}:{i}"
                self.hierarchy.register_block(MemoryBlock(bid, tuple(hp[slot].shape), hp.dtype), Tier.L5,
                                              hp[slot].clone())
            self._spilled[h] = toks
            self.stats["spilled"] += 1
        else:
            self.stats["dropped"] += 1
        return slot

    def on_evict(self, page: int, key: bytes, tokens: Tuple[int, ...]) -> None:
        with self._lock:
            if key in self._index:
                self._index.move_to_end(key)
                return
            slot = self._slot()
            for hp, pool in zip(self.host, self.pools):
                hp[slot].copy_(pool[page], non_blocking=True)
            self._index[key] = (slot, tuple(tokens))
            self.stats["offloaded"] += 1

    def has(self, key: bytes, tokens: Tuple[int, ...]) -> bool:
        with self._lock:
            e = self._index.get(key)
            if e is not None:
                return e[1] == tuple(tokens)
            return self._spilled.get(key) == tuple(tokens)

    def restore(self, key: bytes, page: int) -> None:
        with self._lock:
            e = self._index.get(key)
            if e is None:
                if key not in self._spilled:
                    raise KeyError("prefix page not in the host tier")
                toks = self._spilled.pop(key)
                slot = self._slot()
                for i, hp in enumerate(self.host):
                    bid = f"kv:{key.hex()}:{i}"
                    hp[slot].copy_(self.hierarchy.get(bid, device="cpu"))
                    self.hierarchy.remove(bid)
                self._index[key] = (slot, toks)
                self.stats["unspilled"] += 1
                e = self._index[key]
            self._index.move_to_end(key)
            slot = e[0]
            for hp, pool in zip(self.host, self.pools):
                pool[page].copy_(hp[slot], non_blocking=True)
            self.stats["restored"] += 1
