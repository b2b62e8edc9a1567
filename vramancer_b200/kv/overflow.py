"""KV pages borrowed from another GPU's memory, read in place by the attention kernels.

`ExtensiblePagePool` is a KVPool whose page tensor lives in one reserved virtual range
(csrc/vmm.cpp): the first `num_pages` pages are backed by this GPU's HBM; the tail is
unmapped until the block manager runs out of local pages.  Then it maps a chunk of
physical memory created on the lender GPU into the next slot of the tail (one lease of
the lending pool per chunk) and hands out its pages.  A borrowed page is an ordinary
page id to every kernel: decode / prefill attention and the KV writes index the pool
from its base pointer and reach the lender's memory with plain loads and stores over
NVLink.  When every page of a chunk is free again the chunk is unmapped, which returns
the memory to the lender, and its lease is released.

Reclaim (the lender needs its memory back): `reclaim` copies every borrowed page in use
into a free local page and rewrites the sequences' page lists (block manager
`relocate_borrowed`), then unmaps the chunks; pages that find no local room stay (the
engine's preemption frees them at its next step when the pool is short).

A chunk is the least common multiple of the page size and the allocation granularity
(2 MiB on B200), so chunks are whole pages.

Reference parity: core/paged_attention.py:933-999 (_borrow_overflow_page: a lease of
VRAMLendingPool.borrow per overflow page; the bytes stay unused there, cross-GPU
attention is not wired) and experimental/vram_lending.py:389-475 (borrow),
884-1024 (reclaim).
"""
from __future__ import annotations

import math
from typing import Dict, List, Optional, Set

import torch

from .. import ops
from ..utils.observability import get_logger
from .pool import KVPool, KVPoolSpec

log = get_logger("vramancer.kv.overflow")

_DTYPE_NAME = {torch.bfloat16: "bfloat16", torch.float8_e4m3fn: "float8_e4m3fn", torch.float32: "float32",
               torch.float16: "float16", torch.uint8: "uint8"}


class ExtensiblePagePool(KVPool):
    def __init__(self, spec: KVPoolSpec, device, lender_device: Optional[int], max_borrow_pages: int,
                 kv_scale: Optional[torch.Tensor] = None, lending_pool=None):
        """lender_device: the GPU whose memory backs borrowed chunks; None lets the
        lending pool pick a lender per chunk among its registered GPUs."""
        self.spec = spec
        self.device = torch.device(device)
        if self.device.type != "cuda":
            raise ValueError("borrowed KV pages need CUDA devices")
        nat = ops.native()
        dev = self.device.index if self.device.index is not None else torch.cuda.current_device()
        if lender_device is None and lending_pool is None:
            raise ValueError("a lender device or a lending pool is needed")
        self.local_device = dev
        self.lender_device = int(lender_device) if lender_device is not None else None
        self.lending_pool = lending_pool
        lenders = {self.lender_device} if self.lender_device is not None else set(lending_pool.budgets) - {dev}
        if not lenders:
            raise ValueError("no lender GPU registered")
        page = spec.bytes_per_page
        gran = max(nat.vmm_granularity(d) for d in lenders | {dev})
        self.chunk_bytes = page * gran // math.gcd(page, gran)
        self.pages_per_chunk = self.chunk_bytes // page
        self.local_chunks = -(-spec.num_pages // self.pages_per_chunk)
        self.max_chunks = -(-max(1, max_borrow_pages) // self.pages_per_chunk)
        total = (self.local_chunks + self.max_chunks) * self.chunk_bytes
        self.access = sorted(lenders | {dev})
        self.base = nat.vmm_reserve(total, gran)
        nat.vmm_map(self.base, 0, self.local_chunks * self.chunk_bytes, dev, self.access, False)
        total_pages = (self.local_chunks + self.max_chunks) * self.pages_per_chunk
        shape = [total_pages, spec.num_layers, 2, spec.kv_heads, spec.page_size, spec.row]
        self.cache = nat.tensor_from_ptr(self.base, shape, _DTYPE_NAME[spec.dtype], dev)
        self.cache[:self.local_chunks * self.pages_per_chunk].zero_()
        self.first_borrow_page = self.local_chunks * self.pages_per_chunk
        self.is_fp8 = spec.dtype == torch.float8_e4m3fn
        if self.is_fp8:
            if kv_scale is None:
                kv_scale = torch.ones(spec.num_layers, 2, spec.kv_heads, dtype=torch.float32)
            self.kv_scale = kv_scale.to(self.device, torch.float32).contiguous()
        else:
            self.kv_scale = None
        self._free_in_chunk: Dict[int, Set[int]] = {}      # mapped chunk -> free page ids
        self._leases: Dict[int, object] = {}
        self._chunk_lender: Dict[int, int] = {}
        self._mgr = None
        self.reclaim_requested = False
        self.stats = {"chunks_mapped": 0, "chunks_unmapped": 0, "pages_borrowed": 0, "pages_reclaimed": 0}

    # ----------------------------------------------------------------- chunk mapping
    def _chunk_of(self, page: int) -> int:
        return (page - self.first_borrow_page) // self.pages_per_chunk

    def _chunk_offset(self, c: int) -> int:
        return (self.local_chunks + c) * self.chunk_bytes

    def borrowable_pages(self) -> int:
        free_mapped = sum(len(s) for s in self._free_in_chunk.values())
        return free_mapped + (self.max_chunks - len(self._free_in_chunk)) * self.pages_per_chunk

    def _map_chunk(self) -> Optional[int]:
        for c in range(self.max_chunks):
            if c not in self._free_in_chunk:
                break
        else:
            return None
        lease = None
        lender = self.lender_device
        if self.lending_pool is not None:
            lease = self.lending_pool.borrow(self.local_device, self.chunk_bytes, purpose="kv_overflow",
                                             on_reclaim=self._on_reclaim)
            if lease is None:
                return None
            if lender is None:
                lender = lease.lender
            if lender not in self.access:
                self.lending_pool.release(lease.lease_id)
                return None
        try:
            ops.native().vmm_map(self.base, self._chunk_offset(c), self.chunk_bytes, lender, self.access, False)
        except Exception:
            if lease is not None:
                self.lending_pool.release(lease.lease_id)
            raise
        p0 = self.first_borrow_page + c * self.pages_per_chunk
        self.cache[p0:p0 + self.pages_per_chunk].zero_()    # finite values in never-written slots
        self._free_in_chunk[c] = set(range(p0, p0 + self.pages_per_chunk))
        self._chunk_lender[c] = lender
        if lease is not None:
            self._leases[c] = lease
        self.stats["chunks_mapped"] += 1
        log.info("KV overflow: mapped %d pages of cuda:%d memory into cuda:%d's pool", self.pages_per_chunk,
                 lender, self.local_device)
        return c

    def _unmap_chunk(self, c: int) -> None:
        ops.native().vmm_unmap(self.base, self._chunk_offset(c))
        del self._free_in_chunk[c]
        self._chunk_lender.pop(c, None)
        lease = self._leases.pop(c, None)
        if lease is not None:
            self.lending_pool.release(lease.lease_id)
        self.stats["chunks_unmapped"] += 1

    # ----------------------------------------------------------------- block manager hooks
    def take_page(self, n: int = 1) -> Optional[int]:
        """A free borrowed page (mapping a new chunk from the lender when needed)."""
        for free in self._free_in_chunk.values():
            if free:
                self.stats["pages_borrowed"] += 1
                return self._pop(free)
        c = self._map_chunk()
        if c is None:
            return None
        self.stats["pages_borrowed"] += 1
        return self._pop(self._free_in_chunk[c])

    @staticmethod
    def _pop(free: Set[int]) -> int:
        p = min(free)
        free.remove(p)
        return p

    def give_back(self, page: int) -> None:
        """A borrowed page is no longer referenced; a chunk with no page in use is unmapped."""
        c = self._chunk_of(page)
        free = self._free_in_chunk[c]
        free.add(page)
        if len(free) == self.pages_per_chunk:
            self._unmap_chunk(c)

    def attach(self, mgr) -> None:
        """Installs the hooks on a PagedKVCacheManager over this pool."""
        mgr._overflow = self.take_page
        mgr._release_borrowed = self.give_back
        mgr._overflow_capacity = self.borrowable_pages
        self._mgr = mgr

    def _on_reclaim(self, lease, urgency) -> None:
        # called from the lending pool's monitor thread: the engine performs the move
        # between two steps (LLMEngine.step), never under a running kernel
        self.reclaim_requested = True

    def reclaim(self, mgr=None) -> int:
        """Moves borrowed pages in use back into free local pages (page copies within the
        pool) and releases the chunks that empty; returns the pages moved."""
        mgr = mgr or self._mgr
        self.reclaim_requested = False

        def copy(src: int, dst: int) -> None:
            self.cache[dst].copy_(self.cache[src])
        moved = mgr.relocate_borrowed(copy)
        self.stats["pages_reclaimed"] += moved
        return moved

    def nbytes(self) -> int:
        return self.local_chunks * self.chunk_bytes

    def close(self) -> None:
        if getattr(self, "base", None):
            for c in list(self._free_in_chunk):
                lease = self._leases.pop(c, None)
                if lease is not None and self.lending_pool is not None:
                    self.lending_pool.release(lease.lease_id)
            self.cache = None
            ops.native().vmm_free(self.base)
            self.base = None
