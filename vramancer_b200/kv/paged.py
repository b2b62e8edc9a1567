"""Host-side block manager of the paged KV pool.

Per request it keeps the list of physical pages (the block table the kernels read)
and the token count; pages carry reference counts so that `fork` shares a prefix
copy-on-write, and full pages are registered in a prefix cache keyed by a chained
content hash *and* verified against the stored token ids (the reference keyed its
prefix cache on Python `hash(tuple)` without a collision check,
core/paged_attention.py:542).  Pages whose reference count drops to zero stay
reusable in an LRU list until the allocator needs them back.

When the pool is exhausted, an optional `overflow` callback (the VRAM lending pool)
may supply pages from another device's pool; those are tracked as borrowed and freed
back to their lender.

Reference parity: PagedKVCacheManager, core/paged_attention.py:192-1509 (allocate
403-429, append_token 431-459, free 461-491, fork 493-515, prefix cache 521-562,
LRU evict 1001-1103, borrow overflow 933-999).
"""
from __future__ import annotations

import hashlib
import threading
from collections import OrderedDict, deque
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Tuple

from .pool import PAGE_SIZE


class OutOfPages(RuntimeError):
    pass


@dataclass
class SeqState:
    pages: List[int] = field(default_factory=list)
    num_tokens: int = 0
    cached_tokens: int = 0          # tokens whose KV came from the prefix cache
    hashes: List[bytes] = field(default_factory=list)   # chain hash of each full page


def _chain_hash(prev: bytes, tokens: Sequence[int]) -> bytes:
    h = hashlib.blake2b(digest_size=16)
    h.update(prev)
    h.update(b"".join(int(t).to_bytes(4, "little", signed=False) for t in tokens))
    return h.digest()


class PagedKVCacheManager:
    def __init__(self, num_pages: int, page_size: int = PAGE_SIZE, enable_prefix_cache: bool = True,
                 overflow: Optional[Callable[[int], Optional[int]]] = None,
                 release_borrowed: Optional[Callable[[int], None]] = None, offload=None):
        self.num_pages = num_pages
        self.page_size = page_size
        self.enable_prefix_cache = enable_prefix_cache
        self._free: deque = deque(range(num_pages))
        self._ref = [0] * num_pages
        self._seqs: Dict[object, SeqState] = {}
        self._prefix: Dict[bytes, int] = {}                 # chain hash -> page
        self._page_key: Dict[int, Tuple[bytes, Tuple[int, ...]]] = {}
        self._lru: "OrderedDict[int, None]" = OrderedDict()  # cached pages with ref 0
        self._overflow = overflow
        self._release_borrowed = release_borrowed
        self._overflow_capacity: Optional[Callable[[], int]] = None   # pages the overflow can still give
        self.offload = offload                              # host tier of the prefix cache (kv/offload.py)
        self._borrowed: Dict[int, int] = {}                 # page id (>= num_pages) -> ref
        self._lock = threading.RLock()
        self._cow: List[Tuple[int, int]] = []
        self.stats_counters = {"prefix_hits": 0, "prefix_queries": 0, "evictions": 0, "cow_copies": 0,
                               "borrowed": 0}

    # ------------------------------------------------------------------ capacity
    def num_free_pages(self) -> int:
        with self._lock:
            return len(self._free) + len(self._lru)

    def pages_needed(self, num_tokens: int) -> int:
        return (num_tokens + self.page_size - 1) // self.page_size

    def can_allocate(self, num_tokens: int) -> bool:
        extra = self._overflow_capacity() if self._overflow_capacity is not None else 0
        return self.pages_needed(num_tokens) <= self.num_free_pages() + extra

    def relocate_borrowed(self, copy_page: Callable[[int, int], None]) -> int:
        """Moves borrowed pages that are in use into free local pages: copy_page(src, dst)
        copies the data, every sequence's page list is rewritten and the borrowed page is
        released.  Stops when no local page is free; returns the pages moved."""
        moved = 0
        with self._lock:
            for p in sorted(self._borrowed):
                if not self._free:
                    break
                q = self._free.popleft()
                copy_page(p, q)
                refs = self._borrowed[p]
                self._ref[q] = refs
                for st in self._seqs.values():
                    st.pages = [q if x == p else x for x in st.pages]
                key = self._page_key.pop(p, None)
                if key is not None:
                    self._page_key[q] = key
                    if self._prefix.get(key[0]) == p:
                        self._prefix[key[0]] = q
                self._borrowed[p] = 1
                self._decref(p)                 # releases the borrowed page
                moved += 1
        return moved

    # ------------------------------------------------------------------ page alloc
    def _take_page(self) -> int:
        if self._free:
            p = self._free.popleft()
        elif self._lru:
            p, _ = self._lru.popitem(last=False)
            key = self._page_key.pop(p, None)
            if key is not None and self._prefix.get(key[0]) == p:
                del self._prefix[key[0]]
                if self.offload is not None:
                    self.offload.on_evict(p, key[0], key[1])
            self.stats_counters["evictions"] += 1
        else:
            p = self._overflow(1) if self._overflow is not None else None
            if p is None:
                raise OutOfPages("KV pool exhausted")
            self._borrowed[p] = 0
            self.stats_counters["borrowed"] += 1
        self._incref(p)
        return p

    def _incref(self, p: int) -> None:
        if p in self._borrowed:
            self._borrowed[p] += 1
            return
        if self._ref[p] == 0:
            self._lru.pop(p, None)
        self._ref[p] += 1

    def _decref(self, p: int) -> None:
        if p in self._borrowed:
            self._borrowed[p] -= 1
            if self._borrowed[p] == 0:
                del self._borrowed[p]
                if self._release_borrowed is not None:
                    self._release_borrowed(p)
            return
        self._ref[p] -= 1
        assert self._ref[p] >= 0, f"page {p} refcount underflow"
        if self._ref[p] == 0:
            if p in self._page_key:
                self._lru[p] = None     # keep it findable by the prefix cache
            else:
                self._free.append(p)

    # ------------------------------------------------------------------ sequences
    def allocate(self, seq_id, num_tokens: int, token_ids: Optional[Sequence[int]] = None) -> int:
        """Reserves pages for a new sequence of `num_tokens` (the prompt).  With token ids
        and the prefix cache on, leading full pages already in the cache are shared.
        Returns the number of leading tokens whose KV is already present."""
        with self._lock:
            if seq_id in self._seqs:
                raise KeyError(f"sequence {seq_id!r} already allocated")
            st = SeqState()
            cached = 0
            if self.enable_prefix_cache and token_ids is not None:
                self.stats_counters["prefix_queries"] += 1
                prev = b""
                # keep at least one token to compute: its logits start generation
                max_full = (len(token_ids) - 1) // self.page_size
                for i in range(max_full):
                    toks = tuple(int(t) for t in token_ids[i * self.page_size:(i + 1) * self.page_size])
                    h = _chain_hash(prev, toks)
                    p = self._prefix.get(h)
                    if p is None and self.offload is not None and self.offload.has(h, toks):
                        # host tier hit: bring the page back (stream-ordered copy)
                        try:
                            p = self._take_page()
                        except OutOfPages:
                            break
                        self.offload.restore(h, p)
                        self._prefix[h] = p
                        self._page_key[p] = (h, toks)
                        self.stats_counters["offload_hits"] = self.stats_counters.get("offload_hits", 0) + 1
                        st.pages.append(p)
                        st.hashes.append(h)
                        prev = h
                        cached += self.page_size
                        continue
                    if p is None or self._page_key.get(p, (None, None))[1] != toks:
                        break
                    self._incref(p)
                    st.pages.append(p)
                    st.hashes.append(h)
                    prev = h
                    cached += self.page_size
                if cached:
                    self.stats_counters["prefix_hits"] += 1
            need = self.pages_needed(num_tokens) - len(st.pages)
            if need > len(self._free) + len(self._lru) and self._overflow is None:
                for p in st.pages:
                    self._decref(p)
                raise OutOfPages(f"need {need} pages, {len(self._free) + len(self._lru)} free")
            try:
                for _ in range(need):
                    st.pages.append(self._take_page())
            except OutOfPages:
                for p in st.pages:
                    self._decref(p)
                raise
            st.num_tokens = num_tokens
            st.cached_tokens = cached
            self._seqs[seq_id] = st
            return cached

    def append_slots(self, seq_id, n: int = 1) -> List[int]:
        """Grows the sequence by n tokens; returns their cache slots (page*ps + offset).
        A shared (forked) last page is copied first: the returned list of
        (src, dst) copies is available from `pop_cow_copies`."""
        with self._lock:
            st = self._seqs[seq_id]
            slots = []
            for _ in range(n):
                pos = st.num_tokens
                pi, off = divmod(pos, self.page_size)
                if pi == len(st.pages):
                    st.pages.append(self._take_page())
                else:
                    self._ensure_private(st, pi)
                slots.append(st.pages[pi] * self.page_size + off)
                st.num_tokens += 1
            return slots

    def slots_for(self, seq_id, start: int, n: int) -> List[int]:
        """Slots of tokens [start, start+n) (already allocated)."""
        st = self._seqs[seq_id]
        ps = self.page_size
        return [st.pages[t // ps] * ps + t % ps for t in range(start, start + n)]

    def _ensure_private(self, st: SeqState, pi: int) -> None:
        p = st.pages[pi]
        if p in self._borrowed:
            return
        if self._ref[p] > 1:
            q = self._take_page()
            self._decref(p)
            st.pages[pi] = q
            self._cow.append((p, q))
            self.stats_counters["cow_copies"] += 1

    def pop_cow_copies(self) -> List[Tuple[int, int]]:
        """Page copies (src, dst) the engine must perform before the next write."""
        with self._lock:
            c, self._cow = self._cow, []
            return c

    def commit_prefix(self, seq_id, token_ids: Sequence[int]) -> None:
        """Registers the sequence's full pages (whose KV is now written) in the prefix cache."""
        if not self.enable_prefix_cache:
            return
        with self._lock:
            st = self._seqs[seq_id]
            full = min(len(token_ids), st.num_tokens) // self.page_size
            prev = st.hashes[-1] if st.hashes else b""
            for i in range(len(st.hashes), full):
                toks = tuple(int(t) for t in token_ids[i * self.page_size:(i + 1) * self.page_size])
                h = _chain_hash(prev, toks)
                p = st.pages[i]
                st.hashes.append(h)
                prev = h
                if p in self._borrowed or h in self._prefix:
                    continue
                self._prefix[h] = p
                self._page_key[p] = (h, toks)

    def fork(self, src_id, dst_id) -> None:
        """dst shares all of src's pages (copy-on-write on the next append)."""
        with self._lock:
            src = self._seqs[src_id]
            if dst_id in self._seqs:
                raise KeyError(f"sequence {dst_id!r} exists")
            for p in src.pages:
                self._incref(p)
            self._seqs[dst_id] = SeqState(list(src.pages), src.num_tokens, src.cached_tokens, list(src.hashes))

    def free(self, seq_id) -> None:
        with self._lock:
            st = self._seqs.pop(seq_id, None)
            if st is None:
                return
            for p in st.pages:
                self._decref(p)

    def truncate(self, seq_id, num_tokens: int) -> None:
        """Drops tokens past num_tokens (rejected speculative tokens)."""
        with self._lock:
            st = self._seqs[seq_id]
            if num_tokens >= st.num_tokens:
                return
            keep = self.pages_needed(num_tokens)
            for p in st.pages[keep:]:
                self._decref(p)
            del st.pages[keep:]
            st.hashes = st.hashes[: num_tokens // self.page_size]
            st.num_tokens = num_tokens

    # ------------------------------------------------------------------ queries
    def block_table(self, seq_id) -> List[int]:
        return list(self._seqs[seq_id].pages)

    def seq_len(self, seq_id) -> int:
        return self._seqs[seq_id].num_tokens

    def has(self, seq_id) -> bool:
        return seq_id in self._seqs

    def sequences(self) -> List[object]:
        return list(self._seqs)

    def reset_prefix_cache(self) -> None:
        with self._lock:
            for p in list(self._lru):
                self._free.append(p)
            self._lru.clear()
            self._prefix.clear()
            self._page_key.clear()

    def stats(self) -> Dict[str, float]:
        with self._lock:
            used = self.num_pages - len(self._free) - len(self._lru)
            d = dict(self.stats_counters)
            d.update(total_pages=self.num_pages, used_pages=used, free_pages=len(self._free),
                     cached_pages=len(self._lru), sequences=len(self._seqs),
                     utilization=used / max(1, self.num_pages), borrowed_live=len(self._borrowed))
            q = max(1, d["prefix_queries"])
            d["prefix_hit_rate"] = d["prefix_hits"] / q
            return d
