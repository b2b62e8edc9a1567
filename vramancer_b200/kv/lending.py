"""VRAM lending pool: GPUs with spare memory lend it to GPUs that run out.

Bookkeeping (budgets, leases, policy) is host-side; data moves with the P2P page
copy kernel over NVLink (kv/migration.py), never through host memory.

* `GPUBudget` — total / model / KV / lent / borrowed / reserved (10%) bytes.
* `LendingPolicy` — lend at most 70% of free memory, stop lending above 75%
  utilisation, reclaim at 80%, critical at 95% or 82 C.
* `VRAMLendingPool.borrow(borrower, nbytes)` picks a lender by score
  (capacity 0.4 + link bandwidth 0.3 + idleness 0.3), carves the lease out of the
  lender's pre-allocated lending buffer (bump allocator), and returns a `VRAMLease`;
  `allocate_on_lease` gives a tensor view in that memory; `transfer_into_lease` /
  `transfer_from_lease` copy data in and out; `reclaim(lender, urgency)` migrates
  leases back to their borrower (graceful) or drops them (forced), firing callbacks
  so owners can react; `release` returns the memory.
* `KVPageLender` lends whole KV pages between the per-GPU paged pools: a borrower
  swaps cold sequences out to a lender's pool and back in on demand.
* `suggest_placement_budget` turns budgets into a per-GPU `max_memory` map.

Reference parity: experimental/vram_lending.py:78-1383 (LeaseState/ReclaimUrgency
78-92, VRAMLease 95, GPUBudget 120, LendingPolicy 171, borrow 389-475, _select_lender
477-549, allocate_on_lease 573-637, transfer_into/from_lease 781-878, reclaim
884-1024, release 1054, monitor 1075-1131, suggest_placement_budget 1231-1317).
"""
from __future__ import annotations

import enum
import itertools
import threading
import time
from dataclasses import dataclass, field
from typing import Callable, Dict, List, Optional, Sequence, Tuple

import torch

from ..utils.observability import METRICS, get_logger

log = get_logger("vramancer.lending")


class LeaseState(str, enum.Enum):
    ACTIVE = "active"
    RECLAIMING = "reclaiming"
    RELEASED = "released"


class ReclaimUrgency(str, enum.Enum):
    LOW = "low"            # graceful, when convenient
    HIGH = "high"          # graceful now
    CRITICAL = "critical"  # drop without copying


@dataclass
class VRAMLease:
    lease_id: int
    lender: int
    borrower: int
    nbytes: int
    purpose: str = ""
    offset: int = 0
    created: float = field(default_factory=time.time)
    state: LeaseState = LeaseState.ACTIVE
    tensor: Optional[torch.Tensor] = None
    on_reclaim: Optional[Callable[["VRAMLease", ReclaimUrgency], None]] = None


@dataclass
class GPUBudget:
    device: int
    total: int
    model_bytes: int = 0
    kv_bytes: int = 0
    lent: int = 0
    borrowed: int = 0
    reserved_ratio: float = 0.10
    link_gbs: float = 900.0
    utilization: float = 0.0      # compute utilisation 0..1 (monitor)
    temp_c: float = 0.0

    @property
    def reserved(self) -> int:
        return int(self.total * self.reserved_ratio)

    @property
    def used(self) -> int:
        return self.model_bytes + self.kv_bytes + self.lent

    @property
    def free(self) -> int:
        return max(0, self.total - self.reserved - self.used)

    @property
    def mem_util(self) -> float:
        return (self.used + self.reserved) / self.total if self.total else 1.0


@dataclass
class LendingPolicy:
    max_lend_ratio: float = 0.70
    stop_lending_util: float = 0.75
    reclaim_util: float = 0.80
    critical_util: float = 0.95
    thermal_c: float = 82.0
    cross_vendor_penalty: float = 0.5


class VRAMLendingPool:
    def __init__(self, policy: Optional[LendingPolicy] = None):
        self.policy = policy or LendingPolicy()
        self.budgets: Dict[int, GPUBudget] = {}
        self.buffers: Dict[int, torch.Tensor] = {}
        self._bump: Dict[int, List[Tuple[int, int]]] = {}      # free extents per lender (offset, size)
        self.leases: Dict[int, VRAMLease] = {}
        self._ids = itertools.count(1)
        self._lock = threading.RLock()
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self.sampler: Optional[Callable[[], Dict[int, Dict[str, float]]]] = None
        self.stats = {"borrows": 0, "denied": 0, "reclaims": 0, "bytes_borrowed": 0, "migrated_bytes": 0}

    # ------------------------------------------------------------------ registry
    def register_gpu(self, device: int, total_bytes: int, model_bytes: int = 0, kv_bytes: int = 0,
                     link_gbs: float = 900.0) -> GPUBudget:
        with self._lock:
            b = GPUBudget(device, total_bytes, model_bytes, kv_bytes, link_gbs=link_gbs)
            self.budgets[device] = b
            return b

    def preallocate(self, device: int, nbytes: int, tensor: Optional[torch.Tensor] = None) -> torch.Tensor:
        """Reserves a lending buffer on `device` (uint8); leases are carved from it."""
        with self._lock:
            if tensor is None:
                dev = torch.device("cuda", device) if torch.cuda.is_available() and device >= 0 else "cpu"
                tensor = torch.empty(nbytes, dtype=torch.uint8, device=dev)
            self.buffers[device] = tensor
            self._bump[device] = [(0, tensor.numel())]
            return tensor

    # ------------------------------------------------------------------ lender choice
    def lendable(self, device: int) -> int:
        b = self.budgets[device]
        if b.mem_util >= self.policy.stop_lending_util:
            return 0
        cap = int(self.policy.max_lend_ratio * (b.free + b.lent)) - b.lent
        if device in self._bump:
            cap = min(cap, max((s for _, s in self._bump[device]), default=0))
        return max(0, cap)

    def _score(self, lender: GPUBudget, nbytes: int) -> float:
        cap = self.lendable(lender.device)
        if cap < nbytes:
            return -1.0
        capacity = min(1.0, cap / max(1, lender.total))
        link = min(1.0, lender.link_gbs / 900.0)
        idle = 1.0 - min(1.0, lender.utilization)
        return 0.4 * capacity + 0.3 * link + 0.3 * idle

    def select_lender(self, borrower: int, nbytes: int) -> Optional[int]:
        best, best_s = None, 0.0
        for d, b in self.budgets.items():
            if d == borrower or b.temp_c >= self.policy.thermal_c:
                continue
            s = self._score(b, nbytes)
            if s > best_s:
                best, best_s = d, s
        return best

    def _carve(self, lender: int, nbytes: int, align: int = 256) -> Optional[int]:
        ext = self._bump.get(lender)
        if ext is None:
            return 0
        need = (nbytes + align - 1) // align * align
        for i, (off, size) in enumerate(ext):
            a = (off + align - 1) // align * align
            pad = a - off
            if size - pad >= need:
                rest = (a + need, off + size - (a + need))
                ext[i:i + 1] = ([(off, pad)] if pad else []) + ([rest] if rest[1] > 0 else [])
                return a
        return None

    def _free_extent(self, lender: int, off: int, nbytes: int, align: int = 256) -> None:
        ext = self._bump.get(lender)
        if ext is None:
            return
        need = (nbytes + align - 1) // align * align
        ext.append((off, need))
        ext.sort()
        merged = []
        for o, s in ext:
            if merged and merged[-1][0] + merged[-1][1] == o:
                merged[-1] = (merged[-1][0], merged[-1][1] + s)
            else:
                merged.append((o, s))
        self._bump[lender] = merged

    # ------------------------------------------------------------------ leases
    def borrow(self, borrower: int, nbytes: int, purpose: str = "",
               on_reclaim: Optional[Callable[[VRAMLease, ReclaimUrgency], None]] = None) -> Optional[VRAMLease]:
        with self._lock:
            lender = self.select_lender(borrower, nbytes)
            if lender is None:
                self.stats["denied"] += 1
                return None
            off = self._carve(lender, nbytes)
            if off is None:
                self.stats["denied"] += 1
                return None
            lease = VRAMLease(next(self._ids), lender, borrower, nbytes, purpose, off, on_reclaim=on_reclaim)
            self.leases[lease.lease_id] = lease
            self.budgets[lender].lent += nbytes
            if borrower in self.budgets:
                self.budgets[borrower].borrowed += nbytes
            self.stats["borrows"] += 1
            self.stats["bytes_borrowed"] += nbytes
            METRICS.lending_leases.set(len(self.leases))
            METRICS.lending_bytes.set(sum(l.nbytes for l in self.leases.values()))
            return lease

    def allocate_on_lease(self, lease: VRAMLease, shape: Sequence[int], dtype=torch.bfloat16) -> torch.Tensor:
        buf = self.buffers.get(lease.lender)
        if buf is None:
            raise RuntimeError(f"lender {lease.lender} has no lending buffer")
        n = int(torch.Size(shape).numel()) * torch.empty(0, dtype=dtype).element_size()
        if n > lease.nbytes:
            raise ValueError("tensor larger than the lease")
        lease.tensor = buf[lease.offset:lease.offset + n].view(dtype).view(*shape)
        return lease.tensor

    def transfer_into_lease(self, lease: VRAMLease, src: torch.Tensor) -> torch.Tensor:
        if lease.tensor is None:
            self.allocate_on_lease(lease, src.shape, src.dtype)
        lease.tensor.copy_(src, non_blocking=True)
        self.stats["migrated_bytes"] += src.numel() * src.element_size()
        return lease.tensor

    def transfer_from_lease(self, lease: VRAMLease, device) -> torch.Tensor:
        if lease.tensor is None:
            raise RuntimeError("lease holds no tensor")
        out = lease.tensor.to(device, non_blocking=True)
        self.stats["migrated_bytes"] += out.numel() * out.element_size()
        return out

    def release(self, lease_id: int) -> None:
        with self._lock:
            lease = self.leases.pop(lease_id, None)
            if lease is None:
                return
            lease.state = LeaseState.RELEASED
            self.budgets[lease.lender].lent -= lease.nbytes
            if lease.borrower in self.budgets:
                self.budgets[lease.borrower].borrowed -= lease.nbytes
            self._free_extent(lease.lender, lease.offset, lease.nbytes)
            lease.tensor = None
            METRICS.lending_leases.set(len(self.leases))

    def reclaim(self, lender: int, urgency: ReclaimUrgency = ReclaimUrgency.HIGH) -> int:
        """Takes back every lease of `lender`.  Graceful urgencies let the owner copy
        its data out (callback) before release; CRITICAL drops immediately."""
        with self._lock:
            victims = [l for l in self.leases.values() if l.lender == lender]
        n = 0
        for l in victims:
            l.state = LeaseState.RECLAIMING
            if l.on_reclaim is not None:
                try:
                    l.on_reclaim(l, urgency)
                except Exception as e:
                    log.warning("reclaim callback failed for lease %d: %s", l.lease_id, e)
            self.release(l.lease_id)
            n += 1
        self.stats["reclaims"] += n
        METRICS.lending_reclaims.labels(urgency.value).inc(n)
        return n

    # ------------------------------------------------------------------ monitoring
    def check_pressure(self) -> Dict[int, ReclaimUrgency]:
        """Applies samples (mem utilisation, compute utilisation, temperature) and
        reclaims from lenders under pressure."""
        out = {}
        if self.sampler is not None:
            for d, s in self.sampler().items():
                if d in self.budgets:
                    b = self.budgets[d]
                    b.utilization = s.get("util", b.utilization)
                    b.temp_c = s.get("temp_c", b.temp_c)
                    if "kv_bytes" in s:
                        b.kv_bytes = int(s["kv_bytes"])
        for d, b in self.budgets.items():
            if b.lent <= 0:
                continue
            if b.mem_util >= self.policy.critical_util or b.temp_c >= self.policy.thermal_c:
                out[d] = ReclaimUrgency.CRITICAL
            elif b.mem_util >= self.policy.reclaim_util:
                out[d] = ReclaimUrgency.HIGH
        for d, u in out.items():
            self.reclaim(d, u)
        return out

    def start_monitor(self, interval_s: float = 1.0) -> None:
        if self._thread and self._thread.is_alive():
            return
        self._stop.clear()

        def loop():
            while not self._stop.wait(interval_s):
                try:
                    self.check_pressure()
                except Exception as e:
                    log.warning("lending monitor: %s", e)

        self._thread = threading.Thread(target=loop, name="vrm-lending-monitor", daemon=True)
        self._thread.start()

    def stop(self) -> None:
        self._stop.set()

    def suggest_placement_budget(self, headroom_gb: float = 2.0, cpu_spill_gb: float = 0.0) -> Dict[object, str]:
        out: Dict[object, str] = {}
        for d, b in self.budgets.items():
            gb = max(0.0, (b.total - b.reserved - b.lent) / 2 ** 30 - headroom_gb)
            out[d] = f"{int(gb)}GiB"
        if cpu_spill_gb:
            out["cpu"] = f"{int(cpu_spill_gb)}GiB"
        return out

    def summary(self) -> Dict[str, object]:
        with self._lock:
            return {"budgets": {d: {"total": b.total, "free": b.free, "lent": b.lent, "borrowed": b.borrowed,
                                    "mem_util": round(b.mem_util, 4)} for d, b in self.budgets.items()},
                    "leases": len(self.leases), **self.stats}


class KVPageLender:
    """Moves whole KV pages of sequences between per-GPU paged pools.

    swap_out(seq): allocate pages in the lender's pool, copy (P2P kernel), free the
    borrower's pages; swap_in(seq): the reverse.  The engines' block managers keep
    the page lists; this class only holds where each swapped sequence lives.
    """

    def __init__(self, local_pool, local_mgr, remote_pool, remote_mgr, method: str = "kernel"):
        self.local_pool, self.local_mgr = local_pool, local_mgr
        self.remote_pool, self.remote_mgr = remote_pool, remote_mgr
        self.method = method
        self.swapped: Dict[object, int] = {}

    def swap_out(self, seq_id) -> int:
        from .migration import migrate_pages
        n_tok = self.local_mgr.seq_len(seq_id)
        src = self.local_mgr.block_table(seq_id)
        rid = ("lent", seq_id)
        self.remote_mgr.allocate(rid, n_tok)
        dst = self.remote_mgr.block_table(rid)
        migrate_pages(self.local_pool.cache, self.remote_pool.cache, src, dst, method=self.method)
        self.local_mgr.free(seq_id)
        self.swapped[seq_id] = n_tok
        return len(src)

    def swap_in(self, seq_id) -> int:
        from .migration import migrate_pages
        n_tok = self.swapped.pop(seq_id)
        rid = ("lent", seq_id)
        src = self.remote_mgr.block_table(rid)
        self.local_mgr.allocate(seq_id, n_tok)
        dst = self.local_mgr.block_table(seq_id)
        migrate_pages(self.remote_pool.cache, self.local_pool.cache, src, dst, method=self.method)
        self.remote_mgr.free(rid)
        return len(src)
