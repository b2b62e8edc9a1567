"""Hierarchical block store: tensors move between memory tiers by heat and budget.

Tiers (lower number = faster):
  L1  VRAM of the owning GPU          (resident tensor)
  L2  VRAM of a peer GPU              (NVLink peer copy, torch on a copy stream)
  L3  remote node RAM                 (signed TCP tensor frames to a BlockServer)
  L4  pinned host DRAM                (page-locked copy, async H2D on the way back)
  L5  local NVMe / SSD                (C++ pwrite / pread spill, raw bytes)
  L6  network / shared filesystem     (same spill, a different directory)
  L7  compressed archive              (zlib / zstd of the raw bytes, on disk)

Every block has a heat score: +1 per access, decayed by exp(-dt / tau).  Blocks
above `promote_heat` move one tier up on access; `eviction_cycle` demotes the
coldest unpinned L1 blocks until the VRAM budget has the requested free share.
Spilled blocks of equal size can be grouped under XOR parity (ParityKVManager) so
one lost file is rebuilt.  State (registry, tiers, paths) saves to / loads from JSON.

Reference parity: experimental/hierarchical_memory.py:376-1010
(HierarchicalMemoryManager: register_block, get_tier, migrate, touch,
promote_policy, spill_to_nvme, load_from_nvme, policy_demote_if_needed,
update_all_scores, eviction_cycle, summary, save_state, load_state,
schedule_prefetch) with L1..L7 tiers; its L3 (RDMA) has no B200-box equivalent and is
served by the TCP block server here.
"""
from __future__ import annotations

import json
import math
import os
import threading
import time
from dataclasses import dataclass, field
from enum import IntEnum
from typing import Any, Dict, Iterable, List, Optional

import torch

from .. import runtime as rt
from .compressor import Compressor
from .parity import ParityKVManager


class Tier(IntEnum):
    L1 = 1
    L2 = 2
    L3 = 3
    L4 = 4
    L5 = 5
    L6 = 6
    L7 = 7


TIER_NAMES = {Tier.L1: "vram", Tier.L2: "peer_vram", Tier.L3: "remote_ram", Tier.L4: "pinned_dram",
              Tier.L5: "nvme", Tier.L6: "network_disk", Tier.L7: "archive"}

_DT = {str(d): d for d in (torch.float32, torch.float16, torch.bfloat16, torch.int64, torch.int32, torch.int16,
                           torch.int8, torch.uint8, torch.bool, torch.float64)}


@dataclass
class MemoryBlock:
    id: str
    shape: tuple
    dtype: torch.dtype
    home_device: str = "cpu"          # the device the block is consumed on
    pinned: bool = False              # never evicted from L1
    heat: float = 0.0
    last_access: float = field(default_factory=time.time)
    tier: Optional[Tier] = None
    meta: dict = field(default_factory=dict)

    @property
    def nbytes(self) -> int:
        return int(torch.Size(self.shape).numel()) * torch.empty((), dtype=self.dtype).element_size()


class HierarchicalMemoryManager:
    def __init__(self, nvme_dir: str = ".hm_cache", max_nvme_mb: int = 2048, *,
                 vram_budget_bytes: Optional[int] = None, dram_budget_bytes: int = 16 << 30,
                 peer_device: Optional[str] = None, network_dir: Optional[str] = None,
                 remote: Optional[tuple] = None, remote_key: bytes = b"", tau_s: float = 60.0,
                 promote_heat: float = 3.0, codec: str = "auto", parity_group: int = 0, io_workers: int = 4):
        self.nvme_dir = nvme_dir
        self.network_dir = network_dir or os.path.join(nvme_dir, "net")
        self.archive_dir = os.path.join(nvme_dir, "archive")
        for d in (self.nvme_dir, self.network_dir, self.archive_dir):
            os.makedirs(d, exist_ok=True)
        self.max_nvme_bytes = max_nvme_mb << 20
        self.vram_budget = vram_budget_bytes
        self.dram_budget = dram_budget_bytes
        self.peer_device = peer_device
        self.remote, self.remote_key = remote, remote_key
        self.tau, self.promote_heat = tau_s, promote_heat
        self.compressor = Compressor(codec)
        self.parity = ParityKVManager(parity_group) if parity_group >= 2 else None
        self._pending_parity: List[str] = []
        self.blocks: Dict[str, MemoryBlock] = {}
        self._data: Dict[str, Any] = {}          # tier payload: tensor, path or archive path
        self._lock = threading.RLock()
        self._io = rt.AsyncFileIO(io_workers)
        self._prefetch: Dict[str, tuple] = {}
        self.stats = {"migrations": 0, "promotions": 0, "demotions": 0, "spilled_bytes": 0, "loaded_bytes": 0,
                      "evictions": 0, "healed": 0}

    # ---------------------------------------------------------------- registry
    def register_block(self, block: MemoryBlock, tier: Tier, tensor: Optional[torch.Tensor] = None) -> MemoryBlock:
        with self._lock:
            if tensor is not None:
                block.shape, block.dtype = tuple(tensor.shape), tensor.dtype
                self._data[block.id] = self._place(block, tensor, Tier(tier))
            block.tier = Tier(tier)
            self.blocks[block.id] = block
            return block

    def get_tier(self, block_id: str) -> Optional[Tier]:
        b = self.blocks.get(block_id)
        return b.tier if b else None

    def remove(self, block_id: str) -> None:
        with self._lock:
            b = self.blocks.pop(block_id, None)
            payload = self._data.pop(block_id, None)
            if b is not None and b.tier in (Tier.L5, Tier.L6, Tier.L7) and isinstance(payload, str):
                try:
                    os.unlink(payload)
                except OSError:
                    pass

    # ---------------------------------------------------------------- physical moves
    def _path(self, block: MemoryBlock, tier: Tier) -> str:
        d = {Tier.L5: self.nvme_dir, Tier.L6: self.network_dir, Tier.L7: self.archive_dir}[tier]
        return os.path.join(d, block.id.replace("/", "_") + (".z" if tier == Tier.L7 else ".bin"))

    def _place(self, block: MemoryBlock, t: torch.Tensor, tier: Tier):
        """Stores tensor `t` in `tier`; returns the tier payload."""
        if tier == Tier.L1:
            return t.to(block.home_device, non_blocking=True)
        if tier == Tier.L2:
            if self.peer_device is None:
                raise RuntimeError("L2 needs a peer_device")
            return t.to(self.peer_device, non_blocking=True)
        if tier == Tier.L4:
            h = torch.empty(t.shape, dtype=t.dtype, pin_memory=torch.cuda.is_available())
            h.copy_(t)
            return h
        if tier in (Tier.L5, Tier.L6):
            path = self._path(block, tier)
            n = rt.dump_tensor(path, t)
            self.stats["spilled_bytes"] += n
            return path
        if tier == Tier.L7:
            path = self._path(block, tier)
            d = self.compressor.compress_tensor(t)
            with open(path, "wb") as f:
                f.write(d["data"])
            self.stats["spilled_bytes"] += len(d["data"])
            return path
        if tier == Tier.L3:
            if self.remote is None:
                raise RuntimeError("L3 needs a remote (host, port) block server")
            conn = rt.connect(*self.remote)
            try:
                rt.send_tensors(conn, {"t": t}, {"op": "put", "id": block.id}, key=self.remote_key)
                rt.recv_tensors(conn, key=self.remote_key)
            finally:
                conn.close()
            return ("remote", block.id)
        raise ValueError(f"unknown tier {tier}")

    def _fetch(self, block: MemoryBlock) -> torch.Tensor:
        """The block's tensor, materialised on the host or its current device."""
        payload = self._data[block.id]
        tier = block.tier
        if tier in (Tier.L1, Tier.L2, Tier.L4):
            return payload
        if tier in (Tier.L5, Tier.L6):
            out = torch.empty(block.shape, dtype=block.dtype, pin_memory=torch.cuda.is_available())
            rt.load_tensor(payload, out)
            self.stats["loaded_bytes"] += block.nbytes
            return out
        if tier == Tier.L7:
            with open(payload, "rb") as f:
                data = f.read()
            return self.compressor.decompress_tensor({"codec": self.compressor.codec, "dtype": str(block.dtype),
                                                      "shape": list(block.shape), "data": data})
        if tier == Tier.L3:
            conn = rt.connect(*self.remote)
            try:
                rt.send_tensors(conn, {}, {"op": "get", "id": block.id}, key=self.remote_key)
                got, _ = rt.recv_tensors(conn, key=self.remote_key)
            finally:
                conn.close()
            return got["t"]
        raise ValueError(f"block {block.id} has no tier")

    def migrate(self, block: MemoryBlock, target: Tier, tensor: Optional[torch.Tensor] = None) -> Any:
        """Moves `block` to `target` (optionally from the caller's fresh `tensor`);
        returns the new payload (a tensor for L1/L2/L4, a path for disk tiers)."""
        target = Tier(target)
        with self._lock:
            prev = block.tier
            if prev == target and tensor is None:
                return self._data.get(block.id)
            src = tensor if tensor is not None else self._fetch(block)
            old = self._data.get(block.id)
            new = self._place(block, src, target)
            self._data[block.id] = new
            block.tier = target
            if prev in (Tier.L5, Tier.L6, Tier.L7) and isinstance(old, str) and old != new:
                try:
                    os.unlink(old)
                except OSError:
                    pass
            self.stats["migrations"] += 1
            if prev is not None and target < prev:
                self.stats["promotions"] += 1
            elif prev is not None and target > prev:
                self.stats["demotions"] += 1
            if self.parity is not None and target in (Tier.L5, Tier.L6):
                self._pending_parity.append(block.id)
                self._maybe_encode_parity()
            return new

    def get(self, block_id: str, device: Optional[str] = None) -> torch.Tensor:
        """The block's tensor on `device` (default: its home device); counts as an access."""
        b = self.blocks[block_id]
        self.touch(b)
        with self._lock:
            t = self._fetch(b)
        return t.to(device or b.home_device, non_blocking=True)

    # ---------------------------------------------------------------- heat and policy
    def _decayed(self, b: MemoryBlock, now: float) -> float:
        return b.heat * math.exp(-(now - b.last_access) / self.tau)

    def touch(self, block: MemoryBlock) -> None:
        now = time.time()
        block.heat = self._decayed(block, now) + 1.0
        block.last_access = now
        self.promote_policy(block)

    def promote_policy(self, block: MemoryBlock) -> None:
        if block.tier is not None and block.tier > Tier.L1 and block.heat >= self.promote_heat:
            up = Tier.L1 if block.tier in (Tier.L2, Tier.L4) else Tier.L4
            self.migrate(block, up)

    def policy_demote_if_needed(self, block: MemoryBlock, gpu_over_pct: float) -> None:
        if block.tier == Tier.L1 and not block.pinned and gpu_over_pct > 0:
            self.migrate(block, Tier.L2 if self.peer_device else Tier.L4)

    def update_all_scores(self, current_time: Optional[float] = None) -> None:
        now = current_time or time.time()
        for b in self.blocks.values():
            b.heat = self._decayed(b, now)
            b.last_access = now

    def tier_bytes(self, tier: Tier) -> int:
        return sum(b.nbytes for b in self.blocks.values() if b.tier == tier)

    def eviction_cycle(self, target_free_pct: float = 10.0, vram_pressure: Optional[float] = None) -> int:
        """Demotes cold L1 blocks (then cold L4 blocks to NVMe, and NVMe overflow to
        the archive) until every tier is within budget; returns blocks moved."""
        moved = 0
        now = time.time()
        with self._lock:
            if self.vram_budget is not None:
                limit = self.vram_budget * (1 - target_free_pct / 100.0)
                if vram_pressure is not None:
                    limit *= max(0.0, 1.0 - vram_pressure)
                for b in sorted((b for b in self.blocks.values() if b.tier == Tier.L1 and not b.pinned),
                                key=lambda b: self._decayed(b, now)):
                    if self.tier_bytes(Tier.L1) <= limit:
                        break
                    self.migrate(b, Tier.L2 if self.peer_device else Tier.L4)
                    moved += 1
            for b in sorted((b for b in self.blocks.values() if b.tier == Tier.L4), key=lambda b: self._decayed(b, now)):
                if self.tier_bytes(Tier.L4) <= self.dram_budget:
                    break
                self.migrate(b, Tier.L5)
                moved += 1
            for b in sorted((b for b in self.blocks.values() if b.tier == Tier.L5), key=lambda b: self._decayed(b, now)):
                if self.tier_bytes(Tier.L5) <= self.max_nvme_bytes:
                    break
                self.migrate(b, Tier.L7)
                moved += 1
        self.stats["evictions"] += moved
        return moved

    # ---------------------------------------------------------------- NVMe helpers (reference names)
    def spill_to_nvme(self, block: MemoryBlock, payload: Optional[torch.Tensor] = None) -> str:
        return self.migrate(block, Tier.L5, payload)

    def load_from_nvme(self, block: MemoryBlock) -> Optional[torch.Tensor]:
        if block.tier != Tier.L5:
            return None
        with self._lock:
            return self._fetch(block)

    # ---------------------------------------------------------------- prefetch
    def schedule_prefetch(self, block_ids: Iterable[str], target_tier: Tier = Tier.L4) -> int:
        """Starts background reads of NVMe / network-disk blocks into pinned buffers;
        `complete_prefetch` installs them in `target_tier`.  Returns reads started."""
        n = 0
        with self._lock:
            for bid in block_ids:
                b = self.blocks.get(bid)
                if b is None or b.tier not in (Tier.L5, Tier.L6) or bid in self._prefetch:
                    continue
                buf = torch.empty(b.shape, dtype=b.dtype, pin_memory=torch.cuda.is_available())
                ticket = self._io.read(self._data[bid], buf.view(-1).view(torch.uint8) if b.nbytes else buf)
                self._prefetch[bid] = (ticket, buf, Tier(target_tier))
                n += 1
        return n

    def complete_prefetch(self) -> int:
        done = 0
        with self._lock:
            for bid, (ticket, buf, target) in list(self._prefetch.items()):
                self._io.wait(ticket)
                del self._prefetch[bid]
                b = self.blocks.get(bid)
                if b is not None:
                    self.stats["loaded_bytes"] += b.nbytes
                    self.migrate(b, target, buf)
                    done += 1
        return done

    # ---------------------------------------------------------------- parity
    def _maybe_encode_parity(self) -> None:
        sizes: Dict[int, List[str]] = {}
        for bid in self._pending_parity:
            b = self.blocks.get(bid)
            if b is not None:
                sizes.setdefault(b.nbytes, []).append(bid)
        for nbytes, ids in sizes.items():
            while len(ids) >= self.parity.group_size:
                group, ids[:] = ids[:self.parity.group_size], ids[self.parity.group_size:]
                gid = "+".join(group)
                self.parity.encode(gid, [self._fetch(self.blocks[i]) for i in group])
                for i in group:
                    self.blocks[i].meta["parity_group"] = gid
                    self._pending_parity.remove(i)

    def heal(self, block_id: str) -> bool:
        """Rebuilds a spilled block whose file was lost, from its parity group."""
        b = self.blocks[block_id]
        gid = b.meta.get("parity_group")
        if gid is None or self.parity is None:
            return False
        ids = gid.split("+")
        idx = ids.index(block_id)
        others = [None if i == block_id else self._fetch(self.blocks[i]) for i in ids]
        data = self.parity.heal(gid, idx, others)
        t = torch.frombuffer(bytearray(data), dtype=torch.uint8).view(b.dtype).reshape(b.shape).clone()
        with self._lock:
            self._data[block_id] = self._place(b, t, b.tier)
        self.stats["healed"] += 1
        return True

    # ---------------------------------------------------------------- state
    def summary(self) -> Dict[str, Any]:
        per = {TIER_NAMES[t]: {"blocks": sum(1 for b in self.blocks.values() if b.tier == t),
                               "bytes": self.tier_bytes(t)} for t in Tier}
        return {"tiers": per, "blocks": len(self.blocks), **self.stats,
                "compression_ratio": self.compressor.ratio,
                "parity": self.parity.stats() if self.parity else None}

    def save_state(self, path: str = ".hm_state.json") -> None:
        """Registry of the disk-resident blocks (tiers L5-L7) with their files."""
        with self._lock:
            rows = [{"id": b.id, "shape": list(b.shape), "dtype": str(b.dtype), "home": b.home_device,
                     "tier": int(b.tier), "heat": b.heat, "path": self._data[b.id], "meta": b.meta}
                    for b in self.blocks.values() if b.tier in (Tier.L5, Tier.L6, Tier.L7)]
        with open(path, "w") as f:
            json.dump({"codec": self.compressor.codec, "blocks": rows}, f)

    def load_state(self, path: str = ".hm_state.json") -> int:
        with open(path) as f:
            st = json.load(f)
        n = 0
        with self._lock:
            for r in st["blocks"]:
                if not os.path.exists(r["path"]):
                    continue
                b = MemoryBlock(r["id"], tuple(r["shape"]), _DT[r["dtype"]], r["home"], heat=r["heat"],
                                tier=Tier(r["tier"]), meta=r.get("meta", {}))
                self.blocks[b.id] = b
                self._data[b.id] = r["path"]
                n += 1
        return n


class BlockServer:
    """Remote-RAM tier (L3) on another node: keeps put tensors in host memory and
    returns them on get, over signed TCP tensor frames."""

    def __init__(self, host: str = "127.0.0.1", port: int = 0, key: bytes = b""):
        self.listener = rt.listen(host, port)
        self.key = key
        self.store: Dict[str, torch.Tensor] = {}
        self._stop = threading.Event()
        self._thread = threading.Thread(target=self._serve, daemon=True)
        self._thread.start()

    @property
    def address(self) -> tuple:
        return ("127.0.0.1", self.listener.port)

    def _serve(self) -> None:
        while not self._stop.is_set():
            conn = self.listener.accept(0.2)
            if conn is None:
                continue
            try:
                tensors, meta = rt.recv_tensors(conn, key=self.key)
                if meta.get("op") == "put":
                    self.store[meta["id"]] = tensors["t"]
                    rt.send_tensors(conn, {}, {"ok": True}, key=self.key)
                else:
                    rt.send_tensors(conn, {"t": self.store[meta["id"]]}, {"ok": True}, key=self.key)
            except Exception:  # noqa: BLE001 - a bad client must not stop the server
                pass
            finally:
                conn.close()

    def close(self) -> None:
        self._stop.set()
        self._thread.join(2)
        self.listener.close()
