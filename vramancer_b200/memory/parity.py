"""XOR parity groups over equal-size blocks (N data + 1 parity): any one lost block of
a group is rebuilt from the others.  Hashing / XOR run in the C++ runtime.

Reference parity: core/parity_memory.py:56-218 (ParityKVManager.encode / heal /
store_engram / heal_engram / stats, single-fault XOR over evicted KV pages).
"""
from __future__ import annotations

import threading
from typing import Dict, List, Optional, Sequence

import torch

from .. import runtime as rt


def _as_bytes(x) -> bytes:
    if isinstance(x, torch.Tensor):
        return x.detach().to("cpu").contiguous().view(torch.uint8).numpy().tobytes()
    return bytes(x)


class ParityKVManager:
    def __init__(self, group_size: int = 4):
        if group_size < 2:
            raise ValueError("a parity group needs at least 2 data blocks")
        self.group_size = group_size
        self._groups: Dict[str, dict] = {}
        self._lock = threading.Lock()
        self.encoded = 0
        self.healed = 0

    def encode(self, group_id: str, blocks: Sequence) -> bytes:
        """Stores the parity of `blocks` (bytes-like or tensors, equal sizes) and a
        checksum of each block; returns the parity."""
        data = [_as_bytes(b) for b in blocks]
        if not data or len({len(d) for d in data}) != 1:
            raise ValueError("parity: blocks must be non-empty and of equal size")
        parity = bytes(rt.xor_parity(data))
        with self._lock:
            self._groups[group_id] = {"parity": parity, "n": len(data), "size": len(data[0]),
                                      "sums": [rt.sha256(d) for d in data]}
            self.encoded += 1
        return parity

    def verify(self, group_id: str, idx: int, block) -> bool:
        g = self._groups[group_id]
        return rt.sha256(_as_bytes(block)) == g["sums"][idx]

    def heal(self, group_id: str, missing_idx: int, available: Sequence[Optional[object]]) -> bytes:
        """Rebuilds block `missing_idx` from the group's other blocks (`available`,
        indexed like the original group; the missing entry may be None) and the
        stored parity; the result is checked against the stored checksum."""
        g = self._groups.get(group_id)
        if g is None:
            raise KeyError(f"no parity group {group_id!r}")
        others = [_as_bytes(b) for i, b in enumerate(available) if i != missing_idx]
        if len(others) != g["n"] - 1:
            raise ValueError("heal: need every other block of the group")
        out = bytes(rt.xor_parity(others + [g["parity"]]))
        if rt.sha256(out) != g["sums"][missing_idx]:
            raise RuntimeError(f"heal: rebuilt block {missing_idx} of {group_id!r} fails its checksum")
        self.healed += 1
        return out

    # reference naming: an "engram" is one parity-protected group
    def store_engram(self, engram_id: str, blocks: Sequence) -> bytes:
        return self.encode(engram_id, blocks)

    def heal_engram(self, engram_id: str, missing_idx: int, available: Sequence) -> Optional[bytes]:
        try:
            return self.heal(engram_id, missing_idx, available)
        except (KeyError, RuntimeError, ValueError):
            return None

    def drop(self, group_id: str) -> None:
        with self._lock:
            self._groups.pop(group_id, None)

    def stats(self) -> Dict[str, int]:
        return {"groups": len(self._groups), "encoded": self.encoded, "healed": self.healed,
                "parity_bytes": sum(len(g["parity"]) for g in self._groups.values())}
