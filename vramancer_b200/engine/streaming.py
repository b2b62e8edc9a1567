"""Layer weight streaming: run a model whose layer weights do not all fit in VRAM.

`StreamManager` keeps every layer's weights in pinned host memory and a bounded set of
layers resident on the GPU.  `prefetch_layers(current, lookahead)` starts host-to-device
copies of the next layers on a dedicated copy stream (an event per layer); `acquire`
makes the compute stream wait for a layer's event; layers past the budget are released
lowest priority first (`swap_if_needed`).  `StreamedDecoderModel` runs decode / prefill
with the manager: while layer i computes, layers i+1..i+lookahead are in flight, so the
PCIe / C2C copy overlaps the GEMMs.  Eager mode only (weights move every step, so the
step is not graph-capturable).

Reference parity: core/stream_manager.py:38-400 (StreamManager: preload_layer,
release_layer, prefetch_layers, unload_unused, swap_if_needed, start_monitoring,
stop_monitoring, stats).
"""
from __future__ import annotations

import threading
import time
from typing import Dict, List, Optional, Sequence

import torch

from ..models.transformer import DecoderModel


class StreamManager:
    def __init__(self, layers: Dict[int, Dict[str, torch.Tensor]], device, budget_layers: int = 4,
                 lookahead: int = 2):
        """layers: {layer index: {weight name: tensor}} (moved to pinned host memory)."""
        self.device = torch.device(device)
        pin = self.device.type == "cuda"
        self.host = {i: {k: (v.detach().cpu().pin_memory() if pin else v.detach().cpu()) for k, v in ws.items()}
                     for i, ws in layers.items()}
        self.budget = max(1, budget_layers)
        self.lookahead = lookahead
        self.resident: Dict[int, Dict[str, torch.Tensor]] = {}
        self.events: Dict[int, Optional[torch.cuda.Event]] = {}
        self.priority: Dict[int, float] = {}
        self.copy_stream = torch.cuda.Stream(device=self.device) if pin else None
        self._lock = threading.RLock()
        self._monitor: Optional[threading.Thread] = None
        self._stop = threading.Event()
        self.counters = {"loads": 0, "evictions": 0, "hits": 0, "bytes": 0}

    # ---------------------------------------------------------------- residency
    def preload_layer(self, idx: int) -> bool:
        """Starts copying layer `idx` to the device; False when it already is there."""
        with self._lock:
            if idx in self.resident or idx not in self.host:
                return False
            self._make_room(keep={idx})
            ws = {}
            if self.copy_stream is not None:
                with torch.cuda.stream(self.copy_stream):
                    for k, v in self.host[idx].items():
                        ws[k] = v.to(self.device, non_blocking=True)
                ev = torch.cuda.Event()
                ev.record(self.copy_stream)
            else:
                ws = {k: v.to(self.device) for k, v in self.host[idx].items()}
                ev = None
            self.resident[idx] = ws
            self.events[idx] = ev
            self.counters["loads"] += 1
            self.counters["bytes"] += sum(v.numel() * v.element_size() for v in ws.values())
            return True

    def acquire(self, idx: int) -> Dict[str, torch.Tensor]:
        """The device weights of layer `idx`, ordered after their copy on the current stream."""
        with self._lock:
            if idx in self.resident:
                self.counters["hits"] += 1
            else:
                self.preload_layer(idx)
            ev = self.events.get(idx)
            ws = self.resident[idx]
            self.priority[idx] = time.monotonic()
        if ev is not None:
            cur = torch.cuda.current_stream(self.device)
            cur.wait_event(ev)
            for v in ws.values():
                v.record_stream(cur)
        return ws

    def release_layer(self, idx: int) -> bool:
        with self._lock:
            if self.resident.pop(idx, None) is None:
                return False
            self.events.pop(idx, None)
            self.priority.pop(idx, None)
            self.counters["evictions"] += 1
            return True

    def _make_room(self, keep=()) -> None:
        while len(self.resident) >= self.budget:
            cands = [i for i in self.resident if i not in keep]
            if not cands:
                return
            self.release_layer(min(cands, key=lambda i: self.priority.get(i, 0.0)))

    def prefetch_layers(self, current_layers: Sequence[int], lookahead: Optional[int] = None) -> int:
        n = len(self.host)
        la = self.lookahead if lookahead is None else lookahead
        last = max(current_layers) if current_layers else -1
        started = 0
        for k in range(1, la + 1):
            nxt = (last + k) % n
            if nxt not in self.resident:
                started += int(self.preload_layer(nxt))
        return started

    def unload_unused(self, active: Sequence[int]) -> int:
        with self._lock:
            drop = [i for i in list(self.resident) if i not in set(active)]
            for i in drop:
                self.release_layer(i)
            return len(drop)

    def swap_if_needed(self, max_util: float = 0.90) -> bool:
        """Releases the least recently used layer when the device is over `max_util`."""
        if self.device.type != "cuda":
            return False
        free, total = torch.cuda.mem_get_info(self.device)
        if 1 - free / total <= max_util or not self.resident:
            return False
        with self._lock:
            victim = min(self.resident, key=lambda i: self.priority.get(i, 0.0))
            return self.release_layer(victim)

    # ---------------------------------------------------------------- monitor
    def start_monitoring(self, interval: float = 1.0, max_util: float = 0.90) -> None:
        if self._monitor is not None:
            return
        self._stop.clear()

        def loop():
            while not self._stop.wait(interval):
                self.swap_if_needed(max_util)

        self._monitor = threading.Thread(target=loop, daemon=True)
        self._monitor.start()

    def stop_monitoring(self) -> None:
        self._stop.set()
        if self._monitor is not None:
            self._monitor.join(2)
        self._monitor = None

    def stats(self) -> Dict[str, int]:
        return dict(self.counters, resident=len(self.resident), layers=len(self.host))


class StreamedDecoderModel(DecoderModel):
    """DecoderModel whose layer weights stream from pinned host memory (StreamManager);
    embeddings, final norm and lm_head stay resident."""

    def __init__(self, cfg, weights, *, budget_layers: int = 4, lookahead: int = 2, **kw):
        layer_w: Dict[int, Dict[str, torch.Tensor]] = {}
        resident = {}
        for k, v in weights.items():
            # norm weights are tiny and read across layer boundaries (the next layer's
            # input norm is fused into this layer's last projection): keep them resident
            if k.startswith("layers.") and "norm" not in k:
                _, i, name = k.split(".", 2)
                layer_w.setdefault(int(i), {})[name] = v
            else:
                resident[k] = v
        dev = kw.get("device", "cpu")
        resident = {k: v.to(dev) for k, v in resident.items()}
        super().__init__(cfg, resident, **kw)
        self.streamer = StreamManager(layer_w, self.device, budget_layers=budget_layers, lookahead=lookahead)

    def layer(self, i, r, batch, pool, x=None):
        ws = self.streamer.acquire(i)
        for name, v in ws.items():
            self.w[f"layers.{i}.{name}"] = v
        self.streamer.prefetch_layers([i])
        try:
            return super().layer(i, r, batch, pool, x)
        finally:
            for name in ws:
                self.w.pop(f"layers.{i}.{name}", None)
