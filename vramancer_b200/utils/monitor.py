"""GPU monitoring (NVML), hot-plug detection, health report and `doctor` diagnostics.

`GPUMonitor` samples memory, utilisation, temperature, power and clocks through NVML
(nvidia-ml-py) with a torch fallback; a polling thread keeps the latest sample and
`detect_overload` flags GPUs above a memory threshold.  `GPUHotPlugMonitor` reports
devices that appear or disappear between polls.  `health_report` and `doctor`
summarise the node for /health and the `vramancer doctor` command.  Nothing here
changes any GPU setting: NVML is used read-only.

Reference parity: core/monitor.py:95-622 (GPUMonitor, vram_usage, detect_overload,
GPUHotPlugMonitor), core/health.py:39-355, core/doctor.py:18-164.
"""
from __future__ import annotations

import os
import platform
import threading
import time
from typing import Callable, Dict, List, Optional

import torch

try:
    import pynvml  # nvidia-ml-py
except Exception:  # pragma: no cover
    pynvml = None


class NVML:
    """Minimal read-only NVML wrapper; `fake` lets tests inject a fake module."""

    def __init__(self, module=None):
        self.m = module if module is not None else pynvml
        self.ok = False
        if self.m is not None:
            try:
                self.m.nvmlInit()
                self.ok = True
            except Exception:
                self.ok = False

    def count(self) -> int:
        if not self.ok:
            return torch.cuda.device_count() if torch.cuda.is_available() else 0
        return int(self.m.nvmlDeviceGetCount())

    def sample(self, i: int) -> Dict[str, float]:
        if not self.ok:
            if torch.cuda.is_available():
                free, total = torch.cuda.mem_get_info(i)
                return {"index": i, "name": torch.cuda.get_device_name(i), "mem_used": total - free,
                        "mem_total": total, "util": -1.0, "temp_c": -1.0, "power_w": -1.0, "sm_mhz": -1.0}
            return {"index": i, "name": "none", "mem_used": 0, "mem_total": 0, "util": -1, "temp_c": -1,
                    "power_w": -1, "sm_mhz": -1}
        m = self.m
        h = m.nvmlDeviceGetHandleByIndex(i)
        mem = m.nvmlDeviceGetMemoryInfo(h)
        name = m.nvmlDeviceGetName(h)
        name = name.decode() if isinstance(name, bytes) else name
        d = {"index": i, "name": name, "mem_used": float(mem.used), "mem_total": float(mem.total)}
        for key, fn in (("util", lambda: m.nvmlDeviceGetUtilizationRates(h).gpu),
                        ("temp_c", lambda: m.nvmlDeviceGetTemperature(h, 0)),
                        ("power_w", lambda: m.nvmlDeviceGetPowerUsage(h) / 1000.0),
                        ("sm_mhz", lambda: m.nvmlDeviceGetClockInfo(h, 1))):
            try:
                d[key] = float(fn())
            except Exception:
                d[key] = -1.0
        return d


class GPUMonitor:
    def __init__(self, interval_s: float = 1.0, nvml: Optional[NVML] = None, overload_threshold: float = 0.95):
        self.nvml = nvml or NVML()
        self.interval = interval_s
        self.threshold = overload_threshold
        self.latest: List[Dict[str, float]] = []
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None
        self.callbacks: List[Callable[[List[Dict[str, float]]], None]] = []

    def poll(self) -> List[Dict[str, float]]:
        self.latest = [self.nvml.sample(i) for i in range(self.nvml.count())]
        from . import observability as obs
        for d in self.latest:
            g = str(int(d["index"]))
            obs.METRICS.gpu_mem_used.labels(g).set(d["mem_used"])
            obs.METRICS.gpu_mem_total.labels(g).set(d["mem_total"])
        for cb in list(self.callbacks):
            try:
                cb(self.latest)
            except Exception:
                pass
        return self.latest

    def vram_usage(self) -> Dict[int, float]:
        s = self.latest or self.poll()
        return {int(d["index"]): (d["mem_used"] / d["mem_total"] if d["mem_total"] else 0.0) for d in s}

    def detect_overload(self) -> List[int]:
        return [i for i, u in self.vram_usage().items() if u >= self.threshold]

    def start(self) -> None:
        if self._thread and self._thread.is_alive():
            return
        self._stop.clear()

        def loop():
            while not self._stop.wait(self.interval):
                try:
                    self.poll()
                except Exception:
                    pass

        self._thread = threading.Thread(target=loop, name="vrm-gpu-monitor", daemon=True)
        self._thread.start()

    def stop(self) -> None:
        self._stop.set()


class GPUHotPlugMonitor:
    def __init__(self, nvml: Optional[NVML] = None):
        self.nvml = nvml or NVML()
        self.known = set(range(self.nvml.count()))
        self.on_add: List[Callable[[int], None]] = []
        self.on_remove: List[Callable[[int], None]] = []

    def check(self) -> Dict[str, List[int]]:
        now = set(range(self.nvml.count()))
        added, removed = sorted(now - self.known), sorted(self.known - now)
        for i in added:
            for cb in self.on_add:
                cb(i)
        for i in removed:
            for cb in self.on_remove:
                cb(i)
        self.known = now
        return {"added": added, "removed": removed}


def system_info() -> Dict[str, object]:
    info = {"platform": platform.platform(), "python": platform.python_version(), "torch": torch.__version__,
            "cuda": torch.version.cuda, "cpus": os.cpu_count()}
    try:
        import psutil
        vm = psutil.virtual_memory()
        info.update(ram_total=vm.total, ram_available=vm.available, load=os.getloadavg()[0])
    except Exception:
        pass
    return info


def health_report(monitor: Optional[GPUMonitor] = None, extra: Optional[Dict] = None) -> Dict[str, object]:
    mon = monitor or GPUMonitor()
    gpus = mon.poll()
    status = "healthy"
    issues = []
    for g in gpus:
        if g["mem_total"] and g["mem_used"] / g["mem_total"] > 0.98:
            issues.append(f"gpu{int(g['index'])} memory > 98%")
        if g.get("temp_c", -1) >= 90:
            issues.append(f"gpu{int(g['index'])} temperature {g['temp_c']:.0f}C")
    if issues:
        status = "degraded"
    rep = {"status": status, "issues": issues, "gpus": gpus, "system": system_info(), "ts": time.time()}
    if extra:
        rep.update(extra)
    return rep


def doctor() -> Dict[str, object]:
    """Environment diagnosis: versions, GPUs, P2P matrix, kernels built, recommendation."""
    from ..parallel.placement import detect_gpus, probe_p2p
    from .. import ops
    rep = {"system": system_info(), "native_kernels": ops.native_available(), "gpus": [],
           "p2p": probe_p2p(), "nvml": NVML().ok}
    gpus = detect_gpus()
    rep["gpus"] = [g.to_dict() for g in gpus]
    total = sum(g.free_bytes for g in gpus)
    from ..quickstart import recommend
    rep["recommendation"] = recommend("chat", total / 2 ** 30, blackwell=any(g.capability[0] >= 10 for g in gpus))
    cc_ok = all(g.capability == (10, 0) for g in gpus) if gpus else False
    rep["sm100a"] = cc_ok
    return rep
