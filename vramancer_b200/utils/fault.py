"""GPU fault tolerance: health state machine, error classification, protected calls,
isolation and recovery probing, block replicas and the OOM auto-heal ladder.

Faults are classified from exception messages (OOM, ECC, thermal, driver, timeout,
device-side wait timeout reported by our kernels' error word).  A GPU with three
consecutive failures is isolated; a recovery thread probes isolated GPUs and
returns them to service.  `protected_call` retries an OOM once after freeing cached
memory, then falls back to another healthy device when the caller provides one.

Failures are injected on the host in tests (functions that raise, fake probes):
nothing here faults or hangs a GPU.

Reference parity: core/gpu_fault_tolerance.py:57-769 (states, _classify_error 198,
_handle_fault 220, _isolate_gpu 304, _recovery_loop 341, protected_call 441-525,
BlockReplicator 615-739), core/inference_pipeline.py:1071-1126 (OOM recover).
"""
from __future__ import annotations

import enum
import threading
import time
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional, Sequence

import torch

from .observability import METRICS, get_logger, send_alert

log = get_logger("vramancer.fault")


class GPUHealth(str, enum.Enum):
    HEALTHY = "healthy"
    DEGRADED = "degraded"
    OOM = "oom"
    FAILED = "failed"
    RECOVERING = "recovering"
    OFFLINE = "offline"


class FaultKind(str, enum.Enum):
    OOM = "oom"
    ECC = "ecc"
    THERMAL = "thermal"
    DRIVER = "driver"
    TIMEOUT = "timeout"
    DEVICE_WAIT = "device_wait_timeout"
    UNKNOWN = "unknown"


def classify_error(exc: BaseException) -> FaultKind:
    msg = str(exc).lower()
    if isinstance(exc, torch.cuda.OutOfMemoryError) or "out of memory" in msg or "cuda oom" in msg:
        return FaultKind.OOM
    if "ecc" in msg or "uncorrectable" in msg:
        return FaultKind.ECC
    if "thermal" in msg or "temperature" in msg:
        return FaultKind.THERMAL
    if "bounded wait" in msg or "device wait" in msg or "error word" in msg:
        return FaultKind.DEVICE_WAIT
    if "timeout" in msg or "timed out" in msg:
        return FaultKind.TIMEOUT
    if "driver" in msg or "cuda error" in msg or "illegal" in msg or "launch failure" in msg:
        return FaultKind.DRIVER
    return FaultKind.UNKNOWN


@dataclass
class GPUState:
    index: int
    health: GPUHealth = GPUHealth.HEALTHY
    consecutive_failures: int = 0
    total_failures: int = 0
    last_error: str = ""
    last_change: float = field(default_factory=time.time)


class GPUFaultManager:
    def __init__(self, gpus: Sequence[int], *, isolate_after: int = 3, probe: Optional[Callable[[int], bool]] = None,
                 recovery_interval_s: float = 5.0):
        self.states: Dict[int, GPUState] = {g: GPUState(g) for g in gpus}
        self.isolate_after = isolate_after
        self.probe = probe or self._default_probe
        self.recovery_interval = recovery_interval_s
        self.on_isolate: List[Callable[[int], None]] = []
        self.on_recover: List[Callable[[int], None]] = []
        self._lock = threading.RLock()
        self._stop = threading.Event()
        self._thread: Optional[threading.Thread] = None

    @staticmethod
    def _default_probe(g: int) -> bool:
        if not torch.cuda.is_available():
            return False
        try:
            with torch.cuda.device(g):
                x = torch.ones(16, device=f"cuda:{g}")
                return bool((x * 2).sum().item() == 32)
        except Exception:
            return False

    def healthy_gpus(self) -> List[int]:
        with self._lock:
            return [g for g, s in self.states.items() if s.health in (GPUHealth.HEALTHY, GPUHealth.DEGRADED)]

    def record_success(self, g: int) -> None:
        with self._lock:
            s = self.states[g]
            s.consecutive_failures = 0
            if s.health in (GPUHealth.OOM, GPUHealth.DEGRADED):
                s.health = GPUHealth.HEALTHY
                s.last_change = time.time()

    def handle_fault(self, g: int, exc: BaseException) -> FaultKind:
        kind = classify_error(exc)
        with self._lock:
            s = self.states[g]
            s.consecutive_failures += 1
            s.total_failures += 1
            s.last_error = str(exc)[:500]
            METRICS.gpu_faults.labels(str(g), kind.value).inc()
            if kind == FaultKind.OOM:
                s.health = GPUHealth.OOM
            elif kind in (FaultKind.ECC, FaultKind.DRIVER):
                s.health = GPUHealth.FAILED
            else:
                s.health = GPUHealth.DEGRADED
            s.last_change = time.time()
            isolate = s.consecutive_failures >= self.isolate_after or s.health == GPUHealth.FAILED
        if isolate:
            self.isolate(g)
        return kind

    def isolate(self, g: int) -> None:
        with self._lock:
            s = self.states[g]
            if s.health == GPUHealth.OFFLINE:
                return
            s.health = GPUHealth.OFFLINE
            s.last_change = time.time()
        log.warning("GPU %d isolated after %d failures (%s)", g, self.states[g].total_failures,
                    self.states[g].last_error[:120])
        send_alert("GPU isolated", f"gpu{g}: {self.states[g].last_error[:200]}", level="critical")
        for cb in list(self.on_isolate):
            cb(g)

    def try_recover(self) -> List[int]:
        back = []
        for g, s in list(self.states.items()):
            if s.health in (GPUHealth.OFFLINE, GPUHealth.FAILED):
                s.health = GPUHealth.RECOVERING
                if self.probe(g):
                    with self._lock:
                        s.health = GPUHealth.HEALTHY
                        s.consecutive_failures = 0
                        s.last_change = time.time()
                    back.append(g)
                    for cb in list(self.on_recover):
                        cb(g)
                else:
                    s.health = GPUHealth.OFFLINE
        return back

    def start_recovery_thread(self) -> None:
        if self._thread and self._thread.is_alive():
            return
        self._stop.clear()

        def loop():
            while not self._stop.wait(self.recovery_interval):
                self.try_recover()

        self._thread = threading.Thread(target=loop, name="vrm-gpu-recovery", daemon=True)
        self._thread.start()

    def stop(self) -> None:
        self._stop.set()

    def protected_call(self, g: int, fn: Callable[..., Any], *args, fallback: Optional[Callable[[int], Any]] = None,
                       **kwargs) -> Any:
        """Runs fn; on OOM frees the cache and retries once; on failure uses fallback(other_gpu)."""
        try:
            out = fn(*args, **kwargs)
            self.record_success(g)
            return out
        except Exception as e:
            kind = self.handle_fault(g, e)
            if kind == FaultKind.OOM:
                if torch.cuda.is_available():
                    torch.cuda.empty_cache()
                try:
                    out = fn(*args, **kwargs)
                    self.record_success(g)
                    return out
                except Exception as e2:
                    self.handle_fault(g, e2)
            others = [h for h in self.healthy_gpus() if h != g]
            if fallback is not None and others:
                return fallback(others[0])
            raise

    def status(self) -> Dict[str, Any]:
        with self._lock:
            return {str(g): {"health": s.health.value, "consecutive_failures": s.consecutive_failures,
                             "total_failures": s.total_failures, "last_error": s.last_error}
                    for g, s in self.states.items()}


class OOMAutoHeal:
    """Generation OOM ladder: free caches, retry with half the new tokens, and keep a
    persistent scale (x0.75 per OOM) applied to later requests' max_new_tokens."""

    def __init__(self, min_scale: float = 0.1):
        self.scale = 1.0
        self.min_scale = min_scale
        self.events = 0

    def scaled(self, max_new_tokens: int) -> int:
        return max(1, int(max_new_tokens * self.scale))

    def run(self, fn: Callable[[int], Any], max_new_tokens: int) -> Any:
        n = self.scaled(max_new_tokens)
        try:
            return fn(n)
        except Exception as e:
            if classify_error(e) != FaultKind.OOM:
                raise
            self.events += 1
            self.scale = max(self.min_scale, self.scale * 0.75)
            if torch.cuda.is_available():
                torch.cuda.empty_cache()
            return fn(max(1, n // 2))


class BlockReplicator:
    """Keeps k host copies of named tensors (layer blocks, hidden-state checkpoints)
    so a failed device's stage can be rebuilt on a survivor."""

    def __init__(self, k: int = 1):
        self.k = k
        self.replicas: Dict[str, List[torch.Tensor]] = {}
        self.checkpoints: Dict[str, torch.Tensor] = {}

    def replicate(self, name: str, t: torch.Tensor) -> None:
        self.replicas[name] = [t.detach().to("cpu", copy=True) for _ in range(self.k)]

    def restore(self, name: str, device) -> torch.Tensor:
        return self.replicas[name][0].to(device)

    def checkpoint(self, name: str, hidden: torch.Tensor) -> None:
        self.checkpoints[name] = hidden.detach().to("cpu", copy=True)

    def resume(self, name: str, device) -> Optional[torch.Tensor]:
        t = self.checkpoints.get(name)
        return None if t is None else t.to(device)


_manager: Optional[GPUFaultManager] = None


def get_fault_manager() -> GPUFaultManager:
    global _manager
    if _manager is None:
        n = torch.cuda.device_count() if torch.cuda.is_available() else 0
        _manager = GPUFaultManager(list(range(n)))
    return _manager
