"""API protection: bearer token, HMAC request signing, per-IP rate limit, body-size
cap, read-only mode, audit log, circuit breaker, request validation, queue counter.

Reference parity: core/security/__init__.py:38-523 (install_security 326),
core/security/audit_log.py:65-171, core/api/circuit_breaker.py:37-210,
core/api/validation.py:14-77, core/production_api.py:50-127 (_QueueCounter).
"""
from __future__ import annotations

import hashlib
import hmac
import os
import sqlite3
import threading
import time
from collections import defaultdict, deque
from typing import Any, Deque, Dict, Optional, Tuple


class ValidationError(ValueError):
    pass


def validate_generation_params(body: Dict[str, Any], max_tokens_cap: int = 32768) -> Dict[str, Any]:
    out: Dict[str, Any] = {}
    mt = body.get("max_tokens", body.get("max_new_tokens", 128))
    try:
        mt = int(mt)
    except (TypeError, ValueError):
        raise ValidationError("max_tokens must be an integer")
    if not (1 <= mt <= max_tokens_cap):
        raise ValidationError(f"max_tokens must be in [1, {max_tokens_cap}]")
    out["max_new_tokens"] = mt
    t = body.get("temperature", 0.0)
    if t is None:
        t = 0.0
    try:
        t = float(t)
    except (TypeError, ValueError):
        raise ValidationError("temperature must be a number")
    if not (0.0 <= t <= 5.0):
        raise ValidationError("temperature must be in [0, 5]")
    out["temperature"] = t
    p = body.get("top_p", 1.0)
    p = 1.0 if p is None else float(p)
    if not (0.0 < p <= 1.0):
        raise ValidationError("top_p must be in (0, 1]")
    out["top_p"] = p
    k = body.get("top_k", 0)
    k = 0 if k is None else int(k)
    if k < 0:
        raise ValidationError("top_k must be >= 0")
    out["top_k"] = k
    # OpenAI "stop": up to 4 non-empty strings; "n": independent completions per prompt
    stop = body.get("stop")
    if stop is None:
        stop = []
    elif isinstance(stop, str):
        stop = [stop]
    if not isinstance(stop, list) or len(stop) > 4 or not all(isinstance(x, str) and x for x in stop):
        raise ValidationError("stop must be a non-empty string or a list of at most 4")
    out["stop"] = stop
    n = body.get("n", 1)
    try:
        n = int(1 if n is None else n)
    except (TypeError, ValueError):
        raise ValidationError("n must be an integer")
    if not (1 <= n <= 8):
        raise ValidationError("n must be in [1, 8]")
    out["n"] = n
    return out


class CircuitBreaker:
    """CLOSED -> OPEN after `threshold` consecutive failures; OPEN -> HALF_OPEN after
    `reset_s`; one success in HALF_OPEN closes it, a failure reopens it."""

    CLOSED, HALF_OPEN, OPEN = "closed", "half_open", "open"

    def __init__(self, threshold: int = 5, reset_s: float = 30.0):
        self.threshold, self.reset_s = threshold, reset_s
        self.state = self.CLOSED
        self.failures = 0
        self.opened_at = 0.0
        self._lock = threading.Lock()

    def allow(self) -> bool:
        with self._lock:
            if self.state == self.OPEN and time.time() - self.opened_at >= self.reset_s:
                self.state = self.HALF_OPEN
            return self.state != self.OPEN

    def success(self) -> None:
        with self._lock:
            self.failures = 0
            self.state = self.CLOSED

    def failure(self) -> None:
        with self._lock:
            self.failures += 1
            if self.state == self.HALF_OPEN or self.failures >= self.threshold:
                self.state = self.OPEN
                self.opened_at = time.time()

    def code(self) -> int:
        return {self.CLOSED: 0, self.HALF_OPEN: 1, self.OPEN: 2}[self.state]


class RateLimiter:
    """Sliding one-minute window per key."""

    def __init__(self, per_minute: int = 600):
        self.per_minute = per_minute
        self.hits: Dict[str, Deque[float]] = defaultdict(deque)
        self._lock = threading.Lock()

    def allow(self, key: str) -> bool:
        now = time.time()
        with self._lock:
            q = self.hits[key]
            while q and now - q[0] > 60.0:
                q.popleft()
            if len(q) >= self.per_minute:
                return False
            q.append(now)
            return True


class QueueCounter:
    """In-flight request counter with a cap (429 beyond it)."""

    def __init__(self, limit: int = 256):
        self.limit = limit
        self.n = 0
        self._lock = threading.Lock()

    def acquire(self) -> bool:
        with self._lock:
            if self.n >= self.limit:
                return False
            self.n += 1
            return True

    def release(self) -> None:
        with self._lock:
            self.n = max(0, self.n - 1)


def sign_request(secret: str, method: str, path: str, body: bytes, ts: Optional[int] = None) -> Tuple[str, str]:
    ts = int(time.time()) if ts is None else int(ts)
    msg = f"{ts}.{method.upper()}.{path}.".encode() + body
    return str(ts), hmac.new(secret.encode(), msg, hashlib.sha256).hexdigest()


def verify_signature(secret: str, method: str, path: str, body: bytes, ts: str, sig: str,
                     max_skew_s: int = 300) -> bool:
    try:
        t = int(ts)
    except (TypeError, ValueError):
        return False
    if abs(time.time() - t) > max_skew_s:
        return False
    _, want = sign_request(secret, method, path, body, t)
    return hmac.compare_digest(want, sig or "")


class AuditLog:
    def __init__(self, path: Optional[str] = None):
        self.path = path or os.environ.get("VRM_AUDIT_DB") or ":memory:"
        self._db = sqlite3.connect(self.path, check_same_thread=False)
        self._lock = threading.Lock()
        self._db.execute("CREATE TABLE IF NOT EXISTS audit (ts REAL, client TEXT, method TEXT, path TEXT, "
                         "status INT, detail TEXT)")
        self._db.commit()

    def log(self, client: str, method: str, path: str, status: int, detail: str = "") -> None:
        with self._lock:
            self._db.execute("INSERT INTO audit VALUES (?,?,?,?,?,?)", (time.time(), client, method, path, status,
                                                                         detail[:500]))
            self._db.commit()

    def recent(self, n: int = 50):
        with self._lock:
            return self._db.execute("SELECT ts, client, method, path, status, detail FROM audit ORDER BY ts DESC "
                                    "LIMIT ?", (n,)).fetchall()


def startup_checks(production: bool) -> list:
    """Warnings (or errors in production) about an unsafe configuration."""
    issues = []
    if not os.environ.get("VRM_API_TOKEN"):
        issues.append("VRM_API_TOKEN is not set: the API is open")
    if os.environ.get("VRM_DISABLE_RATE_LIMIT") in ("1", "true"):
        issues.append("rate limiting disabled")
    if production and issues:
        raise RuntimeError("production startup checks failed: " + "; ".join(issues))
    return issues
