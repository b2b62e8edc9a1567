"""Logging, Prometheus metrics, tracing spans, request history and webhook alerts.

* `get_logger` — plain or JSON (VRM_LOG_JSON=1) log lines.
* `METRICS` — Prometheus counters/gauges/histograms for inference, tokens, TTFT,
  batcher, paged KV, lending pool, transfers, circuit breaker and GPU memory;
  `start_metrics_server(port)` exposes them (default :9108).
* `span(name, **attrs)` — OpenTelemetry span when VRM_TRACING=1 and the SDK is
  present, otherwise a timing no-op that still records duration into the metrics.
* `RequestHistory` — last-N requests in SQLite (no prompt text).
* `send_alert` — webhook alert (Slack/Discord/Telegram-style JSON POST).

Reference parity: core/logger.py:17-78, core/metrics.py:13-121, core/tracing.py:44-88,
core/request_history.py:21-84, core/alerts.py:18-53.
"""
from __future__ import annotations

import contextlib
import json
import logging
import os
import sqlite3
import sys
import threading
import time
from typing import Any, Dict, List, Optional

try:
    import prometheus_client as prom
except Exception:  # pragma: no cover
    prom = None


# ----------------------------------------------------------------------------- logging
class JsonFormatter(logging.Formatter):
    def format(self, record: logging.LogRecord) -> str:
        d = {"ts": round(record.created, 3), "level": record.levelname, "logger": record.name,
             "msg": record.getMessage()}
        if record.exc_info:
            d["exc"] = self.formatException(record.exc_info)
        for k, v in getattr(record, "extra_fields", {}).items():
            d[k] = v
        return json.dumps(d)


def get_logger(name: str = "vramancer") -> logging.Logger:
    log = logging.getLogger(name)
    if not log.handlers:
        h = logging.StreamHandler(sys.stderr)
        if os.environ.get("VRM_LOG_JSON", "0") in ("1", "true"):
            h.setFormatter(JsonFormatter())
        else:
            h.setFormatter(logging.Formatter("%(asctime)s %(levelname)s %(name)s: %(message)s"))
        log.addHandler(h)
        log.setLevel(os.environ.get("VRM_LOG_LEVEL", "INFO").upper())
        log.propagate = False
    return log


# ----------------------------------------------------------------------------- metrics
class _NoMetric:
    def labels(self, *a, **k):
        return self

    def inc(self, *a, **k):
        pass

    def dec(self, *a, **k):
        pass

    def set(self, *a, **k):
        pass

    def observe(self, *a, **k):
        pass


class Metrics:
    def __init__(self, registry=None):
        self.registry = registry if registry is not None else (prom.CollectorRegistry() if prom else None)
        r = self.registry

        def c(name, doc, labels=()):
            return prom.Counter(name, doc, labels, registry=r) if prom else _NoMetric()

        def g(name, doc, labels=()):
            return prom.Gauge(name, doc, labels, registry=r) if prom else _NoMetric()

        def h(name, doc, buckets=None, labels=()):
            if not prom:
                return _NoMetric()
            kw = {"buckets": buckets} if buckets else {}
            return prom.Histogram(name, doc, labels, registry=r, **kw)

        self.infer_requests = c("vrm_infer_requests_total", "inference requests", ("endpoint",))
        self.infer_errors = c("vrm_infer_errors_total", "failed inference requests", ("kind",))
        self.tokens_generated = c("vrm_tokens_generated_total", "generated tokens")
        self.prompt_tokens = c("vrm_prompt_tokens_total", "prompt tokens")
        self.infer_latency = h("vrm_infer_latency_seconds", "request latency")
        self.ttft = h("vrm_ttft_seconds", "time to first token",
                      buckets=(0.005, 0.01, 0.025, 0.05, 0.1, 0.25, 0.5, 1, 2.5, 5, 10))
        self.itl = h("vrm_inter_token_latency_seconds", "inter-token latency",
                     buckets=(0.001, 0.0025, 0.005, 0.01, 0.025, 0.05, 0.1, 0.25))
        self.batch_size = g("vrm_batcher_running", "running requests in the batcher")
        self.queue_depth = g("vrm_batcher_waiting", "waiting requests")
        self.kv_used_pages = g("vrm_kv_used_pages", "paged KV pages in use", ("device",))
        self.kv_free_pages = g("vrm_kv_free_pages", "paged KV pages free", ("device",))
        self.kv_prefix_hits = c("vrm_kv_prefix_hits_total", "prefix cache hits")
        self.lending_leases = g("vrm_lending_active_leases", "active VRAM leases")
        self.lending_bytes = g("vrm_lending_borrowed_bytes", "bytes borrowed through the lending pool")
        self.lending_reclaims = c("vrm_lending_reclaims_total", "lease reclaims", ("urgency",))
        self.transfer_bytes = c("vrm_transfer_bytes_total", "bytes moved between devices", ("method",))
        self.transfer_seconds = h("vrm_transfer_seconds", "device transfer time", labels=("method",))
        self.circuit_state = g("vrm_circuit_breaker_state", "0 closed, 1 half-open, 2 open")
        self.gpu_mem_used = g("vrm_gpu_memory_used_bytes", "GPU memory in use", ("gpu",))
        self.gpu_mem_total = g("vrm_gpu_memory_total_bytes", "GPU memory total", ("gpu",))
        self.gpu_faults = c("vrm_gpu_faults_total", "classified GPU faults", ("gpu", "kind"))
        self.span_seconds = h("vrm_span_seconds", "traced span durations", labels=("span",))

    def exposition(self) -> bytes:
        if not prom:
            return b""
        return prom.generate_latest(self.registry)


METRICS = Metrics()
_metrics_server = None


def start_metrics_server(port: int = 9108, addr: str = "0.0.0.0") -> bool:
    global _metrics_server
    if not prom or _metrics_server is not None:
        return False
    prom.start_http_server(port, addr=addr, registry=METRICS.registry)
    _metrics_server = port
    return True


def reset_metrics() -> None:
    global METRICS
    METRICS = Metrics()


# ----------------------------------------------------------------------------- tracing
_tracer = None


def _get_tracer():
    global _tracer
    if _tracer is not None:
        return _tracer or None
    _tracer = False
    if os.environ.get("VRM_TRACING") in ("1", "true"):
        try:
            from opentelemetry import trace  # type: ignore
            _tracer = trace.get_tracer("vramancer")
        except Exception:
            _tracer = False
    return _tracer or None


@contextlib.contextmanager
def span(name: str, **attrs):
    """OTEL span if enabled; always records the duration under vrm_span_seconds."""
    t0 = time.perf_counter()
    tr = _get_tracer()
    if tr is not None:
        with tr.start_as_current_span(name) as sp:
            for k, v in attrs.items():
                sp.set_attribute(k, v)
            try:
                yield sp
            except Exception as e:
                sp.set_attribute("error", str(e))
                raise
    else:
        yield None
    METRICS.span_seconds.labels(name).observe(time.perf_counter() - t0)


# ----------------------------------------------------------------------------- history
class RequestHistory:
    """Last-N request records in SQLite (model, token counts, latency, status)."""

    def __init__(self, path: Optional[str] = None, keep: int = 1000):
        self.path = path or os.environ.get("VRM_HISTORY_DB") or ":memory:"
        self.keep = keep
        self._lock = threading.Lock()
        self._db = sqlite3.connect(self.path, check_same_thread=False)
        self._db.execute("CREATE TABLE IF NOT EXISTS requests (id INTEGER PRIMARY KEY AUTOINCREMENT, ts REAL, "
                         "endpoint TEXT, model TEXT, prompt_tokens INT, completion_tokens INT, latency_s REAL, "
                         "ttft_s REAL, status TEXT)")
        self._db.commit()

    def record(self, endpoint: str, model: str, prompt_tokens: int, completion_tokens: int, latency_s: float,
               ttft_s: Optional[float] = None, status: str = "ok") -> None:
        with self._lock:
            self._db.execute("INSERT INTO requests (ts, endpoint, model, prompt_tokens, completion_tokens, latency_s,"
                             " ttft_s, status) VALUES (?,?,?,?,?,?,?,?)",
                             (time.time(), endpoint, model, prompt_tokens, completion_tokens, latency_s, ttft_s,
                              status))
            self._db.execute("DELETE FROM requests WHERE id NOT IN (SELECT id FROM requests ORDER BY id DESC LIMIT ?)",
                             (self.keep,))
            self._db.commit()

    def recent(self, limit: int = 20) -> List[Dict[str, Any]]:
        with self._lock:
            cur = self._db.execute("SELECT ts, endpoint, model, prompt_tokens, completion_tokens, latency_s, ttft_s, "
                                   "status FROM requests ORDER BY id DESC LIMIT ?", (limit,))
            cols = [d[0] for d in cur.description]
            return [dict(zip(cols, r)) for r in cur.fetchall()]


# ----------------------------------------------------------------------------- alerts
def send_alert(title: str, message: str, *, level: str = "warning", url: Optional[str] = None,
               timeout: float = 3.0) -> bool:
    url = url or os.environ.get("VRM_ALERT_WEBHOOK")
    if not url:
        return False
    payload = {"text": f"[{level.upper()}] {title}: {message}", "content": f"{title}: {message}",
               "level": level, "title": title, "message": message}
    try:
        import urllib.request
        req = urllib.request.Request(url, data=json.dumps(payload).encode(), headers={"Content-Type":
                                                                                       "application/json"})
        urllib.request.urlopen(req, timeout=timeout).read()
        return True
    except Exception:
        return False
