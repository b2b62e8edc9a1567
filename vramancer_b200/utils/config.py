"""Typed configuration: defaults -> YAML file -> VRM_* environment variables.

`get_config()` returns one `Config` object; `flags` is a live view of the VRM_*
environment flags (each attribute reads os.environ at access time, so tests and
operators can flip them at run time).  The variable names are the reference's, so
existing deployments keep their environment.

Reference parity: core/config.py:36-342 (DEFAULTS, YAML paths, env overrides,
reload hooks), core/env_flags.py:55-630 (typed live-read facade and registry).
"""
from __future__ import annotations

import dataclasses
import os
import threading
from dataclasses import dataclass, field
from typing import Any, Callable, Dict, List, Optional

try:
    import yaml
except Exception:  # pragma: no cover
    yaml = None


def _bool(v: Optional[str], default: bool = False) -> bool:
    if v is None:
        return default
    return v.strip().lower() in ("1", "true", "yes", "on")


# name -> (type, default, category, description)
FLAG_REGISTRY: Dict[str, tuple] = {
    "VRM_API_TOKEN": (str, "", "security", "bearer token required by the API (empty = open)"),
    "VRM_PRODUCTION": (bool, False, "security", "production mode: strict startup checks"),
    "VRM_READ_ONLY": (bool, False, "security", "reject model loads and mutations"),
    "VRM_DISABLE_RATE_LIMIT": (bool, False, "security", "disable per-IP rate limiting"),
    "VRM_RATE_LIMIT_RPM": (int, 600, "security", "requests per minute per client IP"),
    "VRM_MAX_BODY_BYTES": (int, 4 << 20, "api", "maximum request body"),
    "VRM_MAX_CONCURRENT": (int, 4, "api", "concurrent inference requests"),
    "VRM_MAX_QUEUE": (int, 256, "api", "queued requests before 429"),
    "VRM_REQUEST_TIMEOUT": (float, 120.0, "api", "seconds before 504"),
    "VRM_MODEL_ALIAS": (str, "", "api", "model id reported by /v1/models"),
    "VRM_QUANTIZATION": (str, "", "backend", "nvfp4 | fp8 | none"),
    "VRM_KV_CACHE_DTYPE": (str, "bf16", "kv", "bf16 | fp8"),
    "VRM_KV_COMPRESSION": (str, "", "kv", "turboquant to compress cold KV pages"),
    "VRM_KV_COMPRESSION_BITS": (int, 3, "kv", "TurboQuant bits per angle"),
    "VRM_PARALLEL_MODE": (str, "tp", "backend", "tp | pp"),
    "VRM_CONTINUOUS_BATCHING": (bool, True, "backend", "iteration-level scheduler"),
    "VRM_MAX_BATCH_SIZE": (int, 64, "backend", "running requests per step"),
    "VRM_PREFILL_CHUNK": (int, 8192, "backend", "prefill tokens per step"),
    "VRM_CUDA_GRAPH": (bool, True, "backend", "decode under CUDA graphs"),
    "VRM_PDL": (bool, True, "backend", "programmatic dependent launch between kernels"),
    "VRM_PROMPT_LOOKUP": (int, 0, "spec", "prompt-lookup speculative tokens (0 = off)"),
    "VRM_PROMPT_LOOKUP_NGRAM": (int, 3, "spec", "n-gram size for prompt lookup"),
    "VRM_DRAFT_MODEL": (str, "", "spec", "draft model for speculative decoding"),
    "VRM_SPEC_GAMMA": (int, 5, "spec", "draft tokens per round"),
    "VRM_SPEC_ADAPTIVE": (bool, True, "spec", "adapt gamma to acceptance"),
    "VRM_VRAM_LENDING": (bool, True, "lending", "cross-GPU VRAM lending pool"),
    "VRM_LEND_RATIO": (float, 0.7, "lending", "fraction of free VRAM a GPU may lend"),
    "VRM_RECLAIM_THRESHOLD": (float, 0.80, "lending", "lender utilisation that triggers reclaim"),
    "VRM_KV_LEND": (bool, True, "lending", "KV overflow pages may live on a lender GPU"),
    "VRM_GPU_ORDER": (str, "", "placement", "comma-separated GPU order"),
    "VRM_HETERO_STRATEGY": (str, "balanced", "placement", "vram | compute | balanced | profile"),
    "VRM_N_CTX": (int, 4096, "backend", "maximum context length"),
    "VRM_METRICS_PORT": (int, 9108, "observability", "Prometheus exporter port"),
    "VRM_TRACING": (bool, False, "observability", "OpenTelemetry spans"),
    "VRM_LOG_JSON": (bool, False, "observability", "JSON log lines"),
    "VRM_LOG_LEVEL": (str, "INFO", "observability", "log level"),
    "VRM_HISTORY_DB": (str, "", "observability", "request history SQLite path"),
    "VRM_ALERT_WEBHOOK": (str, "", "observability", "webhook URL for alerts"),
    "VRM_TEST_MODE": (bool, False, "test", "test mode (small defaults)"),
    "VRM_MINIMAL_TEST": (bool, False, "test", "stub heavy subsystems"),
    "VRM_CLUSTER_PORT": (int, 5040, "cluster", "data-parallel cluster port"),
    "VRM_DISCOVERY_PORT": (int, 5353, "cluster", "UDP discovery port"),
}


class _Flags:
    """Live view: `flags.VRM_MAX_BATCH_SIZE` reads the environment every time."""

    def __getattr__(self, name: str) -> Any:
        if name not in FLAG_REGISTRY:
            raise AttributeError(name)
        typ, default, _, _ = FLAG_REGISTRY[name]
        raw = os.environ.get(name)
        if raw is None or raw == "":
            return default
        if typ is bool:
            return _bool(raw, default)
        try:
            return typ(raw)
        except ValueError:
            return default

    def describe(self) -> List[Dict[str, Any]]:
        return [{"name": n, "type": t.__name__, "default": d, "category": c, "doc": doc,
                 "value": getattr(self, n)} for n, (t, d, c, doc) in sorted(FLAG_REGISTRY.items())]


flags = _Flags()


@dataclass
class Config:
    model: str = "qwen2.5-14b"
    host: str = "0.0.0.0"
    port: int = 5030
    metrics_port: int = 9108
    max_batch: int = 64
    max_model_len: int = 4096
    kv_cache_dtype: str = "bf16"
    quantization: str = ""
    gpu_memory_utilization: float = 0.9
    prefill_chunk: int = 8192
    cuda_graph: bool = True
    prompt_lookup: int = 0
    tp: int = 1
    pp: int = 1
    lending: bool = True
    log_json: bool = False
    extra: Dict[str, Any] = field(default_factory=dict)

    def validate(self) -> List[str]:
        errs = []
        if not (0 < self.port < 65536):
            errs.append("port out of range")
        if not (0.05 <= self.gpu_memory_utilization <= 1.0):
            errs.append("gpu_memory_utilization must be in [0.05, 1]")
        if self.max_batch < 1:
            errs.append("max_batch must be >= 1")
        if self.kv_cache_dtype not in ("bf16", "fp8"):
            errs.append("kv_cache_dtype must be bf16 or fp8")
        return errs


_ENV_MAP = {"VRM_MAX_BATCH_SIZE": "max_batch", "VRM_N_CTX": "max_model_len", "VRM_KV_CACHE_DTYPE": "kv_cache_dtype",
            "VRM_QUANTIZATION": "quantization", "VRM_PREFILL_CHUNK": "prefill_chunk", "VRM_CUDA_GRAPH": "cuda_graph",
            "VRM_PROMPT_LOOKUP": "prompt_lookup", "VRM_METRICS_PORT": "metrics_port", "VRM_LOG_JSON": "log_json",
            "VRM_VRAM_LENDING": "lending"}


def config_paths() -> List[str]:
    home = os.path.expanduser("~")
    xdg = os.environ.get("XDG_CONFIG_HOME", os.path.join(home, ".config"))
    return [os.environ.get("VRM_CONFIG", ""), "config.yaml", os.path.join(xdg, "vramancer", "config.yaml"),
            os.path.join(home, "Library", "Application Support", "vramancer", "config.yaml")]


_lock = threading.Lock()
_config: Optional[Config] = None
_reload_hooks: List[Callable[[Config], None]] = []


def _load() -> Config:
    c = Config()
    for p in config_paths():
        if p and os.path.exists(p) and yaml is not None:
            try:
                data = yaml.safe_load(open(p)) or {}
            except Exception:
                data = {}
            for k, v in data.items():
                if hasattr(c, k):
                    setattr(c, k, v)
                else:
                    c.extra[k] = v
            break
    for env, attr in _ENV_MAP.items():
        if os.environ.get(env):
            setattr(c, attr, getattr(flags, env))
    return c


def get_config() -> Config:
    global _config
    with _lock:
        if _config is None:
            _config = _load()
        return _config


def reload_config() -> Config:
    global _config
    with _lock:
        _config = _load()
        cfg = _config
    for h in list(_reload_hooks):
        h(cfg)
    return cfg


def on_reload(hook: Callable[[Config], None]) -> None:
    _reload_hooks.append(hook)
