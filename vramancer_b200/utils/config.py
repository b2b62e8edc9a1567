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
    "VRM_NODES": (str, "", "cluster", "static node list (comma-separated host:port)"),
    "VRM_CLUSTER_KEY": (str, "", "cluster", "shared key of the cluster worker routes"),
    # security / accounts
    "VRM_AUTH_SECRET": (str, "", "security", "HS256 signing key of access tokens (random per process when empty)"),
    "VRM_AUTH_EXP": (int, 900, "security", "access-token lifetime, seconds"),
    "VRM_AUTH_REFRESH_EXP": (int, 86400, "security", "refresh-token lifetime, seconds"),
    "VRM_AUTH_USERS_FILE": (str, "", "security", "JSON file of accounts (PBKDF2 hashes)"),
    "VRM_DEFAULT_ADMIN_PASS": (str, "", "security", "password of the bootstrap admin account"),
    "VRM_CORS_ORIGINS": (str, "http://localhost,http://127.0.0.1", "security",
                         "allowed CORS origins (comma-separated, * for any)"),
    "VRM_LEDGER_DB": (str, "", "security", "SQLite file of the credit ledger for sk-VRAM- keys (off when empty)"),
    "VRM_HMAC_SECRET": (str, "", "security", "HMAC-SHA256 request-signing secret"),
    "VRM_AUDIT_DB": (str, "", "security", "SQLite audit log path"),
    "VRM_CONFIG": (str, "", "misc", "YAML configuration file"),
    # engine
    "VRM_LOOKAHEAD": (bool, True, "backend", "launch decode step n+1 before reading back step n"),
    "VRM_FOLD_NORM": (bool, True, "backend", "fold RMSNorm weights into the next GEMM's columns"),
    "VRM_FOLD_MAX_TOKENS": (int, 16, "backend", "largest batch that runs the folded norms (TP=1)"),
    "VRM_FOLD_MAX_TOKENS_TP": (int, 128, "backend", "largest batch that runs the folded norms (TP>1)"),
    "VRM_FUSED_ROPE": (bool, True, "backend", "RoPE + KV write inside decode attention"),
    "VRM_FUSED_AR": (bool, True, "backend", "tensor-parallel all-reduce fused into the GEMMs"),
    "VRM_FUSED_AR_MIN_TOKENS": (int, 1, "backend", "smallest batch on the fused all-reduce"),
    "VRM_FUSED_AR_MAX_TOKENS": (int, 128, "backend", "largest batch on the fused all-reduce"),
    "VRM_VP_SAMPLE": (bool, True, "backend", "vocabulary-parallel sampling under TP"),
    "VRM_NVFP4_DECODE": (str, "mma", "backend", "NVFP4 decode GEMM: mma (warp MMA) | tc (tcgen05)"),
    "VRM_NVFP4_PREFILL": (str, "w4a4", "backend", "NVFP4 prefill: w4a4 (block-scaled tcgen05) or dequant"),
    # kernel selection / tuning (read once per process by the CUDA extension)
    "VRM_GEMM_PREFILL": (str, "", "kernel", "prefill GEMM: tiled | streamk | streamk256 | persistent | persistent256"),
    "VRM_GEMM_PREFILL_STAGES": (int, 3, "kernel", "tiled prefill GEMM pipeline depth (3 or 6)"),
    "VRM_GEMM_PERSIST_SK": (bool, False, "kernel", "persistent GEMM remainder as stream-K instead of split"),
    "VRM_GEMM_PERSIST_SPLITS": (int, 0, "kernel", "persistent GEMM: split the remainder tiles this many ways (0 = cost model)"),
    "VRM_GEMM_CTAS": (int, 0, "kernel", "stream-K decode GEMM CTA count (0 = cost model)"),
    "VRM_GEMM_CLUSTER": (bool, True, "kernel", "cluster split-K reduction in the decode GEMM"),
    "VRM_GEMM_LEGACY_DECODE": (bool, False, "kernel", "older non-stream-K decode GEMM"),
    "VRM_DECODE_CLUSTER": (bool, True, "kernel", "decode attention split merge through cluster shared memory"),
    "VRM_DECODE_TMA": (bool, False, "kernel", "persistent TMA decode attention for bf16 pages"),
    "VRM_PREFILL_TC": (bool, False, "kernel", "tcgen05 prefill attention (bf16 pages)"),
    "VRM_L2_PREFETCH": (bool, False, "kernel", "decode attention prefetches the o_proj weights into L2"),
}

# the reference's names for variables that mean the same thing here (read when the
# name on the left is unset)
FLAG_ALIASES: Dict[str, str] = {
    "VRM_MAX_BODY_BYTES": "VRM_MAX_BODY",
    "VRM_MAX_QUEUE": "VRM_MAX_QUEUE_SIZE",
    "VRM_REQUEST_TIMEOUT": "VRM_GENERATE_TIMEOUT",
    "VRM_RATE_LIMIT_RPM": "VRM_RATE_MAX",
}


class _Flags:
    """Live view: `flags.VRM_MAX_BATCH_SIZE` reads the environment every time."""

    def __getattr__(self, name: str) -> Any:
        if name not in FLAG_REGISTRY:
            raise AttributeError(name)
        typ, default, _, _ = FLAG_REGISTRY[name]
        raw = os.environ.get(name)
        if (raw is None or raw == "") and name in FLAG_ALIASES:
            raw = os.environ.get(FLAG_ALIASES[name])
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
