"""`vramancer` command line (also `python -m vramancer_b200`).

Subcommands: run, serve, generate, status, benchmark, discover, split, dashboard,
quickstart, hub, health, doctor, history, cluster (serve | gateway), auth, version.

Reference parity: vramancer/main.py:14-704 (same subcommands and main options).
"""
from __future__ import annotations

import argparse
import json
import os
import socket
import secrets
import subprocess
import sys
import time
from typing import List, Optional

__version__ = "0.1.0"



# `-q` accepts the reference's names too.  nf4 / int8 are served by the formats the B200
# tensor cores run natively (4-bit NVFP4, 8-bit FP8 e4m3 W8A8); gptq / awq name
# pre-quantised checkpoint layouts, which the loader recognises from the checkpoint's
# quantization_config and dequantises at load (add -q fp8 / nvfp4 to re-quantise).
QUANT_CHOICES = ["nvfp4", "fp8", "none", "nf4", "int8", "gptq", "awq"]
_QUANT_ALIASES = {"nf4": "nvfp4", "int8": "fp8"}


def resolve_quantization(q):
    if q in ("gptq", "awq"):
        print(f"-q {q}: the checkpoint's {q.upper()} tensors are dequantised at load (bf16 weights)")
        return None
    if q in _QUANT_ALIASES:
        print(f"-q {q}: using {_QUANT_ALIASES[q]} (the B200-native {'4' if q == 'nf4' else '8'}-bit weight format)")
        return _QUANT_ALIASES[q]
    return q

def _print(obj) -> None:
    print(json.dumps(obj, indent=1, default=str))


def build_parser() -> argparse.ArgumentParser:
    p = argparse.ArgumentParser(prog="vramancer", description="VRAMancer-B200: multi-GPU LLM inference on B200")
    sub = p.add_subparsers(dest="command")

    r = sub.add_parser("run", help="load a model and generate (one-shot or interactive)")
    r.add_argument("model")
    r.add_argument("--prompt", "-p", default=None)
    r.add_argument("--max-tokens", type=int, default=256)
    r.add_argument("--temperature", type=float, default=0.7)
    r.add_argument("--backend", default="auto")
    r.add_argument("--gpus", type=int, default=None)
    r.add_argument("--quantization", "-q", default=None, choices=QUANT_CHOICES)
    r.add_argument("--num-layers", type=int, default=None, help=argparse.SUPPRESS)

    s = sub.add_parser("serve", help="OpenAI-compatible API server")
    s.add_argument("model_pos", nargs="?", default=None, metavar="model")
    s.add_argument("--model", default=None)
    s.add_argument("--backend", default="auto")
    s.add_argument("--gpus", type=int, default=None)
    s.add_argument("--tp", type=int, default=1, help="tensor-parallel ranks (torchrun, one process per GPU)")
    s.add_argument("--host", default="0.0.0.0")
    s.add_argument("--port", type=int, default=5030)
    s.add_argument("--quantization", "-q", default=None, choices=QUANT_CHOICES)
    s.add_argument("--no-cluster", dest="cluster", action="store_false", default=True)
    s.add_argument("--profile", default=None, choices=["coding", "multi-user"])
    s.add_argument("--max-model-len", type=int, default=None)
    s.add_argument("--num-layers", type=int, default=None, help=argparse.SUPPRESS)

    g = sub.add_parser("generate", help="one generation")
    g.add_argument("--model", required=True)
    g.add_argument("--prompt", required=True)
    g.add_argument("--max-tokens", type=int, default=64)
    g.add_argument("--num-layers", type=int, default=None, help=argparse.SUPPRESS)

    sub.add_parser("status", help="GPUs, kernels and configuration")
    b = sub.add_parser("benchmark", help="kernel microbenchmarks, a model benchmark or a serving workload")
    b.add_argument("--size", type=int, default=4096)
    b.add_argument("--model", default=None)
    b.add_argument("--workload", default=None, choices=["serve", "spec", "prefill", "decode"],
                   help="run a serving workload (vramancer_b200.workloads) on --model; extra options after --")
    b.add_argument("rest", nargs=argparse.REMAINDER)
    d = sub.add_parser("discover", help="listen for nodes announcing themselves")
    d.add_argument("--timeout", type=float, default=5.0)
    sp = sub.add_parser("split", help="show the layer split across GPUs")
    sp.add_argument("model")
    sp.add_argument("--gpus", type=int, default=2)
    sp.add_argument("--profile", dest="profile", action="store_true", default=False)
    sp.add_argument("--no-profile", dest="profile", action="store_false")
    sp.add_argument("--strategy", default="balanced", choices=["vram", "compute", "balanced"])
    db = sub.add_parser("dashboard", help="web (or CLI) dashboard")
    db.add_argument("--port", type=int, default=8500)
    db.add_argument("--cli", action="store_true")
    q = sub.add_parser("quickstart", help="recommend the largest model that fits")
    q.add_argument("use_case", nargs="?", default="chat", choices=["code-assistant", "chat", "summarize"])
    q.add_argument("--run", action="store_true", help="launch the recommended model (interactive, or --prompt)")
    q.add_argument("--serve", action="store_true", help="serve the recommended model (OpenAI API)")
    q.add_argument("--prompt", "-p", default=None)
    q.add_argument("--port", type=int, default=5030)
    h = sub.add_parser("hub", help="inspect a model directory / name")
    h.add_argument("model")
    sub.add_parser("health", help="node health report")
    sub.add_parser("doctor", help="environment diagnosis")
    hi = sub.add_parser("history", help="recent requests of a running server")
    hi.add_argument("--limit", type=int, default=20)
    hi.add_argument("--url", default="http://127.0.0.1:5030")
    c = sub.add_parser("cluster", help="data-parallel cluster")
    c.add_argument("action", choices=["serve", "gateway"])
    c.add_argument("model", nargs="?", default=None)
    c.add_argument("--gpus", default=None, help="comma-separated GPU ids")
    c.add_argument("--nodes", default=None, help="comma-separated node URLs (gateway)")
    c.add_argument("--discover", action="store_true")
    c.add_argument("--check", action="store_true")
    c.add_argument("--port", type=int, default=5040)
    a = sub.add_parser("auth", help="generate an API token")
    a.add_argument("--show", action="store_true")
    sub.add_parser("version", help="version")
    return p


def _cmd_run(a) -> int:
    from .pipeline import InferencePipeline
    pipe = InferencePipeline(verbose=True).load(a.model, num_gpus=a.gpus, quantization=resolve_quantization(a.quantization),
                                                num_layers=a.num_layers)
    try:
        if a.prompt is not None:
            for delta in pipe.generate_stream(a.prompt, max_new_tokens=a.max_tokens, temperature=a.temperature):
                sys.stdout.write(delta)
                sys.stdout.flush()
            sys.stdout.write("\n")
            return 0
        while True:
            try:
                line = input(">>> ")
            except EOFError:
                break
            if line.strip() in ("exit", "quit"):
                break
            for delta in pipe.generate_stream(line, max_new_tokens=a.max_tokens, temperature=a.temperature):
                sys.stdout.write(delta)
                sys.stdout.flush()
            sys.stdout.write("\n")
    finally:
        pipe.shutdown()
    return 0


def _cmd_serve(a) -> int:
    model = a.model or a.model_pos
    if a.profile == "coding":
        os.environ.setdefault("VRM_N_CTX", "16384")
    elif a.profile == "multi-user":
        os.environ.setdefault("VRM_MAX_BATCH_SIZE", "128")
    if a.tp > 1 and int(os.environ.get("WORLD_SIZE", "1")) == 1:
        # relaunch one process per GPU; rank 0 serves HTTP, the others follow
        cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={a.tp}",
               "--master-addr=127.0.0.1", "-m", "vramancer_b200", "serve", model, "--host", a.host, "--port",
               str(a.port), "--tp", str(a.tp)]
        return subprocess.call(cmd)
    from .serving.api import run_server
    from .pipeline import InferencePipeline
    pipe = None
    if model:
        kw = {}
        if a.max_model_len:
            kw["max_model_len"] = a.max_model_len
        pipe = InferencePipeline().load(model, num_gpus=a.gpus, quantization=resolve_quantization(a.quantization),
                                        num_layers=a.num_layers, **kw)
    if int(os.environ.get("RANK", "0")) != 0:
        from .parallel.follower import follow
        return follow(pipe)
    if a.cluster:
        from .cluster.discovery import announce
        from .cluster.mdns import MDNSResponder
        announce(a.host, a.port, {"model": model})
        ip = a.host if a.host not in ("0.0.0.0", "") else socket.gethostbyname(socket.gethostname())
        MDNSResponder(f"vrm-{socket.gethostname()}-{a.port}", ip, a.port, {"model": model or ""}).start()
    run_server(a.host, a.port, pipeline=pipe)
    return 0


def _cmd_split(a) -> int:
    from .models.config import get_config
    from .parallel.placement import detect_gpus, split_model_into_blocks
    cfg = get_config(a.model)
    gpus = detect_gpus()[:a.gpus]
    devs = [f"cuda:{g.index}" for g in gpus] or [f"cpu:{i}" for i in range(a.gpus)]
    blocks = split_model_into_blocks(cfg, devs, strategy=a.strategy, gpus=gpus or None, profile=a.profile)
    _print({"model": a.model, "layers": cfg.num_layers,
            "blocks": [{"device": b.device, "layers": [b.start, b.end], "count": b.num_layers} for b in blocks]})
    return 0


def _cmd_hub(a) -> int:
    from .models.config import get_config
    out = {"model": a.model}
    p = a.model
    if os.path.isdir(p):
        files = os.listdir(p)
        out["files"] = sorted(files)[:50]
        fmt = "safetensors" if any(f.endswith(".safetensors") for f in files) else \
            "gguf" if any(f.endswith(".gguf") for f in files) else "unknown"
        cfgj = os.path.join(p, "config.json")
        if os.path.exists(cfgj):
            c = json.load(open(cfgj))
            qc = c.get("quantization_config", {}) or {}
            out["quantization"] = qc.get("quant_method") or qc.get("quant_algo")
            if "nvfp4" in json.dumps(qc).lower() or os.path.exists(os.path.join(p, "hf_quant_config.json")):
                fmt += "+nvfp4"
        out["format"] = fmt
    try:
        cfg = get_config(p)
        out["config"] = cfg.to_dict()
        out["params_b"] = round(cfg.num_params() / 1e9, 3)
        out["native_engine"] = True
    except (KeyError, ValueError) as e:      # unknown name, or an architecture the engine lacks
        out["error"] = str(e)
        out["native_engine"] = False
    _print(out)
    return 0


def main(argv: Optional[List[str]] = None) -> int:
    p = build_parser()
    a = p.parse_args(argv)
    cmd = a.command
    if cmd is None:
        p.print_help()
        return 0
    if cmd == "version":
        print(f"vramancer-b200 {__version__}")
        return 0
    if cmd == "run":
        return _cmd_run(a)
    if cmd == "serve":
        return _cmd_serve(a)
    if cmd == "generate":
        from .pipeline import InferencePipeline
        pipe = InferencePipeline().load(a.model, num_layers=a.num_layers)
        print(pipe.generate(a.prompt, max_new_tokens=a.max_tokens))
        pipe.shutdown()
        return 0
    if cmd == "status":
        from . import ops
        from .parallel.placement import auto_configure
        st = auto_configure()
        st["native_kernels"] = ops.native_available()
        _print(st)
        return 0
    if cmd == "benchmark":
        if a.workload:
            from . import workloads
            extra = [x for x in a.rest if x != "--"]
            workloads.main([a.workload] + (["--model", a.model] if a.model else []) + extra)
            return 0
        if a.model:
            from .pipeline import InferencePipeline
            pipe = InferencePipeline().load(a.model)
            _print(pipe.benchmark())
            pipe.shutdown()
        else:
            from .ops.microbench import bench_gemm
            _print(bench_gemm(a.size, a.size, a.size))
        return 0
    if cmd == "discover":
        from .cluster.discovery import ClusterDiscovery, known_nodes
        from .cluster.mdns import browse
        d = ClusterDiscovery()
        d.start()
        browse(timeout=min(2.0, a.timeout))      # mDNS / DNS-SD answers go into the same table
        time.sleep(max(0.0, a.timeout - 2.0))
        d.stop()
        _print(known_nodes())
        return 0
    if cmd == "split":
        return _cmd_split(a)
    if cmd == "dashboard":
        if a.cli:
            from .utils.monitor import GPUMonitor
            mon = GPUMonitor()
            try:
                while True:
                    _print(mon.poll())
                    time.sleep(2)
            except KeyboardInterrupt:
                return 0
        from .serving.api import run_server
        run_server("0.0.0.0", a.port)
        return 0
    if cmd == "quickstart":
        from .quickstart import run_quickstart
        rec = run_quickstart(a.use_case, run=a.run, serve=a.serve, prompt=a.prompt, port=a.port)
        _print(rec or {"error": "no catalog model fits the detected GPUs"})
        return int(rec.get("exit_code", 0)) if rec else 2
    if cmd == "hub":
        return _cmd_hub(a)
    if cmd == "health":
        from .utils.monitor import health_report
        _print(health_report())
        return 0
    if cmd == "doctor":
        from .utils.monitor import doctor
        _print(doctor())
        return 0
    if cmd == "history":
        import urllib.request
        try:
            with urllib.request.urlopen(f"{a.url}/api/history?limit={a.limit}", timeout=5) as r:
                print(r.read().decode())
        except Exception as e:
            print(f"no server at {a.url}: {e}")
            return 1
        return 0
    if cmd == "cluster":
        if a.action == "serve":
            from .cluster.router import ClusterRouter
            gpus = [int(x) for x in a.gpus.split(",")] if a.gpus else [0]
            router = ClusterRouter(a.model, gpus).start()
            _print(router.stats())
            return 0
        from .cluster.router import Gateway
        nodes = a.nodes.split(",") if a.nodes else []
        if a.discover:
            from .cluster.discovery import known_nodes
            nodes += [n["url"] for n in known_nodes()]
        gw = Gateway(nodes)
        _print(gw.check())
        return 0
    if cmd == "auth":
        tok = os.environ.get("VRM_API_TOKEN") if a.show else secrets.token_urlsafe(32)
        print(tok or "")
        return 0
    p.print_help()
    return 1


if __name__ == "__main__":
    sys.exit(main())
