"""Serving workloads beyond the headline decode benchmark, on one GPU (or one TP group
under torchrun), all through the public `LLM` / `LLMEngine` API with random-init
weights and synthetic token ids.

    python -m vramancer_b200.workloads serve  [--requests 64 --min-prompt 128 --max-prompt 2048
                                               --output 256 --kv-dtype fp8]
    python -m vramancer_b200.workloads spec   [--quantization nvfp4 --ngram 3 --draft 8]
    python -m vramancer_b200.workloads prefill [--model moe-48l-128e --batch 8 --seq 4096]
    python -m vramancer_b200.workloads decode  [--quantization nvfp4 --batches 1,8,64 --prompt-len 1024]

serve   continuous batching of N requests arriving at once, prompt lengths uniform in
        [min, max], `output` tokens each (EOS ignored): output tok/s over the whole run
        (wall clock between device synchronisations: prefill, decode, scheduling and
        host<->device copies included), TTFT p50 / p99, mean batch per decode step.
spec-cost  verify-step time against draft length 1..8 under forced acceptance (drafts =
        the greedy continuation), and the speed-up it implies at acceptance 0.5..0.9.
spec    prompt-lookup speculative decoding: prompts made of a random 64-token span
        repeated 8 times; greedy decode with speculation off and on (n-gram 3, 8
        drafted tokens), tok/s of each, acceptance and token-for-token equality.
prefill batch x seq random-id prompts prefilled in one engine step (chunk budget =
        batch x seq): prompt tok/s, device-timed.
decode  decode tok/s at several batch sizes after a `prompt-len` prefill, CUDA events
        over `steps` graph-replayed decode steps (the headline method at other shapes).

Each prints one JSON line per measurement.  With torchrun the model runs tensor
parallel over the ranks (serve / decode; MoE models run expert parallel) and rank 0
prints.

Reference parity: benchmarks/bench_continuous_batching.py, benchmarks/
bench_prompt_lookup.py (results/phase7/T7.1_prompt_lookup.md), core/benchmark.py.
"""
from __future__ import annotations

import argparse
import json
import random
import statistics
import time
from contextlib import nullcontext
from typing import List, Optional

import torch


_PP_GRID = None


def _init(args=None):
    """Process group, device and the tensor-parallel context.  With --pp P under torchrun
    the ranks form a P x (world / P) pipeline x tensor-parallel grid (parallel/pp.py)."""
    global _PP_GRID
    from .parallel import comm
    info = comm.init_distributed()
    dev = torch.device("cuda", info.local_rank) if torch.cuda.is_available() else torch.device("cpu")
    if dev.type == "cuda":
        torch.cuda.set_device(dev)
    tp = None
    pp = getattr(args, "pp", 1) if args is not None else 1
    if info.world_size > 1 and pp > 1:
        from .models.config import get_config
        from .parallel.pp import PPGrid
        cfg = get_config(args.model)
        _PP_GRID = PPGrid(pp, info.world_size // pp, num_layers=args.num_layers or cfg.num_layers)
        tp = comm.tp_context(_PP_GRID.tp_group) if _PP_GRID.tp > 1 else None
    elif info.world_size > 1:
        tp = comm.tp_context()
    return info, dev, tp


def _layout(info) -> dict:
    if _PP_GRID is not None:
        return {"pp": _PP_GRID.pp, "tp": _PP_GRID.tp, "parallelism": f"pp{_PP_GRID.pp}xtp{_PP_GRID.tp}"}
    return {"pp": 1, "tp": info.world_size, "parallelism": f"tp{info.world_size}"}


def _sync(dev):
    if dev.type == "cuda":
        torch.cuda.synchronize(dev)


class _Timer:
    """Seconds between construction and stop(): CUDA events on the current stream
    (synchronised on both sides) on a GPU, the host clock otherwise."""

    def __init__(self, dev):
        self.dev = dev
        _sync(dev)
        if dev.type == "cuda":
            self.e0, self.e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            self.e0.record()
        else:
            self.t0 = time.perf_counter()

    def stop(self) -> float:
        if self.dev.type == "cuda":
            self.e1.record()
            _sync(self.dev)
            return self.e0.elapsed_time(self.e1) / 1e3
        return time.perf_counter() - self.t0


def _build(args, dev, tp, *, max_batch: int, max_len: int, kv_pages: Optional[int] = None, **kw):
    from .llm import LLM
    if _PP_GRID is not None:
        kw.setdefault("pp_grid", _PP_GRID)
    return LLM(args.model, device=str(dev), kv_cache_dtype=args.kv_dtype, max_batch=max_batch,
               max_model_len=max_len, kv_pages=kv_pages, quantization=args.quantization, tp=tp,
               num_layers=args.num_layers, **kw)


def _pct(xs: List[float], q: float) -> float:
    xs = sorted(xs)
    if not xs:
        return float("nan")
    i = min(len(xs) - 1, max(0, int(round(q * (len(xs) - 1)))))
    return xs[i]


def run_serve(args, info, dev, tp) -> dict:
    from .engine.engine import SamplingParams
    rng = random.Random(args.seed)
    lens = [rng.randint(args.min_prompt, args.max_prompt) for _ in range(args.requests)]
    max_len = args.max_prompt + args.output + 16
    llm = _build(args, dev, tp, max_batch=args.requests, max_len=max_len,
                 max_prefill_tokens=args.prefill_chunk)
    vocab = llm.cfg.vocab_size
    params = SamplingParams(max_tokens=args.output, ignore_eos=True)
    # warm-up: graph capture of every decode bucket the run will meet, one short request
    llm.warmup()
    llm.engine.generate([[rng.randrange(vocab) for _ in range(min(64, args.min_prompt))]],
                        SamplingParams(max_tokens=4, ignore_eos=True))
    prompts = [[rng.randrange(vocab) for _ in range(n)] for n in lens]
    eng = llm.engine
    s0 = dict(eng.stats)
    _sync(dev)
    t0 = time.perf_counter()
    reqs = [eng.add_request(p, params) for p in prompts]
    batch_hist = []
    while eng.has_unfinished():
        nrun = len(eng.running)
        eng.step()
        batch_hist.append(nrun)
    _sync(dev)
    wall = time.perf_counter() - t0
    from .parallel import comm
    wall = comm.max_over_ranks(wall)            # the slowest rank's time
    out_tok = sum(len(r.output_ids) for r in reqs)
    ttft = [r.ttft * 1e3 for r in reqs if r.ttft is not None]
    decode_steps = eng.stats["steps"] - s0["steps"]
    return {"workload": "serve", "model": args.model, "quantization": args.quantization or "bf16",
            "kv_dtype": args.kv_dtype, "requests": args.requests, "prompt_len": [args.min_prompt, args.max_prompt],
            "prompt_tokens": sum(lens), "output_tokens_each": args.output, "output_tokens": out_tok,
            "wall_s": round(wall, 3), "output_tok_s": round(out_tok / wall, 1),
            "total_tok_s": round((out_tok + sum(lens)) / wall, 1),
            "ttft_p50_ms": round(_pct(ttft, 0.5), 1), "ttft_p99_ms": round(_pct(ttft, 0.99), 1),
            "engine_steps": decode_steps, "mean_running": round(statistics.mean(batch_hist), 1) if batch_hist else 0,
            "preempted": eng.stats["preempted"] - s0["preempted"], **_layout(info),
            "timing": "wall clock between device synchronisations (engine API end to end), max over ranks",
            "data": "synthetic ids, random-init N(0,0.02) weights"}


def run_spec(args, info, dev, tp) -> dict:
    from .engine.engine import SamplingParams
    rng = random.Random(args.seed)
    span_len, reps = 64, 8
    out = {"workload": "spec", "model": args.model, "quantization": args.quantization or "bf16",
           "ngram": args.ngram, "num_draft": args.draft, "prompt": f"random {span_len}-token span x {reps}",
           "temperature": args.temperature, "top_k": args.top_k,
           "output_tokens": args.output, "batch": args.batch}
    results = {}
    ref_tokens = None
    for mode, nd in (("off", 0), ("on", args.draft)):
        llm = _build(args, dev, tp, max_batch=max(args.batch, 1), max_len=span_len * reps + args.output + 64,
                     spec_num_draft=nd, spec_ngram=args.ngram)
        vocab = llm.cfg.vocab_size
        r2 = random.Random(args.seed)
        prompts = []
        for _ in range(args.batch):
            span = [r2.randrange(vocab) for _ in range(span_len)]
            prompts.append(span * reps)
        params = SamplingParams(max_tokens=args.output, ignore_eos=True, temperature=args.temperature,
                                top_k=args.top_k)
        llm.warmup()
        llm.engine.generate([prompts[0][:128]], SamplingParams(max_tokens=16, ignore_eos=True))
        st0 = (llm.engine.spec_stats.proposed, llm.engine.spec_stats.accepted)
        _sync(dev)
        t0 = time.perf_counter()
        reqs = llm.engine.generate(prompts, params)
        _sync(dev)
        wall = time.perf_counter() - t0
        ttft = statistics.median([r.ttft for r in reqs if r.ttft is not None])
        dec_time = max(wall - ttft, 1e-9)
        toks = [list(r.output_ids) for r in reqs]
        res = {"wall_s": round(wall, 3), "decode_tok_s": round(args.batch * (args.output - 1) / dec_time, 1)}
        ss = llm.engine.spec_stats
        if nd > 0:
            drafted = ss.proposed - st0[0]
            accepted = ss.accepted - st0[1]
            res["drafted"] = drafted
            res["accepted"] = accepted
            res["acceptance"] = round(accepted / drafted, 3) if drafted else 0.0
        results[mode] = res
        if ref_tokens is None:
            ref_tokens = toks
        elif args.temperature <= 0:
            out["tokens_equal"] = toks == ref_tokens   # greedy only: sampled runs draw differently
        del llm
        torch.cuda.empty_cache() if dev.type == "cuda" else None
    out.update(results)
    out["speedup"] = round(results["on"]["decode_tok_s"] / results["off"]["decode_tok_s"], 3)
    out["timing"] = "wall clock between device synchronisations; decode = total minus TTFT"
    return out


def run_spec_cost(args, info, dev, tp) -> dict:
    """Verify-step cost against draft length under forced acceptance.

    For every draft length d the prompts decode with speculation whose drafts are d
    tokens of a plain greedy run's continuation (engine.draft_provider) and every draft
    is kept (engine.spec_force_accept): each step verifies d + 1 tokens per sequence and
    emits all of them.  The verify step costs the same whatever is accepted, so its
    measured time t(d) also holds at lower acceptance: with acceptance a per draft token
    a step yields (1 - a^(d+1)) / (1 - a) tokens per sequence, and the expected
    throughput at a is batch x that / t(d), against batch / t(0) for plain decode (d = 0:
    graph-replayed decode steps).  One untimed pass per d captures its CUDA graphs."""
    from .engine.engine import SamplingParams
    B, P, G = args.batch, args.prompt_len, args.output
    lens = [int(x) for x in args.draft_lens.split(",") if x.strip()]
    llm = _build(args, dev, tp, max_batch=B, max_len=P + G + 64, spec_num_draft=0, spec_ngram=args.ngram)
    vocab = llm.cfg.vocab_size
    r2 = random.Random(args.seed)
    prompts = [[r2.randrange(vocab) for _ in range(P)] for _ in range(B)]
    params = SamplingParams(max_tokens=G, ignore_eos=True)
    llm.warmup()
    eng = llm.engine
    ref = [list(r.output_ids) for r in eng.generate(prompts, params)]
    cont = {}
    rows = []
    eng.spec_force_accept = True

    def one_pass():
        reqs = [eng.add_request(p, params) for p in prompts]
        for r, c in zip(reqs, ref):
            cont[r.request_id] = c
        while any(not r.output_ids for r in reqs):          # prefill (and first token)
            eng.step()
        _sync(dev)
        t0 = time.perf_counter()
        n0 = sum(len(r.output_ids) for r in reqs)
        steps = 0
        while any(not r.finished for r in reqs):
            eng.step()
            steps += 1
        _sync(dev)
        return time.perf_counter() - t0, steps, sum(len(r.output_ids) for r in reqs) - n0

    for d in [0] + lens:
        eng.spec_num_draft = d
        eng.draft_provider = (lambda r, d=d: cont[r.request_id][len(r.output_ids):len(r.output_ids) + d]) if d else None
        one_pass()                                           # warm-up: graph captures
        st0 = (eng.spec_stats.proposed, eng.spec_stats.accepted)
        wall, steps, toks = one_pass()
        row = {"draft_len": d, "steps": steps, "ms_per_step": round(wall / max(steps, 1) * 1e3, 3),
               "tokens_per_step": round(toks / max(steps, 1), 2), "tok_s": round(toks / wall, 1)}
        if d:
            drafted = eng.spec_stats.proposed - st0[0]
            row["acceptance"] = round((eng.spec_stats.accepted - st0[1]) / max(drafted, 1), 3)
        rows.append(row)
    eng.draft_provider = None
    eng.spec_force_accept = False
    base = rows[0]["ms_per_step"]
    for row in rows[1:]:
        d, t = row["draft_len"], row["ms_per_step"]
        row["verify_cost_vs_decode"] = round(t / base, 3)
        row["speedup_at_acceptance"] = {str(a): round(((1 - a ** (d + 1)) / (1 - a)) * base / t, 3)
                                        for a in (0.5, 0.7, 0.8, 0.9)}
    return {"workload": "spec-cost", "model": args.model, "quantization": args.quantization or "bf16",
            "batch": B, "prompt_len": P, "output_tokens": G, "rows": rows,
            "timing": "wall clock between device synchronisations over the decode phase (engine API)",
            "data": "synthetic ids, random-init N(0,0.02) weights; drafts = the greedy continuation"}


def run_prefill(args, info, dev, tp) -> dict:
    from .engine.engine import SamplingParams
    rng = random.Random(args.seed)
    B, S = args.batch, args.seq
    llm = _build(args, dev, tp, max_batch=B, max_len=S + 32, max_prefill_tokens=B * S)
    vocab = llm.cfg.vocab_size
    params = SamplingParams(max_tokens=1, ignore_eos=True)
    times = []
    for it in range(args.warmup + args.iters):
        prompts = [[rng.randrange(vocab) for _ in range(S)] for _ in range(B)]
        reqs = [llm.engine.add_request(p, params) for p in prompts]
        tm = _Timer(dev)
        # NVTX range "vrm_prefill" around the measured steps: a launch list of one prefill
        # is `ncu --nvtx --nvtx-include "vrm_prefill/" --metrics gpu__time_duration.sum`
        rng_ctx = torch.cuda.nvtx.range("vrm_prefill") if (dev.type == "cuda" and it >= args.warmup) else nullcontext()
        with rng_ctx:
            llm.engine.step()          # one step: the whole batch in one prefill chunk
        dt = tm.stop()
        while llm.engine.has_unfinished():
            llm.engine.step()
        if it >= args.warmup:
            times.append(dt)
        assert all(r.finished for r in reqs)
    med = statistics.median(times)
    return {"workload": "prefill", "model": args.model, "quantization": args.quantization or "bf16",
            "batch": B, "seq": S, "ms": round(med * 1e3, 2), "prompt_tok_s": round(B * S / med, 1),
            "iters": args.iters, **_layout(info),
            "timing": "CUDA events around one engine step that prefills every prompt (first token sampled)",
            "data": "synthetic ids, random-init N(0,0.02) weights"}


def run_decode(args, info, dev, tp) -> List[dict]:
    from .engine.engine import SamplingParams
    rng = random.Random(args.seed)
    outs = []
    batches = [int(b) for b in args.batches.split(",")]
    P = args.prompt_len
    llm = _build(args, dev, tp, max_batch=max(batches), max_len=P + args.steps + args.warmup + 32)
    vocab = llm.cfg.vocab_size
    runner = llm.runner
    for B in batches:
        prompts = [[rng.randrange(vocab) for _ in range(P)] for _ in range(B)]
        params = SamplingParams(max_tokens=args.steps + args.warmup + 2, ignore_eos=True)
        reqs = [llm.engine.add_request(p, params) for p in prompts]
        while any(not r.prefill_done for r in reqs):
            llm.engine.step()
        for _ in range(args.warmup):
            llm.engine.step()
        tm = _Timer(dev)
        for _ in range(args.steps):
            llm.engine.step()
        ms = tm.stop() * 1e3 / args.steps
        while llm.engine.has_unfinished():
            llm.engine.step()
        outs.append({"workload": "decode", "model": args.model, "quantization": args.quantization or "bf16",
                     "kv_dtype": args.kv_dtype, "batch": B, "prompt_len": P, "ms_per_step": round(ms, 4),
                     "tok_s": round(B / ms * 1e3, 1), **_layout(info),
                     "graph": bool(getattr(runner, "use_graph", False)),
                     "timing": "CUDA events over engine steps (host scheduling and the per-step H2D/D2H included)"})
    return outs


def parse_args(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("what", choices=["serve", "spec", "spec-cost", "prefill", "decode"])
    ap.add_argument("--model", default="qwen2.5-14b")
    ap.add_argument("--quantization", default=None, choices=[None, "nvfp4", "fp8"])
    ap.add_argument("--kv-dtype", default="bf16")
    ap.add_argument("--num-layers", type=int, default=None, help="debug only: truncated model")
    ap.add_argument("--seed", type=int, default=0)
    ap.add_argument("--requests", type=int, default=64)
    ap.add_argument("--min-prompt", type=int, default=128)
    ap.add_argument("--max-prompt", type=int, default=2048)
    ap.add_argument("--output", type=int, default=256)
    ap.add_argument("--prefill-chunk", type=int, default=8192)
    ap.add_argument("--ngram", type=int, default=3)
    ap.add_argument("--draft", type=int, default=8)
    ap.add_argument("--temperature", type=float, default=0.0, help="spec: > 0 measures speculative sampling")
    ap.add_argument("--top-k", type=int, default=0)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--seq", type=int, default=4096)
    ap.add_argument("--batches", default="1,8,64")
    ap.add_argument("--draft-lens", default="1,2,4,8", help="spec-cost: draft lengths to time")
    ap.add_argument("--prompt-len", type=int, default=1024)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--iters", type=int, default=3)
    ap.add_argument("--pp", type=int, default=1, help="torchrun: pipeline stages (ranks = pp x tp)")
    return ap.parse_args(argv)


def main(argv=None) -> None:
    args = parse_args(argv)
    info, dev, tp = _init(args)
    fn = {"serve": run_serve, "spec": run_spec, "spec-cost": run_spec_cost, "prefill": run_prefill,
          "decode": run_decode}[args.what]
    res = fn(args, info, dev, tp)
    if info.rank == 0:
        for r in (res if isinstance(res, list) else [res]):
            print(json.dumps(r), flush=True)


if __name__ == "__main__":
    main()
