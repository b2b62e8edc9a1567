#!/usr/bin/env python
"""Headline benchmark: decode tok/s (bs1, bs32) + p50 TTFT, Qwen2.5-14B architecture,
bf16, random-init weights N(0, 0.02), synthetic token ids, paged KV (16-token pages),
CUDA-graph decode.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference]

N > 1 runs under torchrun (one process per GPU, NCCL) as tensor parallelism TP=N: the
same model and the same batch of 32 on N GPUs (strong scaling), every row-parallel
projection all-reduced inside its GEMM + norm kernels over NVLink.  The same job also
measures N data-parallel replicas of the full model (key "dp", global batch 32 x N,
weak scaling) and checks TP=N logits and greedy tokens against TP=1 on a small model
(key "tp_check").  --parallel dp makes the replicas the headline.  Rank 0 prints one
JSON line.

value   = aggregate decode tok/s at batch 32 (prompt 512), device-timed with CUDA
          events over exactly K decode steps (inputs staged on the device), max over
          ranks.  Each step streams all weights (~29.5 GB at TP=1), far more than
          the 126 MB L2, so no L2 flush is needed between steps.
e2e     = the same decode throughput through the engine API (LLMEngine.step): every
          step copies its inputs host->device from pinned memory and reads the
          sampled token ids back device->host before the host schedules the next.
bs1_*   = the same at batch 1; ttft_p50_ms = median time-to-first-token of a single
          512-token request through the engine (prefill + first token).
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
if ROOT not in sys.path:
    sys.path.insert(0, ROOT)

METRIC = "decode tok/s (bs1, bs32) + p50 TTFT, Qwen2.5-14B-arch bf16 @1/2/4/8 B200"
BASELINE_BS1_TOK_S = 5.41   # reference's published Qwen2.5-14B bf16 decode rate (2 consumer GPUs)


def parse_args(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=200)
    p.add_argument("--warmup", type=int, default=5)
    p.add_argument("--impl", choices=["ours", "reference"], default="ours")
    p.add_argument("--model", default="qwen2.5-14b")
    p.add_argument("--batch", type=int, default=32)
    p.add_argument("--prompt-len", type=int, default=512)
    p.add_argument("--kv-dtype", default="bf16")
    p.add_argument("--ttft-runs", type=int, default=5)
    p.add_argument("--num-layers", type=int, default=None, help="debug only: truncates the model (invalid run)")
    p.add_argument("--quantization", default=None, choices=["nvfp4", "fp8"],
                   help="weight format (the headline is bf16; these are extra measurements)")
    p.add_argument("--parallel", choices=["dp", "tp"], default="tp",
                   help="N > 1: headline at TP=N (default) or on N data-parallel replicas")
    p.add_argument("--shard-of", type=int, default=0,
                   help="debug only: one GPU runs rank 0's shard of a TP=N model without its peers (invalid run)")
    p.add_argument("--no-extras", action="store_true",
                   help="N > 1: skip the data-parallel figure and the TP numeric check")
    return p.parse_args(argv)


# ----------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi sampling of SM clock and throttle reasons during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.idx = gpu_index
        self.proc = None
        self.path = None

    def start(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--id={self.idx}", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except Exception:
            self.proc = None

    def stop(self) -> dict:
        if self.proc is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        rows = []
        with open(self.path) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) >= 9:
                    rows.append(parts)
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}

        def num(x):
            try:
                return float(x)
            except ValueError:
                return None

        power = [num(r[3]) or 0.0 for r in rows]
        pmax = max(power)
        loaded = [r for r, pw in zip(rows, power) if pw >= 0.5 * pmax] or rows
        sm = [num(r[1]) for r in loaded if num(r[1]) is not None]
        reasons = set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in loaded:
            for n, v in zip(names, r[5:9]):
                if v.strip().lower() in ("active", "1"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": num(loaded[0][2]),
                "reasons": sorted(reasons), "samples": len(loaded), "power_w_max": pmax}


# ----------------------------------------------------------------------------- ours
def run_ours(args):
    import torch

    from vramancer_b200 import ops
    from vramancer_b200.engine.engine import SamplingParams
    from vramancer_b200.llm import LLM
    from vramancer_b200.parallel import comm

    info = comm.init_distributed()
    rank, world = info.rank, info.world_size
    dev = torch.device("cuda", info.local_rank)
    torch.cuda.set_device(dev)
    mode = args.parallel if world > 1 else "tp"
    B, P = args.batch, args.prompt_len
    steps, warm = args.steps, args.warmup
    max_len = P + warm + steps + 64
    kv_pages = (B + 2) * ((max_len + 15) // 16) * 2 + 64

    def measure(tp, want_bs32=True, want_bs1=True, want_ttft=True, want_e2e=True, clocks=None):
        """Builds the model (TP=world when tp is given, else a full replica per rank)
        and measures the decode step on it; every rank runs the same calls."""
        llm = LLM(args.model, device=str(dev), kv_cache_dtype=args.kv_dtype, max_batch=B, max_model_len=max_len,
                  kv_pages=kv_pages, enable_prefix_cache=False, seed=1234, tp=tp, num_layers=args.num_layers,
                  quantization=args.quantization)
        runner, eng = llm.runner, llm.engine
        cfg = llm.cfg
        g = torch.Generator().manual_seed(42)

        def prompts(n):
            return [torch.randint(0, cfg.vocab_size, (P,), generator=g).tolist() for _ in range(n)]

        runner.capture_all([1, B])
        comm.barrier()
        res = {"cfg": cfg}

        # ------------------------------------------------------------ TTFT (engine API)
        if want_ttft:
            ttfts = []
            for _ in range(args.ttft_runs + 1):
                torch.cuda.synchronize()
                r = eng.add_request(prompts(1)[0], SamplingParams(max_tokens=1, ignore_eos=True))
                while not r.finished:
                    eng.step()
                ttfts.append(r.ttft * 1000.0)
            res["ttft_p50_ms"] = statistics.median(ttfts[1:])   # the first includes lazy initialisation

        # ------------------------------------------------------------ device-timed decode
        def device_decode(nb: int):
            """K decode steps of nb sequences with inputs pre-staged on the device;
            each step = D2D copy of its metadata + token feedback + graph replay."""
            reqs = [eng.add_request(p, SamplingParams(max_tokens=warm + steps + 2, ignore_eos=True))
                    for p in prompts(nb)]
            while any(not r.output_ids for r in reqs):
                eng.step()          # admission + prefill (+ first token)
            eng.flush()             # the engine's overlapped decode step, if one is in flight
            live = list(reqs)
            assert all(not r.finished for r in live)
            S = warm + steps
            bucket = runner.bucket_for(nb)
            rows_i, rows_f = [], []
            for t in range(S):
                ids, pos, slots, ctx = [], [], [], []
                for r in live:
                    p = r.total_len - 1 + t
                    slots.append(llm.kv.append_slots(r.request_id, 1)[0])
                    pos.append(p)
                    ctx.append(p + 1)
                    ids.append(0)
                bts = [llm.kv.block_table(r.request_id) for r in live]
                runner.stage_decode_inputs(ids, pos, slots, ctx, bts, [0.0] * nb, [0] * nb, [1.0] * nb,
                                           [t] * nb)
                rows_i.append(runner.h_i32.clone())
                rows_f.append(runner.h_f32.clone())
            d_pre_i = torch.stack(rows_i).to(dev)
            d_pre_f = torch.stack(rows_f).to(dev)
            first = torch.tensor([r.output_ids[-1] for r in live] + [0] * (bucket - nb), dtype=torch.int32)
            runner.d_out[:bucket].copy_(first.to(dev))
            graph = runner._graphs[bucket]

            def step(t):
                runner.d_i32.copy_(d_pre_i[t], non_blocking=True)
                runner.d_f32.copy_(d_pre_f[t], non_blocking=True)
                runner.d_ids[:bucket].copy_(runner.d_out[:bucket], non_blocking=True)
                graph.replay()

            if clocks is not None and nb == B:
                clocks.start()      # from the warm-up replays on: short timed regions still get samples
            for t in range(warm):
                step(t)
            torch.cuda.synchronize()
            comm.barrier()
            torch.cuda.synchronize()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            for t in range(warm, S):
                step(t)
            e1.record()
            torch.cuda.synchronize()
            if clocks is not None and nb == B:
                res["clocks"] = clocks.stop()
            comm.barrier()
            ms = e0.elapsed_time(e1)
            for r in live:
                eng.abort(r.request_id)
            return comm.max_over_ranks(ms)

        # ------------------------------------------------------------ e2e decode (engine API)
        def e2e_decode(nb: int):
            reqs = [eng.add_request(p, SamplingParams(max_tokens=warm + steps + 2, ignore_eos=True))
                    for p in prompts(nb)]
            while any(not r.output_ids for r in reqs):
                eng.step()
            for _ in range(warm):
                eng.step()
            torch.cuda.synchronize()
            comm.barrier()
            t0 = time.perf_counter()
            n0 = sum(len(r.output_ids) for r in reqs)
            for _ in range(steps):
                eng.step()
            torch.cuda.synchronize()
            t1 = time.perf_counter()
            comm.barrier()
            n1 = sum(len(r.output_ids) for r in reqs)
            for r in reqs:
                eng.abort(r.request_id)
            el = comm.max_over_ranks(t1 - t0)
            return (n1 - n0) / el, el

        ops.LAUNCHES[0] = 0
        if want_bs32:
            res["ms32"] = device_decode(B)
        if want_bs1:
            res["ms1"] = device_decode(1)
        if want_e2e:
            res["e2e32"], _ = e2e_decode(B)
        # launches per decode step: count one eager decode body of bucket B
        n0 = ops.LAUNCHES[0]
        runner._decode_body(runner.bucket_for(B))
        torch.cuda.synchronize()
        res["per_step"] = ops.LAUNCHES[0] - n0
        res["err"] = ops.read_and_clear_errors()
        res["h2d"] = runner.h2d_bytes_per_decode
        res["d2h"] = 4 * runner.bucket_for(B)
        runner.release_graphs()
        comm.barrier()
        del llm, runner, eng
        torch.cuda.synchronize()
        torch.cuda.empty_cache()
        return res

    sampler = ClockSampler(info.local_rank) if rank == 0 else None
    tp = comm.tp_context()
    if args.shard_of > 1 and world == 1:
        from vramancer_b200.parallel.tp_emulate import shard_context
        tp = shard_context(args.shard_of, str(dev))
    dpres = tpres = check = None
    if world == 1 or mode == "tp":
        main = measure(tp, clocks=sampler)
        lat = main
        if world > 1 and not args.no_extras:
            # the same GPUs as data-parallel replicas (a full model per GPU, batch B each)
            dpres = measure(None, want_bs1=False, want_ttft=False, want_e2e=False)
    else:
        # data parallel headline: a full replica per GPU, global batch B per replica (weak
        # scaling); then the same model as TP=world for the single-stream latency (bs1, TTFT)
        main = measure(None, want_bs1=False, want_ttft=False, clocks=sampler)
        lat = measure(tp, want_e2e=False)
        tpres = lat
    if world > 1 and not args.no_extras:
        check = tp_numeric_check()
    cfg = main["cfg"]
    dp = world > 1 and mode == "dp"
    replicas = world if dp else 1
    ms32, ms1 = main["ms32"], lat["ms1"]
    tok32 = replicas * B * steps / (ms32 / 1000.0)
    tok1 = steps / (ms1 / 1000.0)
    # with data parallelism every replica decodes its own batch through its own engine:
    # the aggregate is world x the rate over the slowest replica's time
    e2e = world * main["e2e32"] if dp else main["e2e32"]
    res = {
        "metric": METRIC,
        "value": round(tok32, 2),
        "unit": "tok/s",
        "n_gpus": world,
        "steps": steps,
        "warmup": warm,
        "ms_per_step": round(ms32 / steps, 4),
        "higher_is_better": True,
        "scaling": "weak" if dp else "strong",
        "vs_baseline": None,
        "dtype": "bf16" if not args.quantization else f"{args.quantization} weights, bf16 activations / KV",
        "data": "synthetic: uniform random token ids, random-init N(0,0.02) bf16 weights",
        "config": {"model": "Qwen2.5-14B architecture" if args.model == "qwen2.5-14b" else args.model,
                   "global_batch": B * replicas, "seq_len": P,
                   "parallelism": f"dp{world}" if dp else f"tp{world}",
                   "kv_cache": f"paged 16-token pages, {args.kv_dtype}",
                   "decode": "CUDA graph per step", "l2": "inputs larger than L2 (all weights streamed each step)",
                   "num_layers": args.num_layers or cfg.num_layers},
        "bs1": {"tok_s": round(tok1, 2), "ms_per_step": round(ms1 / steps, 4),
                "vs_baseline": round(tok1 / BASELINE_BS1_TOK_S, 2), "parallelism": f"tp{world}"},
        "ttft_p50_ms": round(lat["ttft_p50_ms"], 3),
        "ttft_prompt_tokens": P,
        "ttft_parallelism": f"tp{world}",
        "e2e": {"value": round(e2e, 2), "unit": "tok/s", "h2d_bytes_per_step": main["h2d"],
                "d2h_bytes_per_step": main["d2h"], "api": "LLMEngine.step"},
        "gpu_launches": main["per_step"] * steps,
        "gpu_launches_per_step": main["per_step"],
        "device_errors": main["err"] | (tpres["err"] if tpres else 0),
        "clocks": main.get("clocks", {}),
        "impl": "ours",
    }
    if tpres is not None:
        res["tp"] = {"parallelism": f"tp{world}", "global_batch": B, "value": round(B * steps / (tpres["ms32"] / 1000.0), 2),
                     "ms_per_step": round(tpres["ms32"] / steps, 4), "scaling": "strong"}
    if dpres is not None:
        res["dp"] = {"parallelism": f"dp{world}", "global_batch": B * world,
                     "value": round(world * B * steps / (dpres["ms32"] / 1000.0), 2),
                     "ms_per_step": round(dpres["ms32"] / steps, 4), "scaling": "weak"}
        res["device_errors"] |= dpres["err"]
    if check is not None:
        res["tp_check"] = check
    if args.num_layers:
        res["invalid"] = "truncated model (--num-layers): debugging only"
    if args.shard_of > 1 and world == 1:
        res["invalid"] = f"rank 0's shard of TP={args.shard_of} without its peers (--shard-of): debugging only"
    comm.barrier()
    if rank == 0:
        print(json.dumps(res), flush=True)
    comm.destroy()


def tp_numeric_check() -> dict:
    """TP=world vs TP=1 on a small Qwen2-shaped model (8 query / 8 KV heads of 128, bf16,
    CUDA graphs, the fused all-reduce):
    largest prefill logit difference relative to the logit scale, greedy tokens equal."""
    from vramancer_b200.parallel import tp_check
    r = tp_check.run("tiny-qwen2-tp8", n_new=8, device="cuda")
    return {"model": "tiny-qwen2-tp8", "max_logit_diff": round(r["max_logit_diff"], 5),
            "logit_scale": round(r["scale"], 4), "tokens_equal": r["tokens_equal"],
            "fused_ar_rel_diff": r["fused_ar_rel_diff"]}


# ----------------------------------------------------------------------------- reference arm
def run_reference(args):
    from baseline.reference_arm import run  # noqa: WPS433 (kept beside the product: baseline/)
    run(args, METRIC)


def main(argv=None):
    args = parse_args(argv)
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
