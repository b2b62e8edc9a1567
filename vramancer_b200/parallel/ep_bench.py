"""Expert-parallel MoE decode benchmark and multi-GPU check.

    torchrun --nproc-per-node N --master-addr 127.0.0.1 -m vramancer_b200.parallel.ep_bench \\
        --model moe-48l-128e --batch 128 --steps 20

Each rank holds E/N experts and all other weights, runs batch/N sequences (prompt
--prompt-len random ids) and decodes them under CUDA graphs; the ranks exchange
routed rows over NVLink inside every MoE layer (parallel/expert_parallel.py).  The
decode step is timed on the device with CUDA events over --steps graph replays after
--warmup, max over ranks; rank 0 prints one JSON line with the aggregate tok/s.

--check instead compares one expert-parallel MoE layer against the single-GPU layer
(all experts local) on every rank's own tokens and prints {"check": "ok"}.

Reference parity: the reference has no expert parallelism (BASELINE config 5 is a
new measurement).
"""
from __future__ import annotations

import argparse
import json

import torch

from .. import ops
from . import comm


def check(model: str) -> None:
    from ..models.config import get_config
    from . import moe
    from .expert_parallel import ExpertParallel, shard_experts
    info = comm.init_distributed()
    dev = torch.device("cuda", info.local_rank)
    torch.cuda.set_device(dev)
    cfg = get_config(model)
    ep = ExpertParallel(cfg, max_tokens=256, device=dev)
    E, H, I = cfg.num_experts, cfg.hidden_size, cfg.expert_intermediate_size
    g = torch.Generator().manual_seed(11)          # same weights on every rank
    router = (torch.randn(E, H, generator=g) * 0.05).to(dev, torch.bfloat16)
    gu = (torch.randn(E, 2 * I, H, generator=g) * 0.03).to(dev, torch.bfloat16)
    dn = (torch.randn(E, H, I, generator=g) * 0.03).to(dev, torch.bfloat16)
    gul, dnl = shard_experts(gu, ep.rank, ep.world), shard_experts(dn, ep.rank, ep.world)
    gx = torch.Generator().manual_seed(100 + ep.rank)
    worst = 0.0
    for T in (5, 64, 1, 200, 37, 0, 128):        # different per call and per rank
        T = max(0, T - 3 * ep.rank) if T else 0
        x = (torch.randn(T, H, generator=gx) * 0.5).to(dev, torch.bfloat16)
        r0 = torch.randn(T, H, generator=gx).to(dev, torch.bfloat16)
        nw = (torch.rand(H, generator=gx) + 0.5).to(dev, torch.bfloat16)
        got = ep.forward(x, router, gul, dnl)
        r = r0.clone()
        xn = ep.forward(x, router, gul, dnl, residual=r, norm_w=nw)
        if T:
            want = moe.moe_forward(cfg, x, router, gu, dn)
            r_ref = r0.clone()
            xn_ref = moe.moe_forward(cfg, x, router, gu, dn, residual=r_ref, norm_w=nw)
            torch.cuda.synchronize()
            for a, b in ((got, want), (r, r_ref), (xn, xn_ref)):
                worst = max(worst, (a.float() - b.float()).abs().max().item())
    torch.cuda.synchronize()
    err = ops.read_and_clear_errors()
    worst = comm.max_over_ranks(worst)
    ok = worst == 0.0 and err == 0
    if ep.rank == 0:
        print(json.dumps({"check": "ok" if ok else "mismatch", "max_abs_diff": worst, "device_errors": err,
                          "world": ep.world}), flush=True)
    comm.barrier()
    comm.destroy()
    if not ok:
        raise SystemExit(1)


def bench(args) -> None:
    from ..engine.engine import SamplingParams
    from ..llm import LLM
    from .expert_parallel import ExpertParallel
    from ..models.config import get_config
    info = comm.init_distributed()
    dev = torch.device("cuda", info.local_rank)
    torch.cuda.set_device(dev)
    cfg = get_config(args.model)
    W = info.world_size
    Bl = max(1, args.batch // W)
    ep = ExpertParallel(cfg, max_tokens=max(Bl, args.max_tokens), device=dev)
    # requests decode while the others prefill (one chunk per lockstep step)
    max_len = args.prompt_len + Bl + args.steps + args.warmup + 64
    llm = LLM(args.model, device=str(dev), max_batch=Bl, max_model_len=max_len,
              kv_pages=(Bl + 2) * ((max_len + 15) // 16) + 64, enable_prefix_cache=False, seed=1234, ep=ep,
              max_prefill_tokens=args.max_tokens)
    eng, runner, sync = llm.engine, llm.runner, llm.engine.ep_sync
    g = torch.Generator().manual_seed(42 + ep.rank)
    reqs = [eng.add_request(torch.randint(0, cfg.vocab_size, (args.prompt_len,), generator=g).tolist(),
                            SamplingParams(max_tokens=max_len, ignore_eos=True))
            for _ in range(Bl)]
    while sync.any_rank(any(not r.output_ids for r in reqs)):
        eng.step()                                   # admission + prefill in lockstep
    ids = [r.output_ids[-1] for r in reqs]
    pos = [r.total_len - 1 for r in reqs]
    slots = [llm.kv.append_slots(r.request_id, 1)[0] for r in reqs]
    bts = [llm.kv.block_table(r.request_id) for r in reqs]
    B = runner.stage_decode_inputs(ids, pos, slots, [p + 1 for p in pos], bts, [0.0] * Bl, [0] * Bl, [1.0] * Bl,
                                   [1] * Bl)
    runner.upload_decode_inputs()
    graph = runner._graphs[B]
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    comm.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for _ in range(args.steps):
        graph.replay()
    e1.record()
    torch.cuda.synchronize()
    ms = comm.max_over_ranks(e0.elapsed_time(e1))
    err = ops.read_and_clear_errors()
    res = {"metric": "MoE decode tok/s, expert parallel", "model": args.model, "n_gpus": W,
           "parallelism": f"ep{W} + dp-attention", "global_batch": Bl * W, "per_rank_batch": Bl,
           "seq_len": args.prompt_len, "steps": args.steps, "warmup": args.warmup,
           "ms_per_step": round(ms / args.steps, 4), "value": round(Bl * W * args.steps / (ms / 1000.0), 2),
           "unit": "tok/s", "device_errors": err, "dtype": "bf16",
           "data": "synthetic ids, random-init N(0,0.02) weights; each step replays the same decode position"}
    runner.release_graphs()
    comm.barrier()
    if ep.rank == 0:
        print(json.dumps(res), flush=True)
    comm.destroy()


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="moe-48l-128e")
    ap.add_argument("--batch", type=int, default=128)
    ap.add_argument("--prompt-len", type=int, default=512)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--max-tokens", type=int, default=512, help="per-rank tokens per MoE call (prefill chunk)")
    ap.add_argument("--check", action="store_true")
    a = ap.parse_args(argv)
    if a.check:
        check(a.model)
    else:
        bench(a)


if __name__ == "__main__":
    main()
