"""Row-parallel projection microbenchmark: GEMM + all-reduce + residual + norm at TP=N.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m vramancer_b200.parallel.ar_bench

For each shape (tokens M, hidden N, local K) it times, per call, inside CUDA graphs
with CUDA events and reports the max over ranks:
  local   GEMM + residual RMSNorm, no communication (lower bound)
  nccl    GEMM, NCCL all-reduce (bf16), residual RMSNorm
  fused   push GEMM (partials to every rank over NVLink) + reduce/residual/RMSNorm
  fused_one_kernel  the push GEMM whose own warps reduce into the residual and store
          the RMSNorm sums (the next GEMM normalises): one launch
  ar      the NCCL all-reduce alone
One JSON line per shape on rank 0.

Reference parity: the reference times its TP layer only end to end
(benchmarks/bench_tensor_parallel.py); this isolates the collective's cost.
"""
from __future__ import annotations

import argparse
import json

import torch
import torch.distributed as dist

from .. import ops
from . import comm


def _time_graph(fn, iters: int, reps: int = 5) -> float:
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(s)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    g.replay()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(reps):
        comm.barrier()
        torch.cuda.synchronize()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        g.replay()
        b.record()
        torch.cuda.synchronize()
        best = min(best, a.elapsed_time(b) * 1e3 / iters)
    del g
    return comm.max_over_ranks(best)


def run(shapes, iters: int = 48) -> list:
    info = comm.init_distributed()
    tp = comm.tp_context()
    assert tp is not None and tp.fused_ar is not None, "needs >= 2 CUDA ranks with the fused all-reduce enabled"
    dev = torch.device("cuda", info.local_rank)
    far = tp.fused_ar
    out = []
    for m, n, k in shapes:
        g = torch.Generator(device=dev).manual_seed(5 + tp.rank)
        x = torch.randn(m, k, device=dev, generator=g).to(torch.bfloat16)
        w = (torch.randn(n, k, device=dev, generator=g) * 0.02).to(torch.bfloat16)
        r = torch.randn(m, n, device=dev, generator=g).to(torch.bfloat16)
        nw = torch.ones(n, device=dev, dtype=torch.bfloat16)
        y = torch.empty(m, n, device=dev, dtype=torch.bfloat16)
        o = torch.empty(m, n, device=dev, dtype=torch.bfloat16)

        def local():
            ops.linear(x, w, out=y)
            ops.rmsnorm(y, nw, 1e-6, residual=r, out=o)

        def nccl():
            ops.linear(x, w, out=y)
            dist.all_reduce(y)
            ops.rmsnorm(y, nw, 1e-6, residual=r, out=o)

        def fused():
            far.push(x, w)
            far.reduce(m, n, residual=r, out=o, norm_w=nw, eps=1e-6)

        ssq = torch.zeros((n + 127) // 128, 128, device=dev)

        def fused1():
            # one kernel: GEMM + push + reduce into the residual + norm sums
            far.push_reduce(x, w, residual=r, ssq_out=ssq)

        def ar():
            dist.all_reduce(y)

        res = {"world": tp.size, "M": m, "N": n, "K": k}
        for name, fn in (("local", local), ("nccl", nccl), ("fused", fused), ("fused_one_kernel", fused1), ("ar", ar)):
            res[name + "_us"] = round(_time_graph(fn, iters), 2)
        out.append(res)
        if tp.rank == 0:
            print(json.dumps(res), flush=True)
    comm.barrier()
    return out


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--hidden", type=int, default=5120)
    ap.add_argument("--inter", type=int, default=13824)
    ap.add_argument("--tokens", type=int, nargs="+", default=[1, 32])
    ap.add_argument("--iters", type=int, default=48)
    a = ap.parse_args(argv)
    world = comm.env_dist_info().world_size
    shapes = []
    for m in a.tokens:
        shapes.append((m, a.hidden, a.hidden // world))    # o_proj
        shapes.append((m, a.hidden, a.inter // world))     # down_proj
    run(shapes, a.iters)
    comm.destroy()


if __name__ == "__main__":
    main()
