"""Decode-step profiling driver (for ncu / CUDA-event breakdowns).

    python -m vramancer_b200.engine.profile --model qwen2.5-14b --batch 32 --steps 2

Builds the model with random weights, prefills `batch` prompts, then runs `steps`
eager decode steps (no CUDA graph, so every kernel is a separate launch) inside the
NVTX range "vrm_decode"; capture them with
    ncu --clock-control none --nvtx --nvtx-include "vrm_decode/" --metrics gpu__time_duration.sum ...
With --ablate it prints, per op type, how much of the graph-replayed decode step that
op costs on the critical path: the step is re-captured with the op replaced by a no-op
(its output buffer still allocated) and the CUDA-event step times are compared.  Unlike
a serialised ncu launch list this includes the overlap that programmatic dependent
launch gives between neighbouring kernels.  Ablated steps compute garbage; only their
timing is used.
"""
from __future__ import annotations

import argparse
import json

import torch


def _step_ms(runner, B: int, reps: int = 20) -> float:
    from ..parallel import comm
    comm.barrier()
    g = runner.capture(B)
    g.replay()
    torch.cuda.synchronize()
    best = float("inf")
    for _ in range(3):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(reps):
            g.replay()
        b.record()
        torch.cuda.synchronize()
        best = min(best, a.elapsed_time(b) / reps)
    runner._graphs.pop(B, None)
    del g
    return comm.max_over_ranks(best)


def ablate(llm, B: int) -> dict:
    """Step time with each op type removed (see module docstring)."""
    from .. import ops
    runner = llm.runner
    base = _step_ms(runner, B)

    def attn_stub(qkv, cache, layer, block_tables, context_lens, kv_scale, sm_scale, num_q_heads, **kw):
        D = llm.cfg.head_dim
        return torch.empty(qkv.shape[0], num_q_heads * D, dtype=qkv.dtype, device=qkv.device)

    def norm_stub(x, w, *args, residual=None, out=None, **kw):
        return x if out is None else out

    stubs = {
        "attention": {"paged_attention_decode": attn_stub},
        "rope_kv_write": {"rope_kv_write": lambda *a, **k: None},
        "norms": {"rmsnorm": norm_stub, "layernorm": norm_stub},
        "sampler": {"sample": lambda logits, *a, out=None, **k: out},
    }
    res = {"batch": B, "step_ms": round(base, 4)}
    tp = getattr(llm.model, "tp", None)
    if tp is not None:
        # the row-parallel all-reduces (fused push/reduce or NCCL) replaced by nothing
        saved_ar, saved_far = tp.all_reduce, tp.fused_ar
        tp.all_reduce, tp.fused_ar = (lambda x: x), None
        try:
            res["allreduce_ms"] = round(base - _step_ms(runner, B), 4)
        finally:
            tp.all_reduce, tp.fused_ar = saved_ar, saved_far
    for name, patch in stubs.items():
        saved = {k: getattr(ops, k) for k in patch}
        try:
            for k, fn in patch.items():
                setattr(ops, k, fn)
            t = _step_ms(runner, B)
        finally:
            for k, fn in saved.items():
                setattr(ops, k, fn)
        res[name + "_ms"] = round(base - t, 4)
    if llm.cfg.is_moe:
        from ..parallel import moe

        def moe_stub(cfg, x, router_w, gate_up, down, sgu, sdn, sg, residual, norm_w):
            # the whole device MoE block (router GEMM, routing, experts, combine) replaced
            # by the plain next-layer norm it would have fused
            if residual is None:
                return torch.empty_like(x)
            return ops.rmsnorm(residual, norm_w, cfg.norm_eps) if norm_w is not None else None

        def experts_stub(x, logits, *a, **k):
            # routing GEMM kept; routing, grouped GEMMs and combine replaced
            residual, norm_w = a[6], a[7]
            if residual is None:
                return torch.empty_like(x)
            return ops.rmsnorm(residual, norm_w, 1e-6) if norm_w is not None else torch.empty(0)

        saved = moe._moe_device
        try:
            moe._moe_device = moe_stub
            res["moe_block_ms"] = round(base - _step_ms(runner, B), 4)
        finally:
            moe._moe_device = saved
        real_native = ops.native

        class _Native:
            def __getattr__(self, k):
                return experts_stub if k == "moe_layer" else getattr(real_native(), k)

        try:
            ops.native = lambda: _Native()
            res["moe_route_experts_combine_ms"] = round(base - _step_ms(runner, B), 4)
        finally:
            ops.native = real_native
    return res


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen2.5-14b")
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--prompt-len", type=int, default=512)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--num-layers", type=int, default=None)
    ap.add_argument("--kv-dtype", default="bf16")
    ap.add_argument("--graph", action="store_true", help="replay the captured graph instead of eager steps")
    ap.add_argument("--ablate", action="store_true", help="critical-path cost of each op type (graph replay)")
    ap.add_argument("--shard-of", type=int, default=0,
                    help="one GPU runs rank 0's shard of a TP=N model without its peers (parallel/tp_emulate.py)")
    args = ap.parse_args(argv)
    if args.ablate:
        args.graph = True

    from ..engine.engine import SamplingParams
    from ..llm import LLM

    B, P = args.batch, args.prompt_len
    from ..parallel import comm
    info = comm.init_distributed()          # under torchrun: tensor parallelism over the ranks
    tp = comm.tp_context()
    if args.shard_of > 1 and info.world_size == 1:
        from ..parallel.tp_emulate import shard_context
        tp = shard_context(args.shard_of, f"cuda:{info.local_rank}")
    llm = LLM(args.model, device=f"cuda:{info.local_rank}", tp=tp, max_batch=B, max_model_len=P + args.steps + 64,
              kv_pages=(B + 1) * ((P + args.steps + 80) // 16 + 1) + 16, enable_prefix_cache=False,
              use_cuda_graph=args.graph, kv_cache_dtype=args.kv_dtype, num_layers=args.num_layers)
    g = torch.Generator().manual_seed(0)
    reqs = [llm.engine.add_request(torch.randint(0, llm.cfg.vocab_size, (P,), generator=g).tolist(),
                                   SamplingParams(max_tokens=args.steps + 4, ignore_eos=True)) for _ in range(B)]
    while any(not r.output_ids for r in reqs):
        llm.engine.step()
    llm.engine.step()              # warm decode (captures the graph when --graph)
    torch.cuda.synchronize()
    if args.ablate:
        res = ablate(llm, llm.runner.bucket_for(B))
        if info.rank == 0:
            print(json.dumps(res))
        llm.runner.release_graphs()
        comm.barrier()
        comm.destroy()
        return
    torch.cuda.nvtx.range_push("vrm_decode")
    for _ in range(args.steps):
        llm.engine.step()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    print(json.dumps({"ok": True, "batch": B, "steps": args.steps}))


if __name__ == "__main__":
    main()
