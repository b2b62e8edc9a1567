"""Tensor-parallel correctness check: TP=N logits and greedy tokens against TP=1.

    torchrun --nproc-per-node 2 --master-addr 127.0.0.1 -m vramancer_b200.parallel.tp_check --model tiny-qwen2-d128

Every rank builds the TP=1 model (reference) and its own shard from the same seed,
runs the same prompts through both, and rank 0 reports the largest logit difference
and whether greedy continuations agree.  Works on CPU (gloo) and GPU (NCCL).

Reference parity: the reference's TP test sums 3 + 5 on two GPUs
(tests/test_cuda_tp.py:201-208) and never compares TP logits to a single device.
"""
from __future__ import annotations

import argparse
import json
import sys

import torch

from ..engine.engine import SamplingParams
from ..llm import LLM
from ..models.config import get_config
from ..models.weights import random_weights
from . import comm


def run(model: str, n_new: int = 8, device: str = "auto", std: float = 0.05) -> dict:
    info = comm.init_distributed()
    use_cuda = torch.cuda.is_available() if device == "auto" else device == "cuda"
    dev = f"cuda:{info.local_rank}" if use_cuda else "cpu"
    dtype = torch.bfloat16 if use_cuda else torch.float32
    cfg = get_config(model)
    tp = comm.tp_context()
    g = torch.Generator().manual_seed(7)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 23, 40)]
    kw = dict(device=dev, dtype=dtype, max_batch=4, max_model_len=128, kv_pages=64, use_cuda_graph=use_cuda,
              kv_cache_dtype="bf16" if use_cuda else "fp32")
    w_full = random_weights(cfg, device=dev, dtype=dtype, seed=11, std=std)
    ref = LLM(cfg, weights=w_full, **kw)
    w_tp = random_weights(cfg, device=dev, dtype=dtype, seed=11, std=std, tp_rank=tp.rank if tp else 0,
                          tp_size=tp.size if tp else 1)
    sharded = LLM(cfg, weights=w_tp, tp=tp, **kw)
    r_ref = ref.generate(prompts, SamplingParams(max_tokens=n_new))
    r_tp = sharded.generate(prompts, SamplingParams(max_tokens=n_new))
    # logits of the first prompt (prefill) through both
    from ..engine.runner import PrefillItem
    items = []
    for llm in (ref, sharded):
        rid = "probe"
        llm.kv.allocate(rid, len(prompts[1]))
        it = PrefillItem(prompts[1], 0, llm.kv.slots_for(rid, 0, len(prompts[1])), llm.kv.block_table(rid),
                         len(prompts[1]), True)
        items.append(llm.runner.prefill_logits([it])[-1].float().cpu())
        llm.kv.free(rid)
    diff = float((items[0] - items[1]).abs().max())
    fused_diff = None
    if tp is not None and tp.fused_ar is not None:
        # fused GEMM + all-reduce vs GEMM then NCCL all-reduce, several shapes
        from .. import ops
        gg = torch.Generator(device=dev).manual_seed(3 + tp.rank)
        fused_diff = 0.0
        for m, n, k in ((1, 512, 256), (7, 1024, 512), (32, 640, 1280), (100, 256, 384)):
            x = torch.randn(m, k, device=dev, generator=gg).to(dtype)
            w = (torch.randn(n, k, device=dev, generator=gg) * 0.05).to(dtype)
            r = torch.randn(m, n, device=dev, generator=gg).to(dtype)
            bias = torch.randn(n, device=dev, generator=gg).to(dtype)
            nw = (1 + 0.1 * torch.randn(n, device=dev, generator=gg)).to(dtype)
            ref_y = ops.linear(x, w).float()
            torch.distributed.all_reduce(ref_y)
            ref_s = ref_y + bias.float() + r.float()
            ref_n = ref_s * torch.rsqrt(ref_s.pow(2).mean(-1, keepdim=True) + 1e-6) * nw.float()
            for _ in range(3):     # repeated calls exercise the alternating buffers / epochs
                y = tp.fused_ar.linear(x, w, bias, residual=r)
            fused_diff = max(fused_diff, float((y.float() - ref_s).abs().max() / (ref_s.abs().max() + 1e-6)))
            # push + reduce fused with the residual update and RMSNorm
            res = r.clone()
            out = torch.empty_like(r)
            tp.fused_ar.push(x, w)
            tp.fused_ar.reduce(m, n, bias=bias, residual=res, out=out, norm_w=nw, eps=1e-6)
            fused_diff = max(fused_diff, float((res.float() - ref_s).abs().max() / (ref_s.abs().max() + 1e-6)),
                             float((out.float() - ref_n).abs().max() / (ref_n.abs().max() + 1e-6)))
        torch.cuda.synchronize()
    same = [a.output_ids == b.output_ids for a, b in zip(r_ref, r_tp)]
    res = {"world": info.world_size, "max_logit_diff": diff, "scale": float(items[0].abs().max()),
           "tokens_equal": same, "device": dev, "fused_ar_rel_diff": fused_diff}
    comm.barrier()
    ref.runner.release_graphs()
    sharded.runner.release_graphs()
    return res


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny-qwen2-d128")
    ap.add_argument("--device", default="auto")
    ap.add_argument("--n-new", type=int, default=8)
    a = ap.parse_args(argv)
    res = run(a.model, a.n_new, a.device)
    if comm.env_dist_info().rank == 0:
        print(json.dumps(res), flush=True)
    comm.destroy()


if __name__ == "__main__":
    main()
