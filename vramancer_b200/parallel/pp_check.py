"""Pipeline x tensor parallelism correctness check: PP x TP greedy tokens against TP=1.

    torchrun --nproc-per-node 4 --master-addr 127.0.0.1 -m vramancer_b200.parallel.pp_check --pp 2 --tp 2

Every rank builds the single-device model (reference) and its own stage shard of the
PP x TP grid from the same seed, runs the same prompts through both (continuous
batching, paged KV, CUDA graphs on GPUs) and rank 0 reports whether the greedy
continuations agree, for prefill split into micro-batches and for decode with one and
with two micro-batches.  Works on CPU (gloo) and GPU (NCCL).
"""
from __future__ import annotations

import argparse
import json

import torch

from ..engine.engine import SamplingParams
from ..llm import LLM
from ..models.config import get_config
from ..models.weights import random_weights
from . import comm
from .pp import PPGrid


def run(model: str, pp: int, tp: int, n_new: int = 8, device: str = "auto", std: float = 0.05) -> dict:
    info = comm.init_distributed()
    use_cuda = torch.cuda.is_available() if device == "auto" else device == "cuda"
    dev = f"cuda:{info.local_rank}" if use_cuda else "cpu"
    dtype = torch.bfloat16 if use_cuda else torch.float32
    cfg = get_config(model)
    grid = PPGrid(pp, tp, num_layers=cfg.num_layers)
    tpc = comm.tp_context(grid.tp_group) if tp > 1 else None
    g = torch.Generator().manual_seed(7)
    prompts = [torch.randint(0, cfg.vocab_size, (n,), generator=g).tolist() for n in (5, 23, 40, 9)]
    kw = dict(device=dev, dtype=dtype, max_batch=4, max_model_len=128, kv_pages=64, use_cuda_graph=use_cuda,
              kv_cache_dtype="bf16" if use_cuda else "fp32")
    ref = LLM(cfg, weights=random_weights(cfg, device=dev, dtype=dtype, seed=11, std=std), **kw)
    want = [r.output_ids for r in ref.generate(prompts, SamplingParams(max_tokens=n_new))]
    first, last = grid.layers(cfg.num_layers)
    res = {"world": info.world_size, "pp": pp, "tp": tp, "stage_layers": [first, last], "device": dev}
    for dmb in (1, 2):
        w = random_weights(cfg, device=dev, dtype=dtype, seed=11, std=std, layers=range(first, last),
                           embed=grid.is_first, head=grid.is_last, tp_rank=grid.tp_rank, tp_size=tp)
        llm = LLM(cfg, weights=w, tp=tpc, pp_grid=grid, decode_microbatches=dmb, **kw)
        got = [r.output_ids for r in llm.generate(prompts, SamplingParams(max_tokens=n_new))]
        res[f"tokens_equal_decode_mb{dmb}"] = [a == b for a, b in zip(got, want)]
        res[f"hops_mb{dmb}"] = llm.model.hops
        comm.barrier()
        llm.runner.release_graphs()
    ref.runner.release_graphs()
    comm.barrier()
    return res


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="tiny-qwen2-d128")
    ap.add_argument("--pp", type=int, default=2)
    ap.add_argument("--tp", type=int, default=1)
    ap.add_argument("--device", default="auto")
    ap.add_argument("--n-new", type=int, default=8)
    a = ap.parse_args(argv)
    res = run(a.model, a.pp, a.tp, a.n_new, a.device)
    if comm.env_dist_info().rank == 0:
        print(json.dumps(res), flush=True)
    comm.destroy()


if __name__ == "__main__":
    main()
