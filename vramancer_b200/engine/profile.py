"""Decode-step profiling driver (for ncu / CUDA-event breakdowns).

    python -m vramancer_b200.engine.profile --model qwen2.5-14b --batch 32 --steps 2

Builds the model with random weights, prefills `batch` prompts, then runs `steps`
eager decode steps (no CUDA graph, so every kernel is a separate launch) inside the
NVTX range "vrm_decode"; capture them with
    ncu --nvtx --nvtx-include "vrm_decode/" --metrics gpu__time_duration.sum ...
With --events it instead prints a per-op CUDA-event breakdown of one step.
"""
from __future__ import annotations

import argparse
import json

import torch


def main(argv=None):
    ap = argparse.ArgumentParser()
    ap.add_argument("--model", default="qwen2.5-14b")
    ap.add_argument("--batch", type=int, default=32)
    ap.add_argument("--prompt-len", type=int, default=512)
    ap.add_argument("--steps", type=int, default=2)
    ap.add_argument("--num-layers", type=int, default=None)
    ap.add_argument("--kv-dtype", default="bf16")
    ap.add_argument("--graph", action="store_true", help="replay the captured graph instead of eager steps")
    args = ap.parse_args(argv)

    from ..engine.engine import SamplingParams
    from ..llm import LLM

    B, P = args.batch, args.prompt_len
    llm = LLM(args.model, device="cuda:0", max_batch=B, max_model_len=P + args.steps + 64,
              kv_pages=(B + 1) * ((P + args.steps + 80) // 16 + 1) + 16, enable_prefix_cache=False,
              use_cuda_graph=args.graph, kv_cache_dtype=args.kv_dtype, num_layers=args.num_layers)
    g = torch.Generator().manual_seed(0)
    reqs = [llm.engine.add_request(torch.randint(0, llm.cfg.vocab_size, (P,), generator=g).tolist(),
                                   SamplingParams(max_tokens=args.steps + 4, ignore_eos=True)) for _ in range(B)]
    while any(not r.output_ids for r in reqs):
        llm.engine.step()
    llm.engine.step()              # warm decode (captures the graph when --graph)
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_push("vrm_decode")
    for _ in range(args.steps):
        llm.engine.step()
    torch.cuda.synchronize()
    torch.cuda.nvtx.range_pop()
    print(json.dumps({"ok": True, "batch": B, "steps": args.steps}))


if __name__ == "__main__":
    main()
