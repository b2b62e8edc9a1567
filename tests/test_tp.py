"""Tensor parallelism: TP=2 must reproduce TP=1 (CPU gloo ranks; 2-GPU NCCL when available)."""
import json
import os
import socket
import subprocess
import sys

import pytest
import torch

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _torchrun(nproc, args, env_extra=None, timeout=600):
    env = dict(os.environ)
    env.update(env_extra or {})
    env["PYTHONPATH"] = ROOT + os.pathsep + env.get("PYTHONPATH", "")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}", "-m", "vramancer_b200.parallel.tp_check"] + args
    out = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=timeout, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-3000:]
    line = [l for l in out.stdout.splitlines() if l.startswith("{")][-1]
    return json.loads(line)


@pytest.mark.parametrize("model", ["tiny-qwen2", "tiny-gpt2", "tiny-qwen3"])
def test_tp2_matches_tp1_cpu_gloo(model):
    res = _torchrun(2, ["--model", model, "--device", "cpu"], {"CUDA_VISIBLE_DEVICES": ""})
    assert res["world"] == 2
    assert res["max_logit_diff"] < 1e-3 * max(1.0, res["scale"]), res
    assert all(res["tokens_equal"]), res


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_tp2_matches_tp1_gpu_nccl():
    res = _torchrun(2, ["--model", "tiny-qwen2-d128", "--device", "cuda"], {"NCCL_NVLS_ENABLE": "0"})
    assert res["world"] == 2
    # bf16 kernels: different reduction order across ranks -> small differences
    assert res["max_logit_diff"] < 0.05 * max(1.0, res["scale"]), res
    # fused GEMM + all-reduce matches GEMM followed by the NCCL all-reduce
    assert res["fused_ar_rel_diff"] is not None and res["fused_ar_rel_diff"] < 2e-2, res


def test_apply_tensor_parallel_single_process_api_cpu():
    """apply_tensor_parallel spawns its own ranks (gloo on CPU) and matches TP=1."""
    from vramancer_b200.engine.engine import SamplingParams
    from vramancer_b200.llm import LLM
    from vramancer_b200.parallel.tensor_parallel import apply_tensor_parallel
    kw = dict(max_batch=4, max_model_len=128, kv_pages=64)
    prompts = [[1, 2, 3, 4, 5], list(range(10, 40))]
    ref = LLM("tiny-qwen2", device="cpu", dtype=torch.float32, kv_cache_dtype="fp32", use_cuda_graph=False, **kw)
    want = [o.output_ids for o in ref.generate(prompts, SamplingParams(max_tokens=6))]
    tp = apply_tensor_parallel("tiny-qwen2", num_gpus=2, device="cpu", timeout_s=300, **kw)
    try:
        got = tp.generate(prompts, max_tokens=6)
        assert got == want
        full = tp.generate_greedy(torch.tensor([prompts[0]]), max_new_tokens=3)
        assert full.shape == (1, 8) and full[0, :5].tolist() == prompts[0]
    finally:
        tp.shutdown()
