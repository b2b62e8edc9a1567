"""Expert parallelism: host-side logic on the CPU (gloo, two ranks) and the
peer-memory kernels on CUDA (one rank in-process; two ranks when two GPUs are
visible)."""
import os
import socket
import subprocess
import sys

import pytest
import torch
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _ep_worker(rank, world, port, prompts, n_new, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world))
    import torch.distributed as dist

    from vramancer_b200.engine.engine import SamplingParams
    from vramancer_b200.llm import LLM
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        llm = LLM("tiny-moe", device="cpu", dtype=torch.float32, kv_cache_dtype="fp32", use_cuda_graph=False,
                  max_batch=4, max_model_len=128, kv_pages=64, seed=3, ep=True, max_prefill_tokens=24)
        assert llm.weights["layers.0.experts_gate_up_w"].shape[0] == 8 // world
        # ranks get different numbers of prompts: the one that finishes early keeps
        # running dummy steps until the other is done
        mine = prompts[rank::world]
        outs = llm.generate(mine, SamplingParams(max_tokens=n_new))
        q.put((rank, [o.output_ids for o in outs]))
    finally:
        dist.destroy_process_group()


def test_ep_generate_matches_single_process():
    from vramancer_b200.engine.engine import SamplingParams
    from vramancer_b200.llm import LLM
    g = torch.Generator().manual_seed(7)
    prompts = [torch.randint(0, 512, (n,), generator=g).tolist() for n in (5, 40, 17)]
    n_new = 6
    ref = LLM("tiny-moe", device="cpu", dtype=torch.float32, kv_cache_dtype="fp32", use_cuda_graph=False,
              max_batch=4, max_model_len=128, kv_pages=64, seed=3)
    want = [o.output_ids for o in ref.generate(prompts, SamplingParams(max_tokens=n_new))]
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_ep_worker, args=(r, 2, port, prompts, n_new, q)) for r in range(2)]
    for p in procs:
        p.start()
    got = dict(q.get(timeout=300) for _ in range(2))
    for p in procs:
        p.join(60)
        assert p.exitcode == 0
    assert got[0] == want[0::2] and got[1] == want[1::2]


def test_shard_experts_and_weights():
    from vramancer_b200.models.config import get_config
    from vramancer_b200.models.weights import random_weights
    from vramancer_b200.parallel.expert_parallel import shard_experts
    cfg = get_config("tiny-moe")
    full = random_weights(cfg, seed=1, layers=[0], embed=False, head=False)
    part = random_weights(cfg, seed=1, layers=[0], embed=False, head=False, ep_rank=1, ep_size=4)
    for n in ("experts_gate_up_w", "experts_down_w"):
        assert torch.equal(part[f"layers.0.{n}"], full[f"layers.0.{n}"][2:4])
        assert torch.equal(shard_experts(full[f"layers.0.{n}"], 1, 4), part[f"layers.0.{n}"])
    assert torch.equal(part["layers.0.router_w"], full["layers.0.router_w"])
    with pytest.raises(ValueError):
        shard_experts(full["layers.0.experts_down_w"], 0, 3)


# ----------------------------------------------------------------------------- CUDA
@pytest.mark.gpu
def test_ep_single_rank_matches_local_moe(cuda_errors_clean):
    """World 1: the whole peer-memory path (counts, dispatch to itself, owner plan,
    grouped GEMMs, return epilogue, combine) against the single-GPU MoE layer."""
    import torch.distributed as dist

    from vramancer_b200 import ops
    from vramancer_b200.models.config import get_config
    from vramancer_b200.parallel import moe
    from vramancer_b200.parallel.expert_parallel import ExpertParallel
    assert not dist.is_initialized()
    cfg = get_config("tiny-moe").with_(hidden_size=1024, num_experts=32, experts_per_token=4,
                                       expert_intermediate_size=256)
    ep = ExpertParallel(cfg, max_tokens=64, device="cuda:0")
    g = torch.Generator().manual_seed(1)
    bf = lambda t: t.to("cuda", torch.bfloat16)  # noqa: E731
    router = bf(torch.randn(32, 1024, generator=g) * 0.05)
    gu, dn = bf(torch.randn(32, 512, 1024, generator=g) * 0.03), bf(torch.randn(32, 1024, 256, generator=g) * 0.03)
    for T in (1, 7, 64, 33, 64):        # repeated calls alternate the buffer halves
        x = bf(torch.randn(T, 1024, generator=g) * 0.5)
        r0, nw = bf(torch.randn(T, 1024, generator=g)), bf(torch.rand(1024, generator=g) + 0.5)
        want = moe.moe_forward(cfg, x, router, gu, dn)
        got = ep.forward(x, router, gu, dn)
        torch.cuda.synchronize()
        assert torch.equal(got, want), (T, (got.float() - want.float()).abs().max().item())
        r1, r2 = r0.clone(), r0.clone()
        xn1 = moe.moe_forward(cfg, x, router, gu, dn, residual=r1, norm_w=nw)
        xn2 = ep.forward(x, router, gu, dn, residual=r2, norm_w=nw)
        assert torch.equal(r1, r2) and torch.equal(xn1, xn2)
    assert ops.read_and_clear_errors() == 0


@pytest.mark.gpu
def test_ep_two_gpus_matches_single_gpu():
    if torch.cuda.device_count() < 2:
        pytest.skip("needs two GPUs")
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", "--nproc-per-node=2",
           "--master-addr=127.0.0.1", f"--master-port={_port()}", "-m", "vramancer_b200.parallel.ep_bench",
           "--check", "--model", "tiny-moe-wide"]
    r = subprocess.run(["timeout", "-k", "30", "300"] + cmd, cwd=ROOT, env=env, capture_output=True, text=True)
    assert r.returncode == 0, r.stdout[-3000:] + r.stderr[-3000:]
    assert '"check": "ok"' in r.stdout
