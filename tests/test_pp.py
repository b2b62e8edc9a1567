"""Pipeline x tensor parallelism over processes (NCCL / gloo p2p between stages) must
reproduce the single-device model token for token."""
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


def _torchrun(nproc, args, env_extra=None, timeout=900):
    env = dict(os.environ)
    env.update(env_extra or {})
    env["PYTHONPATH"] = ROOT + os.pathsep + env.get("PYTHONPATH", "")
    cmd = [sys.executable, "-m", "torch.distributed.run", "--nnodes=1", f"--nproc-per-node={nproc}",
           "--master-addr=127.0.0.1", f"--master-port={_free_port()}", "-m", "vramancer_b200.parallel.pp_check"] + args
    out = subprocess.run(cmd, env=env, capture_output=True, text=True, timeout=timeout, cwd=ROOT)
    assert out.returncode == 0, out.stderr[-4000:]
    return json.loads([l for l in out.stdout.splitlines() if l.startswith("{")][-1])


def test_pp2_tp2_matches_single_device_cpu_gloo():
    res = _torchrun(4, ["--pp", "2", "--tp", "2", "--device", "cpu"], {"CUDA_VISIBLE_DEVICES": ""})
    assert res["world"] == 4 and res["stage_layers"] == [0, 1]
    assert all(res["tokens_equal_decode_mb1"]), res
    assert all(res["tokens_equal_decode_mb2"]), res
    assert res["hops_mb1"] == 0           # rank 0 is stage 0: it sends, it never receives


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_pp2_matches_single_device_gpu_nccl():
    res = _torchrun(2, ["--pp", "2", "--tp", "1", "--device", "cuda"], {"NCCL_NVLS_ENABLE": "0"})
    assert all(res["tokens_equal_decode_mb1"]), res
    assert all(res["tokens_equal_decode_mb2"]), res
