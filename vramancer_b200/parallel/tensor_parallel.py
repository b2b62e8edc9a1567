"""Tensor parallelism from a single process: `apply_tensor_parallel(model, num_gpus)`.

The model runs one process per GPU (NCCL over NVLink, fused row-parallel all-reduce);
this module spawns those processes itself, so a plain Python program gets a TP=N model
without torchrun.  Rank 0 receives each call from the parent over a queue and
broadcasts it to the other ranks on a gloo control group; every rank then runs the
same `LLM.generate` in lockstep (identical scheduler decisions, so the collectives
line up) and rank 0 returns the result.  On a host without GPUs the workers use gloo
on the CPU.

Reference parity: core/tensor_parallel.py:452-600 (TPModel over a list of devices in
one process, generate_greedy without a KV cache; apply_tensor_parallel(model,
devices)).  Here each rank keeps its paged KV cache.
"""
from __future__ import annotations

import os
import queue
import socket
import traceback
from typing import Dict, List, Optional, Sequence

import torch
import torch.multiprocessing as mp


def _free_port() -> int:
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank: int, world: int, port: int, model, llm_kw: dict, device: str, cmd_q, res_q) -> None:
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), RANK=str(rank), WORLD_SIZE=str(world),
                      LOCAL_RANK=str(rank))
    try:
        import torch.distributed as dist

        from ..engine.engine import SamplingParams
        from ..llm import LLM
        from . import comm
        backend = "nccl" if device == "cuda" else "gloo"
        comm.init_distributed(backend=backend)
        ctrl = dist.new_group(backend="gloo")
        tp = comm.tp_context()
        dev = f"cuda:{rank}" if device == "cuda" else "cpu"
        kw = dict(llm_kw)
        if device != "cuda":
            kw.setdefault("dtype", torch.float32)
            kw.setdefault("kv_cache_dtype", "fp32")
            kw.setdefault("use_cuda_graph", False)
        llm = LLM(model, device=dev, tp=tp, **kw)
        if rank == 0:
            res_q.put(("ready", None))
        while True:
            box = [cmd_q.get() if rank == 0 else None]
            dist.broadcast_object_list(box, src=0, group=ctrl)
            cmd = box[0]
            if cmd[0] == "stop":
                break
            try:
                if cmd[0] == "generate":
                    prompts, params = cmd[1], cmd[2]
                    outs = llm.generate(prompts, SamplingParams(**params))
                    result = [o.output_ids for o in outs]
                else:
                    result = None
                if rank == 0:
                    res_q.put(("ok", result))
            except Exception:  # noqa: BLE001 - reported to the parent
                if rank == 0:
                    res_q.put(("error", traceback.format_exc()))
        if device == "cuda":
            llm.runner.release_graphs()
        comm.destroy()
    except Exception:  # noqa: BLE001
        if rank == 0:
            res_q.put(("error", traceback.format_exc()))
        raise


class TPModel:
    """Handle of a TP=N model running in N worker processes."""

    def __init__(self, model, num_gpus: int, *, device: Optional[str] = None, timeout_s: float = 600.0,
                 **llm_kw):
        if num_gpus < 1:
            raise ValueError("num_gpus must be >= 1")
        self.device = device or ("cuda" if torch.cuda.is_available() else "cpu")
        if self.device == "cuda" and torch.cuda.device_count() < num_gpus:
            raise ValueError(f"{num_gpus} GPUs requested, {torch.cuda.device_count()} visible")
        self.world = num_gpus
        self.timeout = timeout_s
        ctx = mp.get_context("spawn")
        self._cmd = ctx.Queue()
        self._res = ctx.Queue()
        port = _free_port()
        self._procs = [ctx.Process(target=_worker, args=(r, num_gpus, port, model, llm_kw, self.device,
                                                         self._cmd if r == 0 else None, self._res if r == 0 else None),
                                   daemon=True) for r in range(num_gpus)]
        for p in self._procs:
            p.start()
        self._expect("ready")

    def _expect(self, kind: str):
        try:
            tag, payload = self._res.get(timeout=self.timeout)
        except queue.Empty:
            self.shutdown(force=True)
            raise TimeoutError("tensor-parallel workers did not answer")
        if tag == "error":
            self.shutdown(force=True)
            raise RuntimeError("tensor-parallel worker failed:\n" + payload)
        return payload

    def generate(self, prompts: Sequence[Sequence[int]], max_tokens: int = 32, temperature: float = 0.0,
                 **params) -> List[List[int]]:
        """Token ids in -> generated token ids out (one list per prompt)."""
        p = dict(max_tokens=max_tokens, temperature=temperature, **params)
        self._cmd.put(("generate", [list(x) for x in prompts], p))
        return self._expect("ok")

    def generate_greedy(self, input_ids, max_new_tokens: int = 128) -> torch.Tensor:
        """[B, T] ids -> [B, T + max_new_tokens] (greedy), like the reference's TPModel."""
        ids = input_ids.tolist() if isinstance(input_ids, torch.Tensor) else [list(r) for r in input_ids]
        outs = self.generate(ids, max_tokens=max_new_tokens, temperature=0.0, ignore_eos=True)
        return torch.tensor([a + b for a, b in zip(ids, outs)])

    def shutdown(self, force: bool = False) -> None:
        if not force:
            try:
                self._cmd.put(("stop",))
            except Exception:  # noqa: BLE001
                pass
        for p in self._procs:
            p.join(timeout=30 if not force else 1)
            if p.is_alive():
                p.terminate()
                p.join(5)
        self._procs = []

    def __del__(self):
        if getattr(self, "_procs", None):
            self.shutdown()


def apply_tensor_parallel(model, devices: Optional[Sequence] = None, num_gpus: Optional[int] = None,
                          **llm_kw) -> TPModel:
    """TP over `devices` (or the first `num_gpus` GPUs; all visible by default).
    `model` is a preset name, a ModelConfig or a HF directory, as for LLM()."""
    n = len(devices) if devices is not None else (num_gpus or max(1, torch.cuda.device_count()))
    return TPModel(model, n, **llm_kw)
