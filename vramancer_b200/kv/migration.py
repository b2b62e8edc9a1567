"""KV page migration between pools, and its benchmark (10 / 100 /
500 pages of 16 tok x 48 layers x 8 KV heads x 128 dim bf16 = 3 MiB each, GPU->GPU).

Methods
  kernel       the P2P page-copy kernel (csrc/migrate.cu): runs on the source GPU and
               stores into the peer pool over NVLink, one launch for all pages.
  memcpy_peer  one cudaMemcpyPeerAsync (copy engine) per page, for comparison.
  cpu_staged   device -> pinned host -> device, what the reference does on its PCIe box.

Reference parity: benchmarks/bench_kv_migration.py:8-117 (the three reference paths:
Rust GpuPipeline, Python CPU-staged, torch .to()).
"""
from __future__ import annotations

import json
import math
from typing import Dict, List, Sequence

import torch

from .. import ops

PAGE_SHAPE_14B = (48, 2, 8, 16, 128)   # layers, k/v, kv heads, tokens, head dim


def migrate_pages(src_pool: torch.Tensor, dst_pool: torch.Tensor, src_pages: Sequence[int],
                  dst_pages: Sequence[int], method: str = "kernel") -> None:
    """dst_pool[dst_pages[i]] <- src_pool[src_pages[i]] (pools [pages, ...], same page shape)."""
    if len(src_pages) != len(dst_pages):
        raise ValueError("page lists differ in length")
    if not len(src_pages):
        return
    if not src_pool.is_cuda or not dst_pool.is_cuda:
        si = torch.as_tensor(list(src_pages), dtype=torch.long)
        di = torch.as_tensor(list(dst_pages), dtype=torch.long)
        dst_pool[di.to(dst_pool.device)] = src_pool[si.to(src_pool.device)].to(dst_pool.device)
        return
    if method == "kernel":
        si = torch.as_tensor(list(src_pages), dtype=torch.int32, device=src_pool.device)
        di = torch.as_tensor(list(dst_pages), dtype=torch.int32, device=src_pool.device)
        with torch.cuda.device(src_pool.device):
            ops.native().page_copy(src_pool.view(src_pool.shape[0], -1).view(torch.uint8)
                                   if src_pool.dtype != torch.uint8 else src_pool,
                                   dst_pool.view(dst_pool.shape[0], -1).view(torch.uint8)
                                   if dst_pool.dtype != torch.uint8 else dst_pool, si, di)
    elif method == "memcpy_peer":
        with torch.cuda.device(src_pool.device):
            for s, d in zip(src_pages, dst_pages):
                dst_pool[d].copy_(src_pool[s], non_blocking=True)
    elif method == "cpu_staged":
        host = torch.empty((len(src_pages),) + tuple(src_pool.shape[1:]), dtype=src_pool.dtype, pin_memory=True)
        idx = torch.as_tensor(list(src_pages), dtype=torch.long, device=src_pool.device)
        host.copy_(src_pool.index_select(0, idx), non_blocking=True)
        torch.cuda.synchronize(src_pool.device)
        di = torch.as_tensor(list(dst_pages), dtype=torch.long, device=dst_pool.device)
        dst_pool.index_copy_(0, di, host.to(dst_pool.device, non_blocking=True))
    else:
        raise ValueError(f"unknown method {method!r}")


def bench_migration(counts=(10, 100, 500), src_dev: int = 0, dst_dev: int = 1, iters: int = 10,
                    methods=("kernel", "memcpy_peer", "cpu_staged")) -> List[Dict]:
    """Device-timed GPU->GPU page migration; timed on the source stream with events,
    after warm-up; both devices synchronised around each timed region."""
    n_max = max(counts)
    src = torch.randn((n_max + 8,) + PAGE_SHAPE_14B, device=f"cuda:{src_dev}").to(torch.bfloat16)
    dst = torch.zeros((n_max + 8,) + PAGE_SHAPE_14B, device=f"cuda:{dst_dev}", dtype=torch.bfloat16)
    page_bytes = math.prod(PAGE_SHAPE_14B) * 2
    if src_dev != dst_dev:
        ops.native().enable_peer_access(src_dev, dst_dev)
        ops.native().enable_peer_access(dst_dev, src_dev)
    out = []
    g = torch.Generator().manual_seed(0)
    for method in methods:
        for n in counts:
            sp = torch.randperm(n_max + 8, generator=g)[:n].tolist()
            dp = torch.randperm(n_max + 8, generator=g)[:n].tolist()
            for _ in range(2):
                migrate_pages(src, dst, sp, dp, method)
            torch.cuda.synchronize(src_dev)
            torch.cuda.synchronize(dst_dev)
            import time
            t0 = time.perf_counter()
            with torch.cuda.device(src_dev):
                e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                e0.record()
                for _ in range(iters):
                    migrate_pages(src, dst, sp, dp, method)
                e1.record()
            torch.cuda.synchronize(src_dev)
            torch.cuda.synchronize(dst_dev)
            wall_ms = (time.perf_counter() - t0) * 1000 / iters
            # device time on the source stream covers the kernel and the peer copies;
            # the CPU-staged path also waits on the host, so it is reported by wall clock
            ms = e0.elapsed_time(e1) / iters if method != "cpu_staged" else wall_ms
            ok = bool(torch.equal(dst[dp[0]].cpu(), src[sp[0]].cpu()))
            out.append({"method": method, "pages": n, "ms": round(ms, 4), "wall_ms": round(wall_ms, 4),
                        "gb_s": round(n * page_bytes / ms / 1e6, 1),
                        "page_mib": page_bytes / 2 ** 20, "correct": ok})
    return out


if __name__ == "__main__":
    for r in bench_migration():
        print(json.dumps(r))
