"""Prefix-cache host tier: evicted prefix pages come back from pinned host memory (and
from NVMe through the hierarchical memory manager), with identical generations."""
import pytest
import torch

from vramancer_b200.engine.engine import SamplingParams
from vramancer_b200.kv.offload import KVOffloader
from vramancer_b200.kv.paged import PagedKVCacheManager


def _fill(pool, pages, val):
    for i, p in enumerate(pages):
        pool[p].fill_(val + i)


@pytest.mark.parametrize("spill", [False, True])
def test_evicted_prefix_pages_restore(tmp_path, spill):
    pool = torch.zeros(6, 2, 3, 16)
    hm = None
    if spill:
        from vramancer_b200.memory import HierarchicalMemoryManager
        hm = HierarchicalMemoryManager(str(tmp_path))
    off = KVOffloader([pool], max_pages=1 if spill else 8, hierarchy=hm)
    kv = PagedKVCacheManager(6, 16, enable_prefix_cache=True, offload=off)
    prompt = list(range(33))                       # two full pages + 1 token
    kv.allocate("a", 33, prompt)
    pages = kv.block_table("a")
    _fill(pool, pages, 10.0)
    kv.commit_prefix("a", prompt)
    kv.free("a")                                   # pages 0,1 cached (ref 0)
    kv.allocate("b", 16 * 6)                       # takes every page: both prefix pages evicted
    assert off.stats["offloaded"] == 2
    pool.zero_()
    kv.free("b")
    cached = kv.allocate("c", 33, prompt)
    assert cached == 32 and kv.stats_counters.get("offload_hits") == 2
    restored = kv.block_table("c")[:2]
    assert torch.all(pool[restored[0]] == 10.0) and torch.all(pool[restored[1]] == 11.0)
    if spill:
        assert off.stats["spilled"] >= 1 and off.stats["unspilled"] >= 1


def test_engine_generations_identical_with_offload():
    from vramancer_b200.llm import LLM
    kw = dict(device="cpu", dtype=torch.float32, kv_cache_dtype="fp32", use_cuda_graph=False, max_batch=2,
              max_model_len=96, kv_pages=12, seed=3)
    llm = LLM("tiny-qwen2", kv_offload_pages=16, **kw)
    g = torch.Generator().manual_seed(0)
    a = torch.randint(0, 200, (48,), generator=g).tolist()
    sp = SamplingParams(max_tokens=4)
    first = llm.generate([a], sp)[0].output_ids
    for i in range(3):                             # push a's pages out of the VRAM prefix cache
        llm.generate([torch.randint(0, 200, (80,), generator=g).tolist()], sp)
    again = llm.generate([a], sp)[0].output_ids
    assert again == first
    assert llm.offload.stats["restored"] >= 1
