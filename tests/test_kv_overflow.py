"""KV pages borrowed from a lender GPU (kv/overflow.py): block-manager bookkeeping on
the CPU, and on GPUs a sequence larger than the local pool decoding token for token
like an unconstrained run (the lender is the same GPU on one device, the peer on two)."""
import pytest
import torch

from vramancer_b200.kv.paged import PagedKVCacheManager


class FakeLender:
    """Hands out page ids past the local pool, like ExtensiblePagePool.take_page."""

    def __init__(self, first, cap):
        self.first, self.cap = first, cap
        self.free = list(range(first, first + cap))
        self.returned = []

    def take(self, n=1):
        return self.free.pop(0) if self.free else None

    def give_back(self, p):
        self.returned.append(p)
        self.free.append(p)

    def capacity(self):
        return len(self.free)


def _mgr(local=4, borrow=8):
    lend = FakeLender(100, borrow)
    m = PagedKVCacheManager(local, page_size=16, enable_prefix_cache=False)
    m._overflow, m._release_borrowed, m._overflow_capacity = lend.take, lend.give_back, lend.capacity
    return m, lend


def test_overflow_admits_and_grows_past_the_local_pool():
    m, lend = _mgr()
    assert m.can_allocate(16 * 10)               # 4 local + 8 borrowable pages
    assert not m.can_allocate(16 * 13)
    m.allocate("a", 16 * 6)
    pages = m.block_table("a")
    assert len(pages) == 6 and sum(p >= 100 for p in pages) == 2
    for _ in range(16):
        m.append_slots("a", 1)
    assert sum(p >= 100 for p in m.block_table("a")) == 3
    m.free("a")
    assert sorted(lend.returned) == [100, 101, 102]


def test_relocate_borrowed_moves_pages_home():
    m, lend = _mgr()
    m.allocate("a", 16 * 3)
    m.allocate("b", 16 * 3)                       # b holds 1 local + 2 borrowed pages
    bt_b = m.block_table("b")
    borrowed = [p for p in bt_b if p >= 100]
    assert len(borrowed) == 2
    m.free("a")                                   # 3 local pages free again
    copies = []
    moved = m.relocate_borrowed(lambda s, d: copies.append((s, d)))
    assert moved == 2 and [s for s, _ in copies] == sorted(borrowed)
    assert all(p < 4 for p in m.block_table("b"))
    assert sorted(lend.returned) == sorted(borrowed)
    m.free("b")
    assert m.num_free_pages() == 4


def _generate(llm, prompt, n):
    from vramancer_b200.engine.engine import SamplingParams
    return llm.generate([prompt], SamplingParams(max_tokens=n, ignore_eos=True))[0].output_ids


def _check_lender(lender_dev):
    from vramancer_b200.llm import LLM
    from vramancer_b200.models.config import PRESETS
    from vramancer_b200.models.weights import random_weights
    cfg = PRESETS["tiny-qwen2-d128"]
    w = random_weights(cfg, device="cuda:0", dtype=torch.bfloat16, seed=3, std=0.05)
    g = torch.Generator().manual_seed(1)
    prompt = torch.randint(0, cfg.vocab_size, (300,), generator=g).tolist()
    kw = dict(device="cuda:0", max_batch=2, max_model_len=1024, enable_prefix_cache=False)
    want = _generate(LLM(cfg, weights=w, kv_pages=128, **kw), prompt, 200)
    # 8 local pages hold 128 tokens: the other ~24 pages of the 500-token sequence are borrowed
    small = LLM(cfg, weights=w, kv_pages=8, kv_lender=lender_dev, kv_borrow_pages=64, **kw)
    got = _generate(small, prompt, 200)
    st = small.pool.stats
    assert got == want
    assert st["chunks_mapped"] >= 1 and st["pages_borrowed"] >= 20, st
    assert st["chunks_unmapped"] == st["chunks_mapped"], st        # all memory went back at the end
    from vramancer_b200 import ops
    assert ops.read_and_clear_errors() == 0
    small.runner.release_graphs()
    small.pool.close()


@pytest.mark.gpu
def test_sequence_larger_than_the_local_pool_one_gpu():
    _check_lender(0)


@pytest.mark.gpu
@pytest.mark.skipif(not torch.cuda.is_available() or torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_sequence_larger_than_the_local_pool_borrows_from_the_peer():
    _check_lender(1)
