"""VRAM lending pool bookkeeping and KV page migration (CPU pools; GPU kernel when present)."""
import pytest
import torch

from vramancer_b200.kv.lending import KVPageLender, LendingPolicy, ReclaimUrgency, VRAMLendingPool
from vramancer_b200.kv.migration import migrate_pages
from vramancer_b200.kv.paged import PagedKVCacheManager
from vramancer_b200.kv.pool import KVPool, KVPoolSpec

GB = 2 ** 30


def _pool():
    p = VRAMLendingPool()
    p.register_gpu(0, 80 * GB, model_bytes=60 * GB)
    p.register_gpu(1, 180 * GB, model_bytes=30 * GB)
    p.register_gpu(2, 180 * GB, model_bytes=100 * GB)
    for d in (1, 2):
        p.preallocate(d, 1 << 20, torch.empty(1 << 20, dtype=torch.uint8))
    return p


def test_borrow_prefers_capacity_and_releases():
    p = _pool()
    lease = p.borrow(0, 64 << 10, "kv_overflow")
    assert lease is not None and lease.lender == 1          # more free memory
    t = p.allocate_on_lease(lease, (16, 1024), torch.bfloat16)
    src = torch.randn(16, 1024).bfloat16()
    p.transfer_into_lease(lease, src)
    assert torch.equal(p.transfer_from_lease(lease, "cpu"), src)
    assert p.budgets[1].lent == 64 << 10 and p.budgets[0].borrowed == 64 << 10
    p.release(lease.lease_id)
    assert p.budgets[1].lent == 0 and not p.leases


def test_buffer_extents_and_denial():
    p = _pool()
    leases = [p.borrow(0, 256 << 10) for _ in range(8)]
    assert sum(l is not None for l in leases) == 8           # 4 on each lender buffer
    assert p.borrow(0, 256 << 10) is None and p.stats["denied"] == 1
    for l in (leases[0], leases[2]):                        # adjacent extents of lender 1
        p.release(l.lease_id)
    assert p.borrow(0, 512 << 10) is not None               # freed extents coalesce


def test_reclaim_graceful_and_pressure():
    p = _pool()
    seen = []
    lease = p.borrow(0, 4096, on_reclaim=lambda l, u: seen.append((l.lease_id, u)))
    lender = lease.lender
    assert p.reclaim(lender, ReclaimUrgency.HIGH) == 1 and seen[0][1] == ReclaimUrgency.HIGH
    lease = p.borrow(0, 4096)
    p.budgets[lease.lender].kv_bytes = int(0.9 * p.budgets[lease.lender].total)
    urg = p.check_pressure()
    assert lease.lender in urg and not p.leases
    assert "cpu" in p.suggest_placement_budget(cpu_spill_gb=8)


def test_kv_page_swap_roundtrip_cpu():
    spec = KVPoolSpec(32, 2, 2, 64, dtype=torch.float32)
    local, remote = KVPool(spec), KVPool(spec)
    lm, rm = PagedKVCacheManager(32), PagedKVCacheManager(32)
    lm.allocate("s", 40)
    for p in lm.block_table("s"):
        local.cache[p].normal_()
    before = torch.stack([local.cache[p].clone() for p in lm.block_table("s")])
    lender = KVPageLender(local, lm, remote, rm)
    assert lender.swap_out("s") == 3 and not lm.has("s") and rm.stats()["used_pages"] == 3
    assert lender.swap_in("s") == 3
    after = torch.stack([local.cache[p] for p in lm.block_table("s")])
    assert torch.equal(before, after) and rm.stats()["used_pages"] == 0


@pytest.mark.gpu
def test_page_copy_kernel_same_and_peer_gpu():
    from vramancer_b200 import ops
    src = torch.randn(20, 2, 2, 4, 16, 128, device="cuda").bfloat16()
    dst = torch.zeros_like(src)
    migrate_pages(src, dst, [3, 7, 19], [0, 5, 2], "kernel")
    torch.cuda.synchronize()
    assert torch.equal(dst[0], src[3]) and torch.equal(dst[5], src[7]) and torch.equal(dst[2], src[19])
    assert dst[1].abs().sum() == 0
    if torch.cuda.device_count() >= 2:
        d1 = torch.zeros(20, 2, 2, 4, 16, 128, device="cuda:1", dtype=torch.bfloat16)
        migrate_pages(src, d1, list(range(10)), list(range(10, 20)), "kernel")
        torch.cuda.synchronize(0)
        torch.cuda.synchronize(1)
        assert torch.equal(d1[10:20].cpu(), src[:10].cpu())
    assert ops.read_and_clear_errors() == 0
