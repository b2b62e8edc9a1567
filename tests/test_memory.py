"""Hierarchical memory (tiers, heat, eviction, spill, prefetch, parity heal, remote
tier, state), compressor, parity manager: CPU."""
import os

import pytest
import torch

from vramancer_b200.memory import Compressor, HierarchicalMemoryManager, MemoryBlock, ParityKVManager, Tier
from vramancer_b200.memory.hierarchy import BlockServer


def _blk(i, n=1024):
    return MemoryBlock(f"b{i}", (n,), torch.float32), torch.randn(n)


def test_tier_round_trip_through_every_local_tier(tmp_path):
    hm = HierarchicalMemoryManager(str(tmp_path), codec="zlib")
    b, t = _blk(0)
    hm.register_block(b, Tier.L1, t)
    for tier in (Tier.L4, Tier.L5, Tier.L6, Tier.L7, Tier.L4, Tier.L1):
        hm.migrate(b, tier)
        assert hm.get_tier("b0") == tier
        assert torch.equal(hm._fetch(b).cpu(), t), tier
    s = hm.summary()
    assert s["migrations"] == 6 and s["spilled_bytes"] > 0


def test_eviction_moves_coldest_first_and_respects_pins(tmp_path):
    hm = HierarchicalMemoryManager(str(tmp_path), vram_budget_bytes=3 * 4096, dram_budget_bytes=1 * 4096,
                                   max_nvme_mb=1)
    blocks = []
    for i in range(5):
        b, t = _blk(i)
        hm.register_block(b, Tier.L1, t)
        blocks.append(b)
    blocks[0].pinned = True
    for _ in range(5):
        hm.touch(blocks[4])           # hot (promotes nothing: already L1)
    moved = hm.eviction_cycle(target_free_pct=0.0)
    assert moved >= 2
    assert hm.get_tier("b0") == Tier.L1 and hm.get_tier("b4") == Tier.L1
    assert hm.tier_bytes(Tier.L1) <= 3 * 4096
    assert hm.tier_bytes(Tier.L4) <= 4096             # DRAM overflow went to NVMe
    assert any(hm.get_tier(f"b{i}") == Tier.L5 for i in range(1, 4))


def test_heat_promotes_on_access(tmp_path):
    hm = HierarchicalMemoryManager(str(tmp_path), promote_heat=2.5)
    b, t = _blk(1)
    hm.register_block(b, Tier.L5, t)
    hm.get("b1")
    hm.get("b1")
    assert hm.get_tier("b1") == Tier.L5
    hm.get("b1")                                      # heat >= 2.5: NVMe -> DRAM
    assert hm.get_tier("b1") == Tier.L4
    assert torch.equal(hm.get("b1"), t)


def test_prefetch_and_state_reload(tmp_path):
    hm = HierarchicalMemoryManager(str(tmp_path))
    ts = {}
    for i in range(3):
        b, t = _blk(i, 333)
        ts[b.id] = t
        hm.register_block(b, Tier.L5, t)
    assert hm.schedule_prefetch(["b0", "b2"]) == 2
    assert hm.complete_prefetch() == 2
    assert hm.get_tier("b0") == Tier.L4 and hm.get_tier("b1") == Tier.L5
    st = str(tmp_path / "state.json")
    hm.save_state(st)
    hm2 = HierarchicalMemoryManager(str(tmp_path))
    assert hm2.load_state(st) == 1
    assert torch.equal(hm2._fetch(hm2.blocks["b1"]), ts["b1"])


def test_parity_heals_a_lost_spill_file(tmp_path):
    hm = HierarchicalMemoryManager(str(tmp_path), parity_group=3)
    ts = {}
    for i in range(3):
        b, t = _blk(i, 512)
        ts[b.id] = t
        hm.register_block(b, Tier.L1, t)
        hm.spill_to_nvme(b)
    assert hm.blocks["b1"].meta.get("parity_group")
    os.unlink(hm._data["b1"])
    assert hm.heal("b1")
    assert torch.equal(hm.load_from_nvme(hm.blocks["b1"]), ts["b1"])


def test_remote_ram_tier_over_tcp(tmp_path):
    srv = BlockServer(key=b"k")
    try:
        hm = HierarchicalMemoryManager(str(tmp_path), remote=srv.address, remote_key=b"k")
        b, t = _blk(7, 100)
        hm.register_block(b, Tier.L1, t)
        hm.migrate(b, Tier.L3)
        assert "b7" in srv.store
        hm.migrate(b, Tier.L1)
        assert torch.equal(hm._fetch(b), t)
    finally:
        srv.close()


def test_compressor_and_int_quantisation():
    c = Compressor("zlib")
    t = torch.zeros(4096)
    d = c.compress_tensor(t)
    assert len(d["data"]) < 1000 and torch.equal(c.decompress_tensor(d), t)
    w = torch.randn(64, 256)
    p, s, z = Compressor.quantize_weights_int4(w, group=128)
    wd = Compressor.dequantize_int4(p, s, z, group=128, dtype=torch.float32)
    assert (wd - w).abs().max() <= s.max() * 0.51 + 1e-6
    q, sc = Compressor.quantize_dynamic_int8(w)
    assert (Compressor.dequantize_int8(q, sc, torch.float32) - w).abs().max() <= sc.max() * 0.51


def test_parity_manager_checksum_guard():
    pm = ParityKVManager(group_size=2)
    a, b = os.urandom(64), os.urandom(64)
    pm.encode("g", [a, b])
    assert pm.heal("g", 0, [None, b]) == a
    with pytest.raises(RuntimeError):
        pm.heal("g", 0, [None, os.urandom(64)])       # wrong sibling: checksum fails
    assert pm.heal_engram("g", 1, [a, None]) == b
