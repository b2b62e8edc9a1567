"""Block placement strategies, link-health weighting and model placement on CPU."""
import pytest

from vramancer_b200.models.config import PRESETS
from vramancer_b200.parallel.placement_engine import Connectome, DeviceState, PlacementEngine


def _devs():
    return [DeviceState(0, "B200", 180e3, 100e3, 2250), DeviceState(1, "B200", 180e3, 150e3, 2250),
            DeviceState(2, "H100", 80e3, 70e3, 989)]


def test_strategies_and_tiers():
    eng = PlacementEngine(_devs(), host_budget_mb=1000)
    assert eng.place({"size_mb": 1000}, "vram")["gpu_id"] == 1                 # most free memory
    assert eng.place({"size_mb": 1000}, "profiled")["gpu_id"] == 1              # speed x free
    b = PlacementEngine(_devs())
    ids = [b.place({"size_mb": 10}, "balanced")["gpu_id"] for _ in range(6)]
    assert sorted(ids) == [0, 0, 1, 1, 2, 2]                                     # round-robin by load
    big = eng.place({"size_mb": 500e3})
    assert big["level"] == "nvme" and big["gpu_id"] == -1
    small_host = eng.place({"size_mb": 200e3})
    assert small_host["level"] == "nvme"
    eng2 = PlacementEngine(_devs(), host_budget_mb=300e3)
    assert eng2.place({"size_mb": 200e3})["level"] == "cpu"
    # memory is charged
    e3 = PlacementEngine([DeviceState(0, "B200", 10, 10, 1.0)])
    assert e3.place({"size_mb": 8})["level"] == "gpu"
    assert e3.place({"size_mb": 8})["level"] == "cpu"


def test_custom_strategy():
    eng = PlacementEngine(_devs())
    eng.register_strategy("last", lambda d, blk: float(d.index + 1))
    assert eng.place({"size_mb": 1}, "last")["gpu_id"] == 2


def test_connectome_weights_steer_placement():
    c = Connectome(alpha=1.0)
    c.record("gpu_0", 1.0)
    c.record("gpu_1", 10.0)             # a slow link
    assert c.weight("gpu_0") == pytest.approx(1.0) and c.weight("gpu_1") == pytest.approx(0.1)
    eng = PlacementEngine(_devs(), connectome=c)
    assert eng.place({"size_mb": 1}, "vram")["gpu_id"] == 0    # more free memory on 1, but its link is slow
    c.record("gpu_2", 1.0, ok=False)
    assert c.weight("gpu_2") < 1.0
    assert set(c.snapshot()) == {"gpu_0", "gpu_1", "gpu_2"}


def test_place_model_follows_speed_and_health():
    cfg = PRESETS["tiny-qwen2"]
    devs = [DeviceState(0, "a", 1e5, 1e5, 2.0), DeviceState(1, "b", 1e5, 1e5, 2.0)]
    even = PlacementEngine(devs).place_model(cfg, 2)
    assert [e - s for s, e in even] == [1, 1]
    c = Connectome(alpha=1.0)
    c.record("gpu_0", 1.0)
    c.record("gpu_1", 4.0)
    cfg8 = cfg.with_(num_layers=8)
    plan = PlacementEngine([DeviceState(0, "a", 1e5, 1e5, 2.0), DeviceState(1, "b", 1e5, 1e5, 2.0)],
                           connectome=c).place_model(cfg8, 2)
    sizes = [e - s for s, e in plan]
    assert sum(sizes) == 8 and sizes[0] > sizes[1]
    with pytest.raises(ValueError):
        PlacementEngine([DeviceState(0, "a", 1e-3, 1e-3, 1.0)]).place_model(cfg8, 1)
