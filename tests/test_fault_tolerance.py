"""GPU fault handling on the host (no GPU is faulted): error classification, the
health state machine with isolation after repeated failures, probe-driven recovery
(including the background thread), protected calls (OOM retry, fallback to a healthy
device), the OOM auto-heal ladder and block replicas / hidden-state checkpoints."""
import time

import pytest
import torch

from vramancer_b200.utils.fault import (BlockReplicator, FaultKind, GPUFaultManager, GPUHealth, OOMAutoHeal,
                                        classify_error)


def test_classify_error():
    cases = {
        "CUDA out of memory. Tried to allocate 2 GiB": FaultKind.OOM,
        "uncorrectable ECC error encountered": FaultKind.ECC,
        "GPU temperature above slowdown threshold": FaultKind.THERMAL,
        "bounded wait expired: error word 2": FaultKind.DEVICE_WAIT,
        "NCCL watchdog timed out": FaultKind.TIMEOUT,
        "CUDA error: an illegal memory access was encountered": FaultKind.DRIVER,
        "something else": FaultKind.UNKNOWN,
    }
    for msg, kind in cases.items():
        assert classify_error(RuntimeError(msg)) == kind, msg


def test_state_machine_isolation_and_recovery():
    alive = {0: True, 1: False}
    fm = GPUFaultManager([0, 1], isolate_after=3, probe=lambda g: alive[g])
    isolated, recovered = [], []
    fm.on_isolate.append(isolated.append)
    fm.on_recover.append(recovered.append)
    assert fm.handle_fault(0, RuntimeError("CUDA out of memory")) == FaultKind.OOM
    assert fm.states[0].health == GPUHealth.OOM
    fm.record_success(0)
    assert fm.states[0].health == GPUHealth.HEALTHY and fm.states[0].consecutive_failures == 0
    for _ in range(3):
        fm.handle_fault(1, RuntimeError("kernel timed out"))
    assert fm.states[1].health == GPUHealth.OFFLINE and isolated == [1]
    assert fm.healthy_gpus() == [0]
    assert fm.try_recover() == [] and fm.states[1].health == GPUHealth.OFFLINE
    alive[1] = True
    assert fm.try_recover() == [1] and recovered == [1] and fm.healthy_gpus() == [0, 1]
    # a driver fault isolates at once
    fm.handle_fault(0, RuntimeError("CUDA error: unspecified launch failure"))
    assert fm.states[0].health == GPUHealth.OFFLINE
    st = fm.status()
    assert st["0"]["total_failures"] == 2 and "launch failure" in st["0"]["last_error"]


def test_recovery_thread():
    fm = GPUFaultManager([0], probe=lambda g: True, recovery_interval_s=0.05)
    fm.isolate(0)
    fm.start_recovery_thread()
    t0 = time.time()
    while fm.states[0].health != GPUHealth.HEALTHY and time.time() - t0 < 5:
        time.sleep(0.02)
    fm.stop()
    assert fm.states[0].health == GPUHealth.HEALTHY


def test_protected_call_retry_and_fallback():
    fm = GPUFaultManager([0, 1], probe=lambda g: True)
    calls = {"n": 0}

    def oom_once():
        calls["n"] += 1
        if calls["n"] == 1:
            raise RuntimeError("CUDA out of memory")
        return "ok"

    assert fm.protected_call(0, oom_once) == "ok" and calls["n"] == 2
    assert fm.states[0].health == GPUHealth.HEALTHY

    def broken():
        raise RuntimeError("CUDA error: illegal address")

    assert fm.protected_call(0, broken, fallback=lambda g: f"ran on {g}") == "ran on 1"
    with pytest.raises(RuntimeError):
        fm.protected_call(1, broken)          # no healthy device left to fall back to


def test_oom_auto_heal_ladder():
    heal = OOMAutoHeal(min_scale=0.5)
    seen = []

    def gen(n):
        seen.append(n)
        if len(seen) == 1:
            raise RuntimeError("CUDA out of memory")
        return n

    assert heal.run(gen, 100) == 50 and seen == [100, 50]
    assert heal.events == 1 and heal.scale == 0.75 and heal.scaled(100) == 75
    for _ in range(5):
        heal.scale = max(heal.min_scale, heal.scale * 0.75)
    assert heal.scaled(100) == 50
    with pytest.raises(ValueError):
        heal.run(lambda n: (_ for _ in ()).throw(ValueError("not an OOM")), 10)


def test_block_replicas_and_checkpoints():
    rep = BlockReplicator(k=2)
    w = torch.randn(4, 8)
    orig = w.clone()
    rep.replicate("layers.3", w)
    w.add_(1.0)                                   # the live copy changes (or its device dies)
    assert len(rep.replicas["layers.3"]) == 2
    assert torch.equal(rep.restore("layers.3", "cpu"), orig)
    h = torch.randn(2, 8)
    rep.checkpoint("req-1", h)
    assert torch.equal(rep.resume("req-1", "cpu"), h) and rep.resume("nope", "cpu") is None
