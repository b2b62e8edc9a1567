"""Transfer manager: method choice on a synthetic topology, NVLink count through a fake
NVML (CPU); staged and peer copies on GPUs."""
import pytest
import torch

from vramancer_b200.parallel.transfer import GPUTopology, TransferManager, TransportMethod, _nvlink_counts


class FakeNVML:
    def nvmlInit(self):
        pass

    def nvmlDeviceGetCount(self):
        return 2

    def nvmlDeviceGetHandleByIndex(self, i):
        return i

    def nvmlDeviceGetNvLinkState(self, h, link):
        if link >= 18:
            raise RuntimeError("no such link")
        return 1 if (h == 0 or link < 9) else 0


def test_method_choice_and_stats_cpu():
    topo = GPUTopology(num_gpus=3, p2p_matrix={(0, 1): True, (1, 0): True, (0, 2): False, (2, 0): False})
    tm = TransferManager(topology=topo)
    assert tm.method_for(0, 1) == TransportMethod.CUDA_P2P
    assert tm.method_for(0, 2) == TransportMethod.CPU_STAGED
    assert tm.method_for(1, 1) == TransportMethod.SAME_DEVICE
    assert tm.method_for(-1, 0) == TransportMethod.CPU_ONLY
    out, r = tm.send_activation(-1, -1, torch.ones(10))
    assert torch.equal(out, torch.ones(10)) and r.method == TransportMethod.CPU_ONLY
    s = tm.stats()
    assert s["transfers"] == 1 and "cpu_only" in s["by_method"]


def test_nvlink_count_with_fake_nvml():
    assert _nvlink_counts(FakeNVML()) == {0: 18, 1: 9}


@pytest.mark.gpu
def test_staged_copy_on_one_gpu():
    tm = TransferManager(staging_chunk_mb=1)
    x = torch.randn((3 << 20) // 4 + 123, device="cuda:0")     # several 1 MiB chunks + a tail
    out = torch.empty_like(x)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        tm._staged(x, out, s)
    s.synchronize()
    assert torch.equal(out, x)


@pytest.mark.gpu
@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
def test_peer_and_staged_between_two_gpus():
    tm = TransferManager()
    x = torch.randn(1 << 20, device="cuda:0")
    y, r = tm.send_activation(0, 1, x)
    assert y.device.index == 1 and torch.equal(y.cpu(), x.cpu())
    assert r.method in (TransportMethod.CUDA_P2P, TransportMethod.CPU_STAGED) and r.bandwidth_gbs > 0
    forced = TransferManager(topology=GPUTopology(num_gpus=2, p2p_matrix={(0, 1): False, (1, 0): False}),
                             staging_chunk_mb=1)
    z, r2 = forced.send_activation(0, 1, x)
    assert r2.method == TransportMethod.CPU_STAGED and torch.equal(z.cpu(), x.cpu())
    rows = tm.benchmark(sizes_mb=[4], iterations=2, pairs=[(0, 1)])
    assert rows[0]["gbs"] > 0
