"""Fused row-parallel GEMM + all-reduce + residual + norm, checked on one GPU.

Tensor-parallel ranks are emulated on one device: every emulated rank gets its own
receive buffer (filled with the empty pattern), its own epoch and completion counter,
and the push GEMMs of all ranks run (in stream order) before any rank's reduce, so no
kernel ever waits for another kernel that runs at the same time.  Results are compared
with the fp32 PyTorch reference of sum_r x_r @ w_r^T + bias + residual, then RMSNorm.

The timeout test leaves one emulated rank's push out: the reduce must give up after its
spin budget, report kErrFlagTimeout (2) in the error word it was given, count the
missing values as 0, and leave the device usable.
"""
import pytest
import torch

from vramancer_b200 import ops

pytestmark = pytest.mark.gpu

DEV = "cuda"
EMPTY = 0x8000
K_ERR_FLAG_TIMEOUT = 2


class Ranks:
    """Receive buffers of `world` emulated ranks on one GPU."""

    def __init__(self, world, max_tokens=128, max_features=8192):
        nat = ops.native()
        self.world = world
        self.half = max_tokens * max_features
        n = 2 * world * self.half
        self.bufs = [nat.symm_malloc(n * 2) for _ in range(world)]
        for b in self.bufs:
            nat.symm_fill_u16(b, n, EMPTY)
        self.ptrs = torch.tensor(self.bufs, dtype=torch.int64, device=DEV)
        self.epoch = [torch.zeros(1, dtype=torch.int32, device=DEV) for _ in range(world)]
        self.done = [torch.zeros(1, dtype=torch.int32, device=DEV) for _ in range(world)]

    def push(self, r, x, w, sx=None, sw=None):
        ops.native().gemm_ar_push(x, w, self.ptrs, self.epoch[r], r, self.world, self.half, sx, sw)

    def reduce(self, r, T, H, bias=None, residual=None, out=None, norm_w=None, spin_limit=0, err=None):
        mode = 0 if norm_w is None else 1
        ops.native().ar_norm(self.bufs[r], self.epoch[r], self.done[r], r, self.world, self.half, T, H, bias,
                             residual, norm_w, None, out, mode, 1e-6, spin_limit, err)

    def free(self):
        torch.cuda.synchronize()
        for b in self.bufs:
            ops.native().symm_free(b)


def _reference(xs, ws, bias, res, nw, eps=1e-6):
    y = sum(x.float() @ w.float().t() for x, w in zip(xs, ws))
    s = (y + bias.float() + res.float()).bfloat16().float()
    n = s * torch.rsqrt(s.pow(2).mean(-1, keepdim=True) + eps) * nw.float()
    return s, n


def _rel(a, b):
    return float((a.float() - b.float()).abs().max() / (b.float().abs().max() + 1e-6))


@pytest.mark.parametrize("world", [1, 2, 4, 8])
@pytest.mark.parametrize("m", [1, 7, 32, 100])
def test_fused_allreduce_norm_matches_reference(world, m):
    n, k = 1024, 640
    g = torch.Generator(device=DEV).manual_seed(world * 100 + m)
    ranks = Ranks(world)
    try:
        xs = [torch.randn(m, k, device=DEV, generator=g).bfloat16() for _ in range(world)]
        ws = [(torch.randn(n, k, device=DEV, generator=g) * 0.05).bfloat16() for _ in range(world)]
        bias = torch.randn(n, device=DEV, generator=g).bfloat16()
        res0 = torch.randn(m, n, device=DEV, generator=g).bfloat16()
        nw = (1 + 0.1 * torch.randn(n, device=DEV, generator=g)).bfloat16()
        want_s, want_n = _reference(xs, ws, bias, res0, nw)
        for it in range(3):        # alternating halves: each call must find its slots emptied
            resid = [res0.clone() for _ in range(world)]
            outs = [torch.empty(m, n, device=DEV, dtype=torch.bfloat16) for _ in range(world)]
            for r in range(world):
                ranks.push(r, xs[r], ws[r])
            for r in range(world):
                ranks.reduce(r, m, n, bias=bias, residual=resid[r], out=outs[r], norm_w=nw)
            torch.cuda.synchronize()
            for r in range(world):
                assert _rel(resid[r], want_s) < 1e-2
                assert _rel(outs[r], want_n) < 2e-2
                # rank-order sums: every rank holds the same bits
                assert torch.equal(resid[r], resid[0]) and torch.equal(outs[r], outs[0])
        assert all(int(e.item()) == 3 for e in ranks.epoch)
        assert ops.read_and_clear_errors() == 0
    finally:
        ranks.free()


def test_fused_allreduce_fp8_and_nvfp4_pushes():
    from vramancer_b200.quant import fp8 as fp8q
    from vramancer_b200.quant import nvfp4 as nvq
    m, n, k = 5, 1024, 1024
    g = torch.Generator(device=DEV).manual_seed(9)
    ranks = Ranks(2)
    try:
        xs = [torch.randn(m, k, device=DEV, generator=g).bfloat16() for _ in range(2)]
        ws = [(torch.randn(n, k, device=DEV, generator=g) * 0.05).bfloat16() for _ in range(2)]
        for quant in (fp8q.quantize, nvq.quantize):
            qw = [quant(w) for w in ws]
            # expected: each rank's own quantised GEMM (regular entry point), summed in fp32
            want = sum(ops.linear(x, q).float() for x, q in zip(xs, qw))
            outs = [torch.zeros(m, n, device=DEV, dtype=torch.bfloat16) for _ in range(2)]
            for r in range(2):
                if getattr(qw[r], "_vrm_quant") == "fp8":
                    xq, sx = ops.native().fp8_rows_quantize(xs[r].contiguous())
                    ranks.push(r, xq, qw[r].q, sx, qw[r].scale)
                else:
                    ops.native().nvfp4_gemm_ar_push(xs[r], qw[r].q, qw[r].s, qw[r].gs, qw[r].N, ranks.ptrs,
                                                    ranks.epoch[r], r, 2, ranks.half)
            for r in range(2):
                ranks.reduce(r, m, n, residual=outs[r])
            torch.cuda.synchronize()
            for r in range(2):
                assert _rel(outs[r], want) < 2e-2
        assert ops.read_and_clear_errors() == 0
    finally:
        ranks.free()


def test_fused_allreduce_wait_times_out_and_reports():
    """Rank 1 never pushes: rank 0's reduce gives up after ~2e6 cycles (about 1 ms)."""
    m, n, k = 4, 512, 256
    g = torch.Generator(device=DEV).manual_seed(1)
    ranks = Ranks(2)
    try:
        x = torch.randn(m, k, device=DEV, generator=g).bfloat16()
        w = (torch.randn(n, k, device=DEV, generator=g) * 0.05).bfloat16()
        resid = torch.zeros(m, n, device=DEV, dtype=torch.bfloat16)
        err = torch.zeros(1, dtype=torch.int32, device=DEV)
        ranks.push(0, x, w)
        start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        start.record()
        ranks.reduce(0, m, n, residual=resid, spin_limit=2_000_000, err=err)
        end.record()
        torch.cuda.synchronize()
        assert int(err.item()) & K_ERR_FLAG_TIMEOUT
        assert start.elapsed_time(end) < 500.0          # ms: the budget, not the default second
        # the missing rank counted as 0: only rank 0's partial arrived
        want = (x.float() @ w.float().t())
        assert _rel(resid, want) < 1e-2
        # the context is still usable and the global error word was not touched
        assert ops.read_and_clear_errors() == 0
        assert float(torch.ones(4, device=DEV).sum().item()) == 4.0
    finally:
        ranks.free()


@pytest.mark.parametrize("world", [1, 2, 8])
@pytest.mark.parametrize("m", [1, 32])
def test_fused_push_reduce_one_kernel(world, m):
    """GEMM + push + reduce into the residual + norm sums in one launch (rank 0); the
    other emulated ranks' partials are pushed first by plain push GEMMs, so rank 0's
    kernel finds every slot filled and waits on nothing that runs at the same time."""
    n, k = 1024, 512
    g = torch.Generator(device=DEV).manual_seed(7 * world + m)
    ranks = Ranks(world)
    try:
        xs = [torch.randn(m, k, device=DEV, generator=g).bfloat16() for _ in range(world)]
        ws = [(torch.randn(n, k, device=DEV, generator=g) * 0.05).bfloat16() for _ in range(world)]
        bias = torch.randn(n, device=DEV, generator=g).bfloat16()
        res0 = torch.randn(m, n, device=DEV, generator=g).bfloat16()
        want_s, _ = _reference(xs, ws, bias, res0, torch.ones(n, device=DEV).bfloat16())
        want_ssq = want_s.view(m, n // 128, 128).pow(2).sum(-1).t()
        for it in range(3):
            for r in range(1, world):
                ranks.push(r, xs[r], ws[r])
            resid = res0.clone()
            ssq = torch.zeros(n // 128, 128, device=DEV)
            ops.native().gemm_ar_push(xs[0], ws[0], ranks.ptrs, ranks.epoch[0], 0, world, ranks.half, None, None,
                                      resid, bias, ssq, ranks.done[0], 0)
            torch.cuda.synchronize()
            assert _rel(resid, want_s) < 1e-2
            assert _rel(ssq[:, :m], want_ssq) < 2e-2
            # the other ranks' halves were consumed only by rank 0: empty them for the next round
            for r in range(1, world):
                ranks.reduce(r, m, n, residual=torch.zeros(m, n, device=DEV, dtype=torch.bfloat16))
        assert int(ranks.epoch[0].item()) == 3
        assert ops.read_and_clear_errors() == 0
    finally:
        ranks.free()


def test_fused_push_reduce_times_out_and_reports():
    m, n, k = 2, 512, 256
    g = torch.Generator(device=DEV).manual_seed(5)
    ranks = Ranks(2)
    try:
        x = torch.randn(m, k, device=DEV, generator=g).bfloat16()
        w = (torch.randn(n, k, device=DEV, generator=g) * 0.05).bfloat16()
        resid = torch.zeros(m, n, device=DEV, dtype=torch.bfloat16)
        err_before = ops.read_and_clear_errors()
        assert err_before == 0
        ops.native().gemm_ar_push(x, w, ranks.ptrs, ranks.epoch[0], 0, 2, ranks.half, None, None, resid, None,
                                  None, ranks.done[0], 2_000_000)
        torch.cuda.synchronize()
        assert ops.read_and_clear_errors() & K_ERR_FLAG_TIMEOUT
        assert _rel(resid, x.float() @ w.float().t()) < 1e-2       # the missing rank counted as 0
        assert float(torch.ones(4, device=DEV).sum().item()) == 4.0
    finally:
        ranks.free()
