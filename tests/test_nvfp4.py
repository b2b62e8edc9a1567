"""NVFP4 weights: the host oracle (rounding, scales, fragment order) on CPU, and the
CUDA quantise / dequantise / W4A16 GEMM kernels against it on a B200."""
import pytest
import torch

from vramancer_b200 import ops
from vramancer_b200.quant import nvfp4


def test_e2m1_rounding_ties_to_even():
    v = torch.tensor([0.0, 0.2, 0.25, 0.3, 0.75, 1.25, 1.75, 2.5, 3.5, 5.0, 5.1, 7.0, 100.0, -0.75, -5.0])
    got = nvfp4.e2m1_values(nvfp4.e2m1_codes(v))
    want = torch.tensor([0.0, 0.0, 0.0, 0.5, 1.0, 1.0, 2.0, 2.0, 4.0, 4.0, 6.0, 6.0, 6.0, -1.0, -4.0])
    assert torch.equal(got, want)


def test_block_scale_convention():
    w = torch.zeros(16, 64)
    w[0, :16] = torch.linspace(-3, 3, 16)
    w[3, 16] = 12.0                                   # tensor amax
    gs = nvfp4.global_scale(w)
    assert torch.allclose(gs, torch.tensor([12.0 / (6 * 448)]))
    s = nvfp4.block_scales_ref(w, gs).view(torch.float8_e4m3fn).float()
    assert s[3, 1] == 448.0                           # the amax block uses the full e4m3 range
    assert s[5, 0] == 0.0                             # all-zero block


@pytest.mark.parametrize("N,K", [(16, 64), (48, 128), (128, 320)])
def test_fragment_order_round_trip_and_error_bound(N, K):
    g = torch.Generator().manual_seed(N + K)
    w = torch.randn(N, K, generator=g) * torch.rand(N, 1, generator=g) * 3
    qw = nvfp4.quantize_ref(w)
    assert qw.q.numel() == N * K // 2 and qw.s.numel() == N * K // 16
    deq = nvfp4.dequantize_ref(qw)
    # per 16-block: |err| <= half an e2m1 step at the top of the range (1 of 6) * scale,
    # plus the e4m3 rounding of the scale (<= 1/16 relative)
    blk = w.abs().view(N, K // 16, 16).amax(-1, keepdim=True)
    err = (deq - w).abs().view(N, K // 16, 16)
    assert torch.all(err <= blk * (1.0 / 6.0 + 1.0 / 16.0) + 1e-6)
    # requantising the dequantised weight reproduces the same bytes
    again = nvfp4.quantize_ref(deq)
    assert torch.equal(again.s, qw.s)
    assert torch.equal(nvfp4.dequantize_ref(again), deq)


def test_linear_dispatch_cpu():
    g = torch.Generator().manual_seed(3)
    w = torch.randn(32, 128, generator=g)
    x = torch.randn(5, 128, generator=g)
    qw = nvfp4.quantize(w)
    y = ops.linear(x, qw)
    ref = x @ nvfp4.dequantize_ref(qw).t()
    assert torch.allclose(y.float(), ref, atol=1e-4, rtol=1e-4)
    lin = nvfp4.DirectFP4Linear(w)
    assert lin(x.view(1, 5, 128)).shape == (1, 5, 32)


def test_quantize_model_weights_skips_non_projections():
    from vramancer_b200.models.config import get_config
    from vramancer_b200.models.weights import random_weights
    cfg = get_config("tiny-qwen2")
    w = random_weights(cfg, device="cpu", dtype=torch.float32, seed=1)
    q = nvfp4.quantize_model_weights(w, cfg)
    kinds = {k: type(v).__name__ for k, v in q.items()}
    assert kinds["embed"] == "Tensor" and kinds["layers.0.in_norm_w"] == "Tensor"
    assert all(kinds[k] == "NVFP4Weight" for k in q if k.endswith(("qkv_w", "o_w", "gate_up_w", "down_w"))
               and nvfp4.quantizable(w[k]))


# ---------------------------------------------------------------- GPU kernels
@pytest.mark.gpu
@pytest.mark.parametrize("N,K", [(16, 64), (256, 512), (1024, 5120)])
def test_quantize_kernel_matches_oracle(N, K):
    g = torch.Generator().manual_seed(K)
    w = (torch.randn(N, K, generator=g) * torch.rand(N, 1, generator=g) * 2).to(torch.bfloat16)
    got = nvfp4.quantize(w.cuda())
    assert torch.equal(got.gs.cpu(), nvfp4.global_scale(w))
    ref = nvfp4.quantize_ref(w, got.gs)
    assert torch.equal(got.s.cpu(), ref.s)
    # bytes may differ only in the sign of zero codes: compare values
    assert torch.equal(nvfp4.dequantize_ref(got), nvfp4.dequantize_ref(ref))
    deq = got.dequantize().float().cpu()
    assert torch.allclose(deq, nvfp4.dequantize_ref(ref).to(torch.bfloat16).float(), atol=0, rtol=0)


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 3, 8, 17, 32])
@pytest.mark.parametrize("N,K", [(256, 512), (5120, 1280), (1040, 13824)])
def test_w4a16_gemm_matches_fp32(M, N, K):
    g = torch.Generator().manual_seed(M * 7 + N)
    w = (torch.randn(N, K, generator=g) * 0.05).to(torch.bfloat16).cuda()
    x = torch.randn(M, K, generator=g).to(torch.bfloat16).cuda()
    b = torch.randn(N, generator=g).to(torch.bfloat16).cuda()
    r = torch.randn(M, N, generator=g).to(torch.bfloat16).cuda()
    qw = nvfp4.quantize(w)
    wd = nvfp4.dequantize_ref(qw).cuda()
    ref = x.float() @ wd.t() + b.float() + r.float()
    for _ in range(2):       # second call reuses the split-K counters
        y = ops.linear(x, qw, b, residual=r)
    torch.cuda.synchronize()
    err = (y.float() - ref).abs().max() / ref.abs().max()
    assert err < 1e-2, float(err)
    # SiLU(gate) * up over interleaved rows
    ys = ops.linear(x, qw, epilogue=ops.EPI_SILU_MUL)
    h = x.float() @ wd.t()
    refs = torch.nn.functional.silu(h[:, 0::2]) * h[:, 1::2]
    assert (ys.float() - refs).abs().max() / refs.abs().max() < 1e-2
    assert ops.read_and_clear_errors() == 0


@pytest.mark.gpu
def test_nvfp4_model_generates():
    from vramancer_b200.engine.engine import SamplingParams
    from vramancer_b200.llm import LLM
    llm = LLM("tiny-qwen2-d128", device="cuda:0", quantization="nvfp4", max_batch=4, max_model_len=128,
              kv_pages=64)
    assert type(llm.runner.model.w["layers.0.qkv_w"]).__name__ == "NVFP4Weight"
    out = llm.generate([[1, 2, 3, 4], list(range(40))], SamplingParams(max_tokens=6))
    assert all(len(o.output_ids) == 6 for o in out)
    llm.runner.release_graphs()


# ----------------------------------------------------------------------------- block-scaled (W4A4) path
def test_rows_ref_roundtrip_cpu():
    from vramancer_b200.quant import nvfp4 as nv
    g = torch.Generator().manual_seed(0)
    x = torch.randn(130, 512, generator=g) * 3
    q, atoms, gs = nv.quantize_rows_ref(x)
    assert q.shape == (256, 256) and atoms.numel() == 2 * 8 * 512 and gs.shape == (256,)
    deq = nv.dequantize_rows_ref(q, atoms, gs, 130)
    rel = (deq - x).norm() / x.norm()
    assert rel < 0.15                               # 4-bit values with e4m3 scales per 16
    assert torch.equal(nv.atoms_to_sf(nv.sf_to_atoms(torch.arange(256 * 32).to(torch.uint8).view(256, 32)), 256, 512),
                       torch.arange(256 * 32).to(torch.uint8).view(256, 32))


@pytest.mark.gpu
@pytest.mark.parametrize("valid,K,per_row", [(200, 512, True), (128, 1024, False), (1, 256, True)])
def test_rows_quantize_matches_ref(valid, K, per_row, cuda_errors_clean):
    from vramancer_b200 import ops
    from vramancer_b200.quant import nvfp4 as nv
    g = torch.Generator().manual_seed(valid + K)
    x = (torch.randn(valid, K, generator=g) * 2).bfloat16()
    gs = None if per_row else nv.global_scale(x.float())
    rows = (valid + 127) // 128 * 128
    q, atoms, gr = ops.native().nvfp4_rows_quantize(x.cuda(), rows, gs.cuda() if gs is not None else None)
    rq, ratoms, rg = nv.quantize_rows_ref(x, rows, gs)
    assert torch.equal(q.cpu(), rq)
    assert torch.equal(atoms.cpu(), ratoms)
    if per_row:
        assert torch.equal(gr.cpu(), rg)


@pytest.mark.gpu
@pytest.mark.parametrize("M,N,K", [(128, 128, 256), (200, 384, 1024), (1, 256, 512), (300, 1280, 5120)])
def test_blockscaled_gemm_matches_dequant(M, N, K, cuda_errors_clean):
    """tcgen05 kind::mxf4nvf4 GEMM against fp32 math on the dequantised operands."""
    from vramancer_b200 import ops
    from vramancer_b200.quant import nvfp4 as nv
    g = torch.Generator().manual_seed(M + N + K)
    x = torch.randn(M, K, generator=g).bfloat16()
    w = (torch.randn(N, K, generator=g) * 0.02).bfloat16()
    gw = nv.global_scale(w.float())
    Mp = (M + 127) // 128 * 128
    qa, sfa, gsa = ops.native().nvfp4_rows_quantize(x.cuda(), Mp, None)
    qb, sfb, _ = ops.native().nvfp4_rows_quantize(w.cuda(), N, gw.cuda())
    out = ops.native().nvfp4_bs_gemm(qa, sfa, gsa, M, qb, sfb, gw.cuda())
    torch.cuda.synchronize()
    a = nv.dequantize_rows_ref(qa, sfa, gsa, M)
    b = nv.dequantize_rows_ref(qb, sfb, gw, N)
    ref = a @ b.t()
    err = (out.float().cpu() - ref).abs().max().item()
    assert err <= 1e-2 * ref.abs().max().item() + 1e-3, (err, ref.abs().max().item())


@pytest.mark.gpu
@pytest.mark.parametrize("epi", ["none", "bias_residual", "silu_mul"])
def test_nvfp4_weight_prefill_linear(epi, cuda_errors_clean):
    """NVFP4Weight.linear for a prefill batch: activation quantisation + block-scaled
    GEMM + epilogue, against fp32 math on the same quantised operands."""
    from vramancer_b200 import ops
    from vramancer_b200.quant import nvfp4 as nv
    g = torch.Generator().manual_seed(9)
    M, N, K = 150, 512, 1024
    w = (torch.randn(N, K, generator=g) * 0.02).bfloat16()
    x = torch.randn(M, K, generator=g).bfloat16()
    qw = nv.quantize(w.cuda())
    assert qw.q_rows is not None
    # same codes / scales as the fragment-order copy
    assert torch.equal(nv.dequantize_rows_ref(qw.q_rows, qw.s_atoms, qw.gs, N), nv.dequantize_ref(qw))
    qa, sfa, gsa = nv.quantize_rows_ref(x)
    y = nv.dequantize_rows_ref(qa, sfa, gsa, M) @ nv.dequantize_ref(qw).t()
    kw = {}
    if epi == "bias_residual":
        b = (torch.randn(N, generator=g) * 0.1).bfloat16()
        r = torch.randn(M, N, generator=g).bfloat16()
        kw = dict(bias=b.cuda(), residual=r.cuda())
        y = y + b.float() + r.float()
    elif epi == "silu_mul":
        kw = dict(epilogue=ops.EPI_SILU_MUL)
        y = torch.nn.functional.silu(y[:, 0::2]) * y[:, 1::2]
    out = ops.linear(x.cuda(), qw, **kw)
    torch.cuda.synchronize()
    err = (out.float().cpu() - y).abs().max().item()
    assert err <= 2e-2 * y.abs().max().item() + 2e-2, err


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 7, 16, 33, 100, 128])
@pytest.mark.parametrize("N,K", [(256, 512), (1280, 5120), (512, 13824)])
@pytest.mark.parametrize("epi", ["none", "bias_residual", "silu_mul"])
def test_nvfp4_tc_decode_gemm(M, N, K, epi, cuda_errors_clean):
    """tcgen05 W4A16 decode GEMM (codes x block scales -> f16 tiles in shared memory)
    against fp32 math on the dequantised weight and the f16-rounded activations."""
    from vramancer_b200 import ops
    from vramancer_b200.quant import nvfp4 as nv
    g = torch.Generator().manual_seed(M * 31 + N + K)
    w = (torch.randn(N, K, generator=g) * 0.02).bfloat16()
    x = torch.randn(M, K, generator=g).bfloat16()
    qw = nv.quantize(w.cuda())
    assert qw.q_rows is not None
    wd = nv.dequantize_ref(qw)
    y = x.half().float() @ wd.t()
    kw = {}
    epilogue = ops.EPI_NONE
    if epi == "bias_residual":
        b = (torch.randn(N, generator=g) * 0.1).bfloat16()
        r = torch.randn(M, N, generator=g).bfloat16()
        kw = dict(bias=b.cuda(), residual=r.cuda())
        y = y + b.float() + r.float()
    elif epi == "silu_mul":
        epilogue = ops.EPI_SILU_MUL
        gg, u = y[:, 0::2], y[:, 1::2]
        y = gg * torch.sigmoid(gg) * u
    n_out = N // 2 if epi == "silu_mul" else N
    out = torch.empty(M, n_out, dtype=torch.bfloat16, device="cuda")
    ops.native().nvfp4_tc_gemm_out(x.cuda(), qw.q_rows, qw.s_atoms, qw.gs, kw.get("bias"), out, epilogue,
                                   kw.get("residual"))
    torch.cuda.synchronize()
    err = (out.float().cpu() - y).abs()
    tol = 2e-2 * y.abs().max().item() + 1e-2
    assert err.max().item() <= tol, (err.max().item(), tol)
    # the linear dispatch with the tcgen05 decode kernel selected gives the same bits
    old = nv.DECODE_KERNEL
    nv.DECODE_KERNEL = "tc"
    try:
        out2 = qw.linear(x.cuda(), kw.get("bias"), epilogue=epilogue, residual=kw.get("residual"))
    finally:
        nv.DECODE_KERNEL = old
    assert torch.equal(out2, out)
