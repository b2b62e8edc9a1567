"""FP8 (e4m3) W8A8: host oracle on the CPU, CUDA kernels against it on the GPU."""
import pytest
import torch

from vramancer_b200 import ops
from vramancer_b200.quant import fp8


def test_rows_ref_roundtrip():
    x = torch.randn(5, 256) * 3
    q, s = fp8.quantize_rows_ref(x)
    assert q.dtype == torch.uint8 and s.shape == (5,)
    rel = (fp8.dequantize_rows_ref(q, s) - x).norm() / x.norm()
    assert rel < 0.05


def test_cpu_linear_uses_quantised_math():
    w = torch.randn(64, 256) * 0.02
    x = torch.randn(3, 256)
    qw = fp8.quantize(w)
    xq, sx = fp8.quantize_rows_ref(x)
    want = fp8.dequantize_rows_ref(xq, sx) @ qw.dequantize().t()
    torch.testing.assert_close(qw.linear(x), want, rtol=1e-5, atol=1e-5)


@pytest.mark.gpu
@pytest.mark.parametrize("M", [1, 7, 32, 100, 300])
@pytest.mark.parametrize("epi", ["none", "bias_residual", "silu_mul"])
def test_gemm_fp8_matches_ref(M, epi, cuda_errors_clean):
    g = torch.Generator().manual_seed(M)
    N, K = 640, 1280
    x = torch.randn(M, K, generator=g).bfloat16()
    w = (torch.randn(N, K, generator=g) * 0.02).bfloat16()
    qw = fp8.quantize(w.cuda())
    rq, rs = fp8.quantize_rows_ref(w)
    assert torch.equal(qw.q.cpu(), rq) and torch.equal(qw.scale.cpu(), rs)
    xq, sx = fp8.quantize_rows_ref(x)
    y = fp8.dequantize_rows_ref(xq, sx) @ fp8.dequantize_rows_ref(rq, rs).t()
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
    assert err <= 1e-2 * y.abs().max().item() + 1e-2, err


@pytest.mark.gpu
def test_fp8_model_decodes_under_graphs(cuda_errors_clean):
    from vramancer_b200.engine.engine import SamplingParams
    from vramancer_b200.llm import LLM
    kw = dict(device="cuda:0", max_batch=4, max_model_len=128, kv_pages=64, seed=5, quantization="fp8")
    prompts = [[1, 2, 3, 4, 5], list(range(10, 50))]
    eager = LLM("tiny-qwen2-d128", use_cuda_graph=False, **kw)
    want = [o.output_ids for o in eager.generate(prompts, SamplingParams(max_tokens=6))]
    graph = LLM("tiny-qwen2-d128", use_cuda_graph=True, **kw)
    got = [o.output_ids for o in graph.generate(prompts, SamplingParams(max_tokens=6))]
    assert got == want
    graph.runner.release_graphs()
