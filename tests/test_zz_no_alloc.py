"""The allocation-free decode attention entry point, called through its exported C
symbol the way a caller that cannot allocate GPU memory would call it (no tensor
framework involvement in the call itself), checked against the regular entry point.

This file sorts last on purpose: if it fails, a run that stops at the first failure
has already run every other test.
"""
import ctypes
import math

import pytest
import torch

from vramancer_b200 import ops

pytestmark = pytest.mark.gpu

DEV = "cuda"


def _close(a, b, rtol=3e-2, atol=3e-2):
    a, b = a.float().cpu(), b.float().cpu()
    err = (a - b).abs()
    bad = (err > atol + rtol * b.abs()).sum().item()
    assert bad == 0, f"{bad} / {a.numel()} out of tolerance, max err {err.max().item():.4g}"


def _lib():
    import vramancer_b200._C as C

    lib = ctypes.CDLL(C.__file__)
    f = lib.vrm_paged_attention_decode_noalloc
    c = ctypes
    f.restype = c.c_int
    f.argtypes = [c.c_void_p, c.c_int64, c.c_void_p, c.c_int, c.c_int, c.c_int, c.c_int, c.c_int, c.c_int,
                  c.c_void_p, c.c_int, c.c_void_p, c.c_void_p, c.c_float, c.c_void_p, c.c_int64, c.c_int, c.c_int,
                  c.c_int, c.c_void_p]
    lib.vrm_noalloc_last_error.restype = c.c_char_p
    lib.vrm_noalloc_scratch_capacity.restype = c.c_size_t
    return lib


def _problem(fp8, seed=0):
    torch.manual_seed(seed)
    lens = [1, 17, 300, 64, 1033]
    L, layer, KH, Hq, D = 2, 1, 8, 40, 128
    ps = 16
    pages_per = [(n + ps - 1) // ps for n in lens]
    P = sum(pages_per) + 3
    perm = torch.randperm(P)
    bt = torch.zeros(len(lens), max(pages_per) + 1, dtype=torch.int32)
    k = 0
    for b, n in enumerate(pages_per):
        bt[b, :n] = perm[k:k + n].to(torch.int32)
        k += n
    cache = torch.randn(P, L, 2, KH, ps, D) * 1.5
    scale = None
    if fp8:
        scale = (torch.rand(L, 2, KH) + 0.5) / 50
        cache = (cache / scale.view(1, L, 2, KH, 1, 1)).clamp(-448, 448).to(torch.float8_e4m3fn)
        scale = scale.to(DEV)
    else:
        cache = cache.bfloat16()
    q = torch.randn(len(lens), (Hq + 2 * KH) * D).bfloat16()
    return dict(q=q.to(DEV), cache=cache.to(DEV), bt=bt.to(DEV), cl=torch.tensor(lens, dtype=torch.int32).to(DEV),
                scale=scale, L=L, layer=layer, KH=KH, Hq=Hq, D=D, B=len(lens))


def _call(lib, p, out, splits):
    stream = torch.cuda.current_stream().cuda_stream
    ptr = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
    return lib.vrm_paged_attention_decode_noalloc(
        ptr(p["q"]), p["q"].stride(0), ptr(p["cache"]), int(p["scale"] is not None), p["L"], p["layer"], p["KH"],
        p["D"], p["Hq"], ptr(p["bt"]), p["bt"].stride(0), ptr(p["cl"]), ptr(p["scale"]), 1.0 / math.sqrt(p["D"]),
        ptr(out), out.stride(0), p["B"], p["bt"].shape[1], splits, ctypes.c_void_p(stream))


@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("splits", [4, 0])
def test_noalloc_matches_regular_entry_point(fp8, splits):
    lib = _lib()
    p = _problem(fp8)
    want_splits = splits if splits > 0 else ops.decode_attention_splits(p["B"], p["KH"], p["bt"].shape[1])
    ref = ops.paged_attention_decode(p["q"], p["cache"], p["layer"], p["bt"], p["cl"], p["scale"],
                                     1.0 / math.sqrt(p["D"]), p["Hq"], num_splits=want_splits)
    torch.cuda.synchronize()
    for _ in range(2):      # two calls in a row share (and must clear) the static scratch
        out = torch.full_like(ref, float("nan"))
        torch.cuda.synchronize()
        before = torch.cuda.memory_allocated()
        rc = _call(lib, p, out, splits)
        assert rc == 0, lib.vrm_noalloc_last_error().decode()
        torch.cuda.synchronize()
        assert torch.cuda.memory_allocated() == before
        _close(out, ref)


def test_noalloc_rejects_oversized_request():
    lib = _lib()
    p = _problem(False, seed=1)
    out = torch.empty(p["B"], p["Hq"] * p["D"], dtype=torch.bfloat16, device=DEV)
    cap = lib.vrm_noalloc_scratch_capacity()
    # 128 splits of 5 x 40 heads x 128 dims of fp32 partials exceed the static scratch
    assert 5 * 40 * 128 * 128 * 4 > cap
    rc = _call(lib, p, out, 128)
    assert rc != 0
    assert b"scratch" in lib.vrm_noalloc_last_error()
