"""The allocation-free decode attention entry point, called through its exported C
symbol the way a caller that cannot allocate GPU memory would call it (no tensor
framework involvement in the call itself).

Such callers (a host framework whose allocator owns every device allocation, a job
held to a memory budget measured up front, a plain C program loading the shared
library) need the call to add no device memory.  The tests check that three ways:
the library's own count of device allocations, the device's free memory
(cudaMemGetInfo, which also sees allocations torch's caching allocator does not),
and a fresh process in which this entry point is the first call of the library on
the device, so that nothing set up lazily by an earlier call hides an allocation.
Results are compared with the fp32 PyTorch reference of the op (CPU) and with the
regular entry point.

This file sorts last on purpose: if it fails, a run that stops at the first failure
has already run every other test.
"""
import ctypes
import json
import math
import os
import subprocess
import sys

import pytest
import torch

pytestmark = pytest.mark.gpu

DEV = "cuda"
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


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
    lib.vrm_noalloc_setup.restype = c.c_int
    lib.vrm_noalloc_read_and_clear_errors.restype = c.c_int
    lib.vrm_noalloc_read_and_clear_errors.argtypes = [c.POINTER(c.c_uint32)]
    lib.vrm_host_device_allocations.restype = c.c_uint64
    return lib


def _problem(fp8, seed=0):
    """Host tensors of one decode step: 5 sequences of mixed lengths over a shuffled pool."""
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
    else:
        cache = cache.bfloat16()
    q = torch.randn(len(lens), (Hq + 2 * KH) * D).bfloat16()
    return dict(q=q, cache=cache, bt=bt, cl=torch.tensor(lens, dtype=torch.int32), scale=scale, L=L, layer=layer,
                KH=KH, Hq=Hq, D=D, B=len(lens))


def _to(p, dev):
    return {k: (v.to(dev) if isinstance(v, torch.Tensor) else v) for k, v in p.items()}


def _oracle(p):
    """fp32 PyTorch reference of the op (the ops layer's CPU path)."""
    from vramancer_b200 import ops
    return ops.paged_attention_decode(p["q"], p["cache"], p["layer"], p["bt"], p["cl"], p["scale"],
                                      1.0 / math.sqrt(p["D"]), p["Hq"])


def _call(lib, p, out, splits):
    stream = torch.cuda.current_stream().cuda_stream
    ptr = lambda t: ctypes.c_void_p(t.data_ptr()) if t is not None else None
    return lib.vrm_paged_attention_decode_noalloc(
        ptr(p["q"]), p["q"].stride(0), ptr(p["cache"]), int(p["scale"] is not None), p["L"], p["layer"], p["KH"],
        p["D"], p["Hq"], ptr(p["bt"]), p["bt"].stride(0), ptr(p["cl"]), ptr(p["scale"]), 1.0 / math.sqrt(p["D"]),
        ptr(out), out.stride(0), p["B"], p["bt"].shape[1], splits, ctypes.c_void_p(stream))


def _errors(lib):
    flags = ctypes.c_uint32(0)
    assert lib.vrm_noalloc_read_and_clear_errors(ctypes.byref(flags)) == 0, lib.vrm_noalloc_last_error().decode()
    return flags.value


@pytest.mark.parametrize("fp8", [False, True])
@pytest.mark.parametrize("splits", [4, 0])
def test_noalloc_matches_oracle_and_regular_entry_point(fp8, splits):
    from vramancer_b200 import ops
    lib = _lib()
    host = _problem(fp8)
    want = _oracle(host)
    p = _to(host, DEV)
    want_splits = splits if splits > 0 else ops.decode_attention_splits(p["B"], p["KH"], p["bt"].shape[1])
    regular = ops.paged_attention_decode(p["q"], p["cache"], p["layer"], p["bt"], p["cl"], p["scale"],
                                         1.0 / math.sqrt(p["D"]), p["Hq"], num_splits=want_splits)
    torch.cuda.synchronize()
    _close(regular, want)
    assert lib.vrm_noalloc_setup() == 0, lib.vrm_noalloc_last_error().decode()
    for _ in range(2):      # two calls in a row share (and must clear) the static scratch
        out = torch.full_like(regular, float("nan"))
        torch.cuda.synchronize()
        allocs, free0 = lib.vrm_host_device_allocations(), torch.cuda.mem_get_info()[0]
        rc = _call(lib, p, out, splits)
        assert rc == 0, lib.vrm_noalloc_last_error().decode()
        torch.cuda.synchronize()
        assert lib.vrm_host_device_allocations() == allocs
        assert torch.cuda.mem_get_info()[0] == free0
        _close(out, want)
        _close(out, regular)
    assert _errors(lib) == 0


def test_noalloc_rejects_oversized_request():
    lib = _lib()
    p = _to(_problem(False, seed=1), DEV)
    out = torch.empty(p["B"], p["Hq"] * p["D"], dtype=torch.bfloat16, device=DEV)
    cap = lib.vrm_noalloc_scratch_capacity()
    # 128 splits of 5 x 40 heads x 128 dims of fp32 partials exceed the static scratch
    assert 5 * 40 * 128 * 128 * 4 > cap
    rc = _call(lib, p, out, 128)
    assert rc != 0
    assert b"scratch" in lib.vrm_noalloc_last_error()
    rc = _call(lib, p, out, 129)
    assert rc != 0
    assert b"128" in lib.vrm_noalloc_last_error()


_FRESH = r"""
import ctypes, json, math, sys
import torch
sys.path.insert(0, {root!r})
sys.path.insert(0, {tests!r})
import test_zz_no_alloc as t
lib = t._lib()
host = t._problem(fp8=False, seed=3)
want = t._oracle(host)                      # CPU only: the device is untouched by the library
p = t._to(host, "cuda")
outs = []
torch.cuda.synchronize()
allocs0, free0 = lib.vrm_host_device_allocations(), torch.cuda.mem_get_info()[0]
for _ in range(2):
    out = torch.full((p["B"], p["Hq"] * p["D"]), float("nan"), dtype=torch.bfloat16, device="cuda")
    torch.cuda.synchronize()
    f0 = torch.cuda.mem_get_info()[0]
    rc = t._call(lib, p, out, 4)            # the first call also resolves the static scratch
    torch.cuda.synchronize()
    outs.append(dict(rc=rc, msg=lib.vrm_noalloc_last_error().decode(), free_delta=torch.cuda.mem_get_info()[0] - f0,
                     err=(out.float().cpu() - want).abs().max().item(),
                     bad=int(((out.float().cpu() - want).abs() > 3e-2 + 3e-2 * want.abs()).sum().item())))
print(json.dumps(dict(calls=outs, allocs=lib.vrm_host_device_allocations() - allocs0, errors=t._errors(lib))))
"""


def test_noalloc_first_call_in_fresh_process_allocates_nothing():
    """The entry point is the first call of the library on the device; modules load
    eagerly so that lazy module loading does not show up as a change of free memory."""
    script = _FRESH.format(root=ROOT, tests=os.path.join(ROOT, "tests"))
    env = dict(os.environ, CUDA_MODULE_LOADING="EAGER")
    r = subprocess.run([sys.executable, "-c", script], capture_output=True, text=True, env=env, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    res = json.loads(r.stdout.strip().splitlines()[-1])
    assert res["allocs"] == 0, res
    assert res["errors"] == 0, res
    for c in res["calls"]:
        assert c["rc"] == 0, c["msg"]
        assert c["free_delta"] == 0, res
        assert c["bad"] == 0, res
