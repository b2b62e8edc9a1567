"""Host runtime under sanitizers (CPU only): the C++ sources of vramancer_b200._runtime
are compiled with a standalone self-test driver (runtime/selftest.cpp) once with
AddressSanitizer + UndefinedBehaviorSanitizer and once with ThreadSanitizer, and the
binaries must finish with no failed check and no sanitizer report.  The threaded paths
(batched HMAC, parity, tokenizer, the async I/O pool fed from several threads, a TCP
sender thread) are where ThreadSanitizer looks for data races."""
import os
import shutil
import subprocess

import pytest

RT = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "vramancer_b200", "runtime")
SOURCES = ["selftest.cpp", "crypto.cpp", "parity.cpp", "file_io.cpp", "page_alloc.cpp", "tokenizer.cpp",
           "transport.cpp"]


def _build_and_run(tmp_path, flags, env_extra):
    cxx = shutil.which("g++")
    if cxx is None:
        pytest.skip("no g++")
    exe = tmp_path / "selftest"
    cmd = [cxx, "-std=c++17", "-O1", "-g", "-fno-omit-frame-pointer", "-pthread", *flags,
           *[os.path.join(RT, s) for s in SOURCES], "-o", str(exe)]
    b = subprocess.run(cmd, capture_output=True, text=True, timeout=600)
    if b.returncode != 0 and "sanitize" in b.stderr and "unrecognized" in b.stderr:
        pytest.skip("compiler without this sanitizer")
    assert b.returncode == 0, b.stderr[-2000:]
    env = dict(os.environ, **env_extra)
    r = subprocess.run([str(exe), str(tmp_path)], capture_output=True, text=True, timeout=600, env=env)
    out = r.stdout + r.stderr
    assert r.returncode == 0, out[-4000:]
    assert "runtime selftest: 0 failure(s)" in out
    assert "Sanitizer" not in out and "runtime error" not in out, out[-4000:]


def test_runtime_asan_ubsan(tmp_path):
    _build_and_run(tmp_path, ["-fsanitize=address,undefined", "-fno-sanitize-recover=undefined"],
                   {"ASAN_OPTIONS": "detect_leaks=1:abort_on_error=0"})


def test_runtime_tsan(tmp_path):
    _build_and_run(tmp_path, ["-fsanitize=thread"], {"TSAN_OPTIONS": "halt_on_error=1"})


def test_kernel_bounds_check_build_compiles(tmp_path):
    """The bounds-check variant (-DVRM_BOUNDS_CHECK=1) of the kernels that index the KV
    pool through tables (paged attention, RoPE + KV write, page copy) still compiles
    for sm_100a."""
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("no nvcc")
    csrc = os.path.join(os.path.dirname(RT), "csrc")
    for f in ("norm_rope.cu", "migrate.cu", "attention.cu"):
        r = subprocess.run([nvcc, "-gencode", "arch=compute_100a,code=sm_100a", "-O1", "-std=c++17",
                            "--expt-relaxed-constexpr", "-DVRM_BOUNDS_CHECK=1", "-c", os.path.join(csrc, f),
                            "-o", str(tmp_path / (f + ".o"))], capture_output=True, text=True, timeout=900)
        assert r.returncode == 0, (f, r.stderr[-2000:])
