"""Build of the vramancer_b200 native extensions (in-tree, sm_100a only).

    python setup.py build_ext --inplace

produces vramancer_b200/_C*.so (CUDA kernels) and vramancer_b200/_runtime*.so
(host-side C++ runtime: page allocator, parity, file spill, HMAC).
"""
import os

from setuptools import Extension, find_packages, setup
from torch.utils.cpp_extension import BuildExtension, CUDAExtension

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join("vramancer_b200", "csrc")
RT = os.path.join("vramancer_b200", "runtime")

# Explicit -gencode: torch's own arch list is bypassed, only sm_100a code is built.
NVCC_FLAGS = [
    "-gencode", "arch=compute_100a,code=sm_100a",
    "-O3", "-lineinfo", "-std=c++17",
    "--expt-relaxed-constexpr",
    "-U__CUDA_NO_HALF_OPERATORS__", "-U__CUDA_NO_HALF_CONVERSIONS__",
    "-U__CUDA_NO_BFLOAT16_CONVERSIONS__",
]
if os.environ.get("VRM_BOUNDS_CHECK") == "1":
    NVCC_FLAGS.append("-DVRM_BOUNDS_CHECK=1")


def _sources(d, exts):
    full = os.path.join(HERE, d)
    if not os.path.isdir(full):
        return []
    return sorted(os.path.join(d, f) for f in os.listdir(full) if f.endswith(exts))


cuda_sources = _sources(CSRC, (".cu", ".cpp"))
# selftest.cpp is the standalone sanitizer driver (tests/test_runtime_sanitizers.py), not part of the module
runtime_sources = [f for f in _sources(RT, (".cpp",)) if not f.endswith("selftest.cpp")]

ext_modules = [
    CUDAExtension(
        name="vramancer_b200._C",
        sources=cuda_sources,
        extra_compile_args={"cxx": ["-O3", "-std=c++17"], "nvcc": NVCC_FLAGS},
    ),
]
if runtime_sources:
    # host runtime: plain C++17 + pybind11, no torch or CUDA headers (compiles in seconds)
    import pybind11
    ext_modules.append(
        Extension(
            name="vramancer_b200._runtime",
            sources=runtime_sources,
            include_dirs=[pybind11.get_include(), RT],
            language="c++",
            extra_compile_args=["-O3", "-std=c++17", "-pthread", "-fvisibility=hidden"],
            extra_link_args=["-pthread"],
        )
    )

setup(
    name="vramancer_b200",
    version="0.1.0",
    packages=find_packages(include=["vramancer_b200", "vramancer_b200.*"]),
    package_data={"vramancer_b200.utils": ["monitoring/*.yml", "monitoring/*.json"]},
    entry_points={"console_scripts": ["vramancer = vramancer_b200.cli:main"]},
    ext_modules=ext_modules,
    cmdclass={"build_ext": BuildExtension.with_options(use_ninja=True)},
)
