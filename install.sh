#!/usr/bin/env bash
# Installs vramancer_b200 from this source tree on a Linux host with a B200 (sm_100a).
#
#   ./install.sh            build the CUDA / C++ extensions in place and install the
#                           package (editable, no dependency downloads) with its
#                           `vramancer` console script
#   ./install.sh --check    only report what the build needs and whether it is there
#
# Needs: Python >= 3.10 with PyTorch built for CUDA 12.8+, nvcc 12.8+ (sm_100a),
# g++ with C++17, pybind11, ninja.  Optional: fastapi + uvicorn (API server),
# prometheus_client (metrics), nvidia-ml-py (GPU monitor), transformers (HF backend).
set -euo pipefail
cd "$(dirname "$0")"
PY=${PYTHON:-python3}

ok=1
say() { printf '%-28s %s\n' "$1" "$2"; }
if $PY -c 'import sys; sys.exit(0 if sys.version_info >= (3, 10) else 1)' 2>/dev/null; then
  say "python" "$($PY -c 'import sys; print(sys.version.split()[0])')"
else
  say "python" "missing or older than 3.10"; ok=0
fi
if $PY -c 'import torch' 2>/dev/null; then
  say "torch" "$($PY -c 'import torch; print(torch.__version__, "cuda", torch.version.cuda)')"
else
  say "torch" "missing"; ok=0
fi
NVCC=${NVCC:-$(command -v nvcc || echo /usr/local/cuda/bin/nvcc)}
if [ -x "$NVCC" ]; then
  say "nvcc" "$("$NVCC" --version | grep -o 'release [0-9.]*')"
else
  say "nvcc" "missing (set NVCC=...)"; ok=0
fi
for m in pybind11 ninja; do
  if $PY -c "import $m" 2>/dev/null; then say "$m" "ok"; else say "$m" "missing"; ok=0; fi
done
for m in fastapi uvicorn prometheus_client pynvml transformers; do
  if $PY -c "import $m" 2>/dev/null; then say "$m (optional)" "ok"; else say "$m (optional)" "not installed"; fi
done
if $PY -c 'import torch; import sys; sys.exit(0 if torch.cuda.is_available() else 1)' 2>/dev/null; then
  say "GPU" "$($PY -c 'import torch; p = torch.cuda.get_device_properties(0); print(p.name, "sm_%d%d" % (p.major, p.minor))')"
else
  say "GPU" "none visible (the build still works; kernels need a B200 at run time)"
fi
[ "${1:-}" = "--check" ] && exit $((1 - ok))
[ "$ok" = 1 ] || { echo "missing requirements: see above" >&2; exit 1; }

$PY setup.py build_ext --inplace
$PY -m pip install --no-deps --no-build-isolation -e . >/dev/null
$PY -c 'import vramancer_b200._C, vramancer_b200._runtime; print("vramancer_b200 built and installed")'
echo "next: vramancer doctor | vramancer quickstart | python -m pytest tests -m 'not gpu' -q"
