#!/usr/bin/env bash
# Compiles the reference's own CUDA kernel (sm89_cuda.cu, its C-ABI launcher
# launch_qsa_cuda, sm89_cuda.cu:232-301) for sm_100a as a shared library in
# oracle/_ref/, exactly as its header describes ("Shared library (for Python /
# PyTorch ctypes)", sm89_cuda.cu:21-22) with the standalone main() left out.
#
# TEST INFRASTRUCTURE ONLY: the GPU comparator tests load it to check the
# build against the reference's fastest kernel on the same B200. It is built
# from the reference checkout where it lies ($QSA_REFERENCE_DIR, else a
# directory named "reference" beside this repository's own directory); no
# reference source is copied into this repository.
set -euo pipefail
here="$(cd "$(dirname "${BASH_SOURCE[0]}")" && pwd)"
ref="${QSA_REFERENCE_DIR:-$(dirname "$(dirname "$here")")/reference}"
src="$ref/sm89_cuda.cu"
if [[ ! -f "$src" ]]; then
  echo "reference source $src not found; oracle/_ref not rebuilt" >&2
  exit 0
fi
mkdir -p "$here/_ref"
nvcc="${CUDA_HOME:-/usr/local/cuda}/bin/nvcc"
"$nvcc" -O3 -gencode arch=compute_100a,code=sm_100a -lineinfo -DNO_MAIN \
  -Xcompiler -fPIC -shared "$src" -o "$here/_ref/libqsa_sm89_ref.so"
echo "built $here/_ref/libqsa_sm89_ref.so"
