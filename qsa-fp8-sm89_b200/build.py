"""Build recipe for the qsa_b200 native code (run on any machine with nvcc).

    python qsa-fp8-sm89_b200/build.py [--force] [--verbose]

Produces, inside the package directory ``qsa-fp8-sm89_b200/qsa_b200/``:

* ``libqsa_b200.so`` -- the CUDA kernels for sm_100a and the C ABI declared
  in ``include/qsa_b200.h`` (nvcc, ``-gencode arch=compute_100a,code=sm_100a``);
* ``_qsa_b200_torch.so`` -- the ``torch.ops.qsa_b200`` operators, a thin C++
  layer over that C ABI (g++ against the installed PyTorch headers).

Objects go to ``qsa-fp8-sm89_b200/_build/``. Rebuilds only what is out of date
unless ``--force`` is given. nvcc cross-compiles, so no GPU is needed.
"""

from __future__ import annotations

import argparse
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG_ROOT = Path(__file__).resolve().parent
CSRC = PKG_ROOT / "csrc"
PKG = PKG_ROOT / "qsa_b200"
BUILD = PKG_ROOT / "_build"
REPO = PKG_ROOT.parent
INCLUDE = REPO / "include"

CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC,-fvisibility=hidden", "--expt-relaxed-constexpr",
              "-Xptxas", "-warn-spills"] + ARCH

CU_SOURCES = ["qsa_capi.cu", "qsa_decode_tc.cu", "qsa_decode_simt.cu", "qsa_noalloc.cu", "qsa_cache_write.cu",
              "qsa_topk.cu"]
HEADERS = ["qsa_common.cuh", "qsa_internal.h"]

LIB = PKG / "libqsa_b200.so"
TORCH_EXT = PKG / "_qsa_b200_torch.so"


def _run(cmd, verbose):
    if verbose:
        print(" ".join(str(c) for c in cmd), flush=True)
    subprocess.run([str(c) for c in cmd], check=True)


def _stale(target: Path, deps) -> bool:
    if not target.exists():
        return True
    t = target.stat().st_mtime
    return any(Path(d).stat().st_mtime > t for d in deps)


def build_lib(force=False, verbose=False) -> Path:
    BUILD.mkdir(exist_ok=True)
    PKG.mkdir(exist_ok=True)
    headers = [CSRC / h for h in HEADERS] + sorted(INCLUDE.glob("*.h"))
    objs = []
    for src in CU_SOURCES:
        obj = BUILD / (Path(src).stem + ".o")
        if force or _stale(obj, [CSRC / src] + headers + [Path(__file__)]):
            _run([NVCC, *NVCC_FLAGS, "-I", INCLUDE, "-c", CSRC / src, "-o", obj], verbose)
        objs.append(obj)
    if force or _stale(LIB, objs):
        tmp = BUILD / LIB.name
        _run([NVCC, *ARCH, "-shared", "-Xcompiler", "-fPIC", *objs, "-o", tmp], verbose)
        shutil.copy2(tmp, LIB)
    return LIB


def _torch_flags():
    import torch
    from torch.utils import cpp_extension

    inc = cpp_extension.include_paths()
    libdir = os.path.join(os.path.dirname(torch.__file__), "lib")
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    return inc, libdir, abi


def build_torch_ext(force=False, verbose=False) -> Path:
    src = CSRC / "qsa_torch_ext.cpp"
    if not (force or _stale(TORCH_EXT, [src, INCLUDE / "qsa_b200.h", LIB, Path(__file__)])):
        return TORCH_EXT
    inc, libdir, abi = _torch_flags()
    tmp = BUILD / TORCH_EXT.name
    cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
           *[f"-I{p}" for p in inc], f"-I{CUDA_HOME}/include", f"-I{INCLUDE}",
           src, "-o", tmp,
           f"-L{libdir}", "-lc10", "-lc10_cuda", "-ltorch_cpu", "-ltorch",
           f"-L{PKG}", "-lqsa_b200",
           f"-Wl,-rpath,{libdir}", "-Wl,-rpath,$ORIGIN"]
    _run(cmd, verbose)
    shutil.copy2(tmp, TORCH_EXT)
    return TORCH_EXT


def build(force=False, verbose=False):
    build_lib(force, verbose)
    build_torch_ext(force, verbose)
    return LIB, TORCH_EXT


def main(argv=None):
    ap = argparse.ArgumentParser(description=__doc__.splitlines()[0])
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--verbose", action="store_true")
    args = ap.parse_args(argv)
    lib, ext = build(args.force, args.verbose)
    print(f"built {lib}\nbuilt {ext}")


if __name__ == "__main__":
    sys.exit(main())
