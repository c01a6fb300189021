"""Build recipe for the in-tree native libraries (no JIT cache, nothing pip-installed).

* ``_build/libnq_b200.so`` -- the CUDA kernels behind the C ABI of include/nq_b200.h,
  compiled by nvcc for sm_100a only (``-gencode arch=compute_100a,code=sm_100a``), CUDA
  runtime linked statically, so it loads without PyTorch.
* ``_build/libnq_torch.so`` -- the PyTorch dispatcher registrations (torch_ops.cpp),
  linked against libnq_b200.so with an $ORIGIN rpath; loaded with torch.ops.load_library.

Both are rebuilt only when a source is newer than the library.
"""
from __future__ import annotations

import glob
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
OUT = os.path.join(HERE, "_build")
INCLUDE = os.path.join(os.path.dirname(HERE), "include")
CUDA_HOME = os.environ.get("CUDA_HOME", "/usr/local/cuda")
NVCC = os.path.join(CUDA_HOME, "bin", "nvcc")
ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
CUDA_LIB = os.path.join(OUT, "libnq_b200.so")
TORCH_LIB = os.path.join(OUT, "libnq_torch.so")


def _stale(target: str, sources) -> bool:
    if not os.path.exists(target):
        return True
    t = os.path.getmtime(target)
    return any(os.path.getmtime(s) > t for s in sources)


def _run(cmd, verbose):
    if verbose:
        print(" ".join(cmd), file=sys.stderr)
    subprocess.check_call(cmd)


def build_cuda(force=False, verbose=False) -> str:
    """Compile every csrc/*.cu into libnq_b200.so.  NQ_NVCC_EXTRA (space-separated nvcc flags,
    e.g. -DNQ_GEMV_TRACE for the GEMV phase timeline) makes a debug build; the flags are
    recorded beside the library, so changing them triggers a rebuild."""
    cu = sorted(glob.glob(os.path.join(CSRC, "*.cu")))
    deps = cu + glob.glob(os.path.join(CSRC, "*.cuh")) + glob.glob(os.path.join(INCLUDE, "*.h"))
    extra = os.environ.get("NQ_NVCC_EXTRA", "").split()
    stamp = CUDA_LIB + ".flags"
    prev = open(stamp).read() if os.path.exists(stamp) else ""
    if force or _stale(CUDA_LIB, deps) or prev != " ".join(extra):
        os.makedirs(OUT, exist_ok=True)
        cmd = [NVCC, *ARCH, "-lineinfo", "-O3", "-std=c++17", "--expt-relaxed-constexpr", "-Xcompiler", "-fPIC",
               "-Xcompiler", "-fvisibility=hidden", "-shared", "-cudart", "static", "-I", INCLUDE, *extra, *cu, "-o",
               CUDA_LIB + ".tmp"]
        _run(cmd, verbose)
        os.replace(CUDA_LIB + ".tmp", CUDA_LIB)
        with open(stamp, "w") as f:
            f.write(" ".join(extra))
    return CUDA_LIB


def build_torch(force=False, verbose=False) -> str:
    import torch.utils.cpp_extension as ext
    src = os.path.join(CSRC, "torch_ops.cpp")
    deps = [src, CUDA_LIB] + glob.glob(os.path.join(INCLUDE, "*.h"))
    if force or _stale(TORCH_LIB, deps):
        os.makedirs(OUT, exist_ok=True)
        import torch
        abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
        incs = []
        for p in ext.include_paths():
            incs += ["-isystem", p]
        libdirs = ext.library_paths()
        cmd = ["g++", "-O2", "-std=c++17", "-fPIC", "-shared", f"-D_GLIBCXX_USE_CXX11_ABI={abi}",
               "-DTORCH_API_INCLUDE_EXTENSION_H", *incs, "-isystem", os.path.join(CUDA_HOME, "include"), "-I",
               INCLUDE, src, "-o", TORCH_LIB + ".tmp", "-L", OUT, "-lnq_b200"]
        for d in libdirs:
            cmd += ["-L", d, f"-Wl,-rpath,{d}"]
        cmd += ["-lc10", "-ltorch", "-ltorch_cpu", "-lc10_cuda", "-ltorch_cuda", "-Wl,-rpath,$ORIGIN"]
        _run(cmd, verbose)
        os.replace(TORCH_LIB + ".tmp", TORCH_LIB)
    return TORCH_LIB


def build(force=False, verbose=False):
    build_cuda(force, verbose)
    build_torch(force, verbose)
    return CUDA_LIB, TORCH_LIB


if __name__ == "__main__":
    build(force="--force" in sys.argv, verbose=True)
