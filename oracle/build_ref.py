"""Build the reference's own CUDA extension from its sources, for comparison on the GPU.

Test infrastructure, not product: the library built here is the reference's ``binary_kernels``
torch extension (``src/nanoquant/kernel/{pybind.cpp, cuda/gemm.cpp, cuda/gemv_kernel.cu,
cuda/gemm_kernel.cu}``, listed in ``src/nanoquant/kernel/setup.py:55-74``) compiled where the
sources lie, with the reference's own nvcc flags (``setup.py:36-52``: ``-O3 --use_fast_math
-std=c++17``) for sm_100a only.  Its own build system (setuptools ``BuildExtension``) is not run:
each source is compiled by one nvcc / g++ command against the installed torch headers and the
objects are linked into ``oracle/_ref/binary_kernels_ref.so``.  Nothing under the reference tree is
written.

The library registers the ``binary_kernels`` op namespace, the same one this package registers,
so it is only ever loaded in a process that has not imported ``nanoquant_b200`` (the reference
arm of ``bench.py`` and the subprocess of the reference-kernel GPU tests).

    python oracle/build_ref.py [--src <reference>/src/nanoquant/kernel] [--jobs 8]
"""
import argparse
import os
import subprocess
import sys
import sysconfig
from concurrent.futures import ThreadPoolExecutor

HERE = os.path.dirname(os.path.abspath(__file__))
OUT_DIR = os.path.join(HERE, "_ref")
LIB = os.path.join(OUT_DIR, "binary_kernels_ref.so")
SOURCES = ["pybind.cpp", "cuda/gemm.cpp", "cuda/gemv_kernel.cu", "cuda/gemm_kernel.cu"]
DEFAULT_SRC = os.path.join(os.path.dirname(os.path.dirname(HERE)), "reference", "src", "nanoquant", "kernel")


def _torch_flags():
    import torch
    import torch.utils.cpp_extension as ce
    inc = ce.include_paths(device_type="cuda") + [sysconfig.get_paths()["include"]]
    abi = int(torch._C._GLIBCXX_USE_CXX11_ABI)
    defs = ["-DTORCH_EXTENSION_NAME=binary_kernels", "-DTORCH_API_INCLUDE_EXTENSION_H",
            f"-D_GLIBCXX_USE_CXX11_ABI={abi}"]
    libs = ce.library_paths(device_type="cuda")
    return [f"-I{p}" for p in inc], defs, libs


def build(src_dir: str = DEFAULT_SRC, jobs: int = 8, force: bool = False) -> str:
    """Compile the reference extension into ``oracle/_ref``; returns the library path."""
    srcs = [os.path.join(src_dir, s) for s in SOURCES]
    missing = [s for s in srcs if not os.path.isfile(s)]
    if missing:
        raise FileNotFoundError(f"reference kernel sources not found: {missing}")
    if not force and os.path.isfile(LIB) and all(os.path.getmtime(LIB) >= os.path.getmtime(s) for s in srcs):
        return LIB
    os.makedirs(os.path.join(OUT_DIR, "obj"), exist_ok=True)
    inc, defs, libs = _torch_flags()
    nvcc = os.path.join(os.environ.get("CUDA_HOME", "/usr/local/cuda"), "bin", "nvcc")

    def compile_one(src):
        obj = os.path.join(OUT_DIR, "obj", os.path.basename(src) + ".o")
        if src.endswith(".cu"):
            cmd = [nvcc, "-c", src, "-o", obj, "-O3", "--use_fast_math", "-std=c++17",
                   "-gencode", "arch=compute_100a,code=sm_100a", "-Xcompiler", "-fPIC",
                   "--expt-relaxed-constexpr", "-D__CUDA_NO_HALF_OPERATORS__", "-D__CUDA_NO_HALF_CONVERSIONS__",
                   "-D__CUDA_NO_BFLOAT16_CONVERSIONS__", "-D__CUDA_NO_HALF2_OPERATORS__"] + inc + defs
        else:
            cmd = ["g++", "-c", src, "-o", obj, "-O3", "-std=c++17", "-fPIC"] + inc + defs
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError(f"compiling {src} failed:\n{r.stderr[-4000:]}")
        return obj

    with ThreadPoolExecutor(max_workers=max(1, jobs)) as ex:
        objs = list(ex.map(compile_one, srcs))
    link = ["g++", "-shared", "-o", LIB] + objs + [f"-L{p}" for p in libs] + \
           [f"-Wl,-rpath,{p}" for p in libs] + ["-lc10", "-lc10_cuda", "-ltorch", "-ltorch_cpu", "-ltorch_cuda",
                                                 "-ltorch_python", "-lcudart"]
    r = subprocess.run(link, capture_output=True, text=True)
    if r.returncode != 0:
        raise RuntimeError(f"linking {LIB} failed:\n{r.stderr[-4000:]}")
    return LIB


def main():
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--src", default=os.environ.get("NQ_REFERENCE_KERNEL_SRC", DEFAULT_SRC))
    ap.add_argument("--jobs", type=int, default=8)
    ap.add_argument("--force", action="store_true")
    a = ap.parse_args()
    print(build(a.src, a.jobs, a.force))


if __name__ == "__main__":
    sys.exit(main())
