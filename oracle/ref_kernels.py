"""The reference's own CUDA kernels, built from its sources by oracle/build_ref.py.

Test and measurement infrastructure, not product.  Two uses of its decode GEMV
(``binary_kernels::nanoquant_dyn_forward``, kernel/cuda/gemv_kernel.cu:308-429):

* a checker: ``python -m oracle.ref_kernels <in.npz> <out.npz>`` runs it on the packed inputs of
  the file and writes its outputs, so the GPU tests compare this package's GEMV with the
  reference's on identical words;
* the reference arm of ``bench.py --impl reference --layer``, which times it on the same GPU.

The reference's Marlin GEMM (``marlin_nanoquant_forward``, gemm.cpp:112-122) is built into the
same library but never run: compiled for sm_100a it stopped with "an illegal instruction was
encountered" on a B200 on inputs that satisfy its host-side shape checks, so it stays off the GPU.

The library registers the op namespace ``binary_kernels``, which this package registers too, so
``load()`` refuses to run in a process that has this package's libraries mapped: callers run it in
a process of its own.
"""
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB = os.path.join(HERE, "_ref", "binary_kernels_ref.so")

# the reference module's launch configuration for its GEMV (modules/linear.py:210-219)
GEMV_KWARGS = dict(num_thread_stage1=128, num_thread_stage2=128, num_row_per_warp_stage1=2,
                   num_row_per_warp_stage2=2, num_acc_stage1=1, num_acc_stage2=1, num_pipeline_stage1=8,
                   num_pipeline_stage2=8)
GEMV_ROWS_PER_CTA = 8  # num_thread / 32 * num_row_per_warp


def available() -> bool:
    return os.path.isfile(LIB)


def _repo_libraries_mapped():
    pkg = os.path.join(os.path.dirname(HERE), "nanoquant_b200") + os.sep
    try:
        with open("/proc/self/maps") as f:
            return sorted({ln.split()[-1] for ln in f if ".so" in ln and ln.split()[-1].startswith(pkg)})
    except OSError:
        return []


def load():
    """torch.ops.binary_kernels of the reference library (loaded once)."""
    import torch
    mapped = _repo_libraries_mapped()
    if mapped:
        raise RuntimeError(f"the reference kernels share the binary_kernels namespace with {mapped}; "
                           "run them in a process that has not imported nanoquant_b200")
    if not available():
        raise FileNotFoundError(f"{LIB} is not built (python oracle/build_ref.py)")
    if not getattr(load, "done", False):
        torch.ops.load_library(LIB)
        load.done = True
    return torch.ops.binary_kernels


def gemv_shape_ok(out_f: int, in_f: int, rank: int) -> bool:
    """Shapes the reference GEMV handles without reading or writing out of bounds: every row
    block full (rank and out multiples of 8 rows per CTA) and whole words and uint4 loads along
    both reductions (in and rank multiples of 32; gemv_kernel.cu:72-73, 166-167)."""
    return rank % 32 == 0 and in_f % 32 == 0 and rank % GEMV_ROWS_PER_CTA == 0 and out_f % GEMV_ROWS_PER_CTA == 0


def gemv(ops, x, s2, v_half2, smid, u_half2, s1):
    """The reference module's kernel call (modules/linear.py:155-164): its op takes the module's
    V planes as ``Ubits`` and U planes as ``Vbits``."""
    return ops.nanoquant_dyn_forward(x, s2, v_half2, smid, u_half2, s1, **GEMV_KWARGS)


def run_file(src: str, dst: str) -> None:
    """Run every GEMV case of ``src`` (gemv_<k>_* arrays) and save the outputs."""
    import torch
    ops = load()
    d = dict(np.load(src))
    out = {}
    dev = torch.device("cuda", 0)

    def t(a, dtype=None):
        v = torch.from_numpy(np.ascontiguousarray(a)).to(dev)
        return v.to(dtype) if dtype is not None else v

    for key in sorted({k.split("_")[1] for k in d if k.startswith("gemv_")}):
        p = f"gemv_{key}_"
        out_f, in_f = int(d[p + "s1"].size), int(d[p + "s2"].size)
        if not gemv_shape_ok(out_f, in_f, int(d[p + "vb"].shape[0])):
            raise ValueError(f"case {key}: a shape the reference GEMV does not handle in bounds")
        td = torch.float16 if int(d[p + "dtype"][0]) == 0 else torch.bfloat16
        smid = t(d[p + "smid"], td) if p + "smid" in d else None
        y = gemv(ops, t(d[p + "x"], td), t(d[p + "s2"], td), t(d[p + "vb"]), smid, t(d[p + "ub"]), t(d[p + "s1"], td))
        out[p + "y"] = y.float().cpu().numpy()
    torch.cuda.synchronize(dev)
    np.savez(dst, **out)


if __name__ == "__main__":
    run_file(sys.argv[1], sys.argv[2])
