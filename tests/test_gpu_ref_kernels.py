"""This package's decode GEMV against the reference's own CUDA GEMV on the same GPU and words.

The reference extension is built from its sources by oracle/build_ref.py into oracle/_ref
(skipped when it is not built).  It registers the same ``binary_kernels`` namespace as this
package, so it runs in a subprocess (``python -m oracle.ref_kernels``) on the packed inputs
written here; this process runs this package's ops of the same schema on the same words.  Both
are compared with the float64 oracle:

nanoquant_dyn_forward (gemv_kernel.cu:308-429, the reference module's launch configuration) on
half2 planes, at shapes where the reference kernel stays in bounds (rank and in multiples of 32,
full row blocks): this package within rel-L2 1e-3 (nq_testutil); the reference, which accumulates
in fp16/bf16, within 2e-2; and this package never less accurate than the reference.  The
reference's Marlin GEMM is not run (oracle/ref_kernels.py says why); this package's Marlin ops
are checked against the oracle and the reference packers' goldens in test_gpu_marlin.py.
"""
import os
import subprocess
import sys

import numpy as np
import pytest
import torch

import nanoquant_b200  # noqa: F401  (registers this package's binary_kernels ops)
from oracle import oracle as orc
from oracle import ref_kernels as rk

from .nq_testutil import assert_close_to_oracle

pytestmark = [pytest.mark.gpu,
              pytest.mark.skipif(not rk.available(), reason="reference kernels not built (oracle/build_ref.py)")]
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF_TOL = 2e-2

GEMV_CASES = [  # (out, in, rank, batch, dtype, smid)
    (4096, 4096, 1088, 1, "f16", False),    # 7B attention at the reference planner's rank
    (11008, 4096, 1600, 1, "f16", False),   # 7B gate/up
    (4096, 11008, 1600, 4, "f16", False),   # 7B down, batch 4
    (1024, 8192, 480, 1, "f16", False),     # 70B k/v
    (512, 1024, 256, 2, "bf16", True),
]


def _cases():
    data, exact = {}, {}
    for i, (out_f, in_f, r, b, dt, mid) in enumerate(GEMV_CASES):
        assert rk.gemv_shape_ok(out_f, in_f, r)
        L = orc.make_layer(900 + i, out_f, in_f, r, b, dt, with_mid=mid)
        vb, ub = L.packed("half2")
        p = f"gemv_{i}_"
        data.update({p + "x": L.x.astype(np.float32), p + "s2": L.s2, p + "s1": L.s1, p + "vb": vb, p + "ub": ub,
                     p + "dtype": np.array([0 if dt == "f16" else 1])})
        if mid:
            data[p + "smid"] = L.smid
        exact[p] = (orc.forward(L.x, L.s2, vb, r, L.smid, ub, L.s1, "half2"), dt)
    return data, exact


@pytest.fixture(scope="module")
def runs(tmp_path_factory):
    data, exact = _cases()
    d = tmp_path_factory.mktemp("refk")
    src, dst = str(d / "in.npz"), str(d / "out.npz")
    np.savez(src, **data)
    env = dict(os.environ, PYTHONPATH=ROOT)
    r = subprocess.run([sys.executable, "-m", "oracle.ref_kernels", src, dst], cwd=ROOT, env=env,
                       capture_output=True, text=True, timeout=600)
    assert r.returncode == 0, r.stderr[-3000:]
    return data, exact, dict(np.load(dst))


def _err(y, want, dt):
    """rel-L2 against the float64 result rounded once to the output type."""
    y = y.float().cpu().numpy() if isinstance(y, torch.Tensor) else y
    return orc.rel_l2(y, orc.round_to(want, dt))


def _t(a, dt=None):
    v = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return v if dt is None else v.to({"f16": torch.float16, "bf16": torch.bfloat16}[dt])


@pytest.mark.parametrize("i", range(len(GEMV_CASES)))
def test_gemv_against_reference_kernel(runs, i):
    data, exact, ref = runs
    p = f"gemv_{i}_"
    want, dt = exact[p]
    smid = _t(data[p + "smid"], dt) if p + "smid" in data else None
    ours = torch.ops.binary_kernels.nanoquant_dyn_forward(
        _t(data[p + "x"], dt), _t(data[p + "s2"], dt), _t(data[p + "vb"]), smid, _t(data[p + "ub"]),
        _t(data[p + "s1"], dt), **rk.GEMV_KWARGS)
    theirs = ref[p + "y"]
    e_ours, e_ref = _err(ours, want, dt), _err(theirs, want, dt)
    print(f"{GEMV_CASES[i]}: rel-L2 vs the rounded float64 oracle: this package {e_ours:.2e}, "
          f"reference kernel {e_ref:.2e}")
    assert_close_to_oracle(ours, want, dt)
    assert e_ref <= REF_TOL, f"the reference kernel computes another function here ({e_ref:.3e})"
    assert e_ours <= max(e_ref, 1e-3)
