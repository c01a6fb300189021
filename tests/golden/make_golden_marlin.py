"""Generate golden vectors of the reference's Marlin packers by running the reference code.

Run once in a container that has the reference checkout; the output is committed next to
this script (golden_marlin_v1.npz):

    NQ_REFERENCE_SRC=<reference>/src python tests/golden/make_golden_marlin.py

Reference functions exercised (paths inside the reference project):
  * kernel/utils.py:186-214  pack_binary_marlin (alias marlin_onebit_packer): sign words in the
    Marlin tile order, permuted input / output scales, workspace size
  * kernel/utils.py:217-284  pack_binary_marlin_fused (alias marlin_nanoquant_packer): both
    factors of a layer, rank padded to a multiple of 256 with +1 signs and zero scale_mid

Inputs come from the splitmix64 generator in oracle/oracle.py.
"""
import os
import sys

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.environ.get("NQ_REFERENCE_SRC", os.path.join(os.path.dirname(REPO), "reference", "src")))

import numpy as np  # noqa: E402
import torch  # noqa: E402

from nanoquant.kernel.utils import pack_binary_marlin, pack_binary_marlin_fused  # noqa: E402

from oracle import oracle as orc  # noqa: E402

ONEBIT = [(64, 16), (128, 48), (192, 256), (256, 1024), (64, 4096)]  # weight [N_out, K]
FUSED = [  # (in, rank, out): the reference pads rank to 256 but needs rank % 32 == 0 (its planner's ranks
    (256, 96, 128),   # are multiples of 32; utils.py:251-262 rounds only a local copy of R to 32)
    (512, 288, 256),
    (1024, 512, 192),
]


def main():
    out = {}
    for i, (n, k) in enumerate(ONEBIT):
        w = orc.random_signs(3000 + i, n, k)
        s_in = orc.random_normal(3100 + i, k).astype(np.float32)
        s_out = orc.random_normal(3200 + i, n).astype(np.float32)
        bits, si, so, ws = pack_binary_marlin(torch.from_numpy(w), torch.from_numpy(s_in), torch.from_numpy(s_out))
        key = f"onebit_{n}x{k}"
        out[f"{key}_signs"] = w
        out[f"{key}_sin"] = s_in
        out[f"{key}_sout"] = s_out
        out[f"{key}_bits"] = bits.numpy()
        out[f"{key}_sin_perm"] = si.numpy()
        out[f"{key}_sout_perm"] = so.numpy()
        out[f"{key}_ws"] = np.array([ws], dtype=np.int64)
    for i, (n_in, r, n_out) in enumerate(FUSED):
        V = orc.random_signs(4000 + i, r, n_in)   # module layout [rank, in]
        U = orc.random_signs(4100 + i, n_out, r)  # module layout [out, rank]
        sg = orc.random_normal(4200 + i, n_in).astype(np.float32)
        sl = np.abs(orc.random_normal(4300 + i, r)).astype(np.float32)
        sh = orc.random_normal(4400 + i, n_out).astype(np.float32)
        t = lambda a: torch.from_numpy(np.ascontiguousarray(a))  # noqa: E731
        # the reference's _prepare_kernel("gemm") passes V.T [in, rank] and U.T [rank, out]
        vb, ub, s1, s2, s3, ws = pack_binary_marlin_fused(t(V.T), t(U.T), t(sg), t(sl), t(sh))
        key = f"fused_{n_in}_{r}_{n_out}"
        out[f"{key}_V"] = V
        out[f"{key}_U"] = U
        out[f"{key}_sg"] = sg
        out[f"{key}_sl"] = sl
        out[f"{key}_sh"] = sh
        out[f"{key}_vbits"] = vb.numpy()
        out[f"{key}_ubits"] = ub.numpy()
        out[f"{key}_s1"] = s1.numpy()
        out[f"{key}_s2"] = s2.numpy()
        out[f"{key}_s3"] = s3.numpy()
        out[f"{key}_ws_numel"] = np.array([ws.numel()], dtype=np.int64)
    path = os.path.join(HERE, "golden_marlin_v1.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
