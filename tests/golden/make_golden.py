"""Generate golden vectors by running the reference NanoQuant code itself.

Run once in a container that has the reference checkout (it cannot run on the GPU
box, which has no reference tree); the outputs are committed next to this script:

    NQ_REFERENCE_SRC=<reference>/src python tests/golden/make_golden.py

Reference functions exercised (paths inside the reference project):
  * kernel/utils.py:51-113   pack_binary_gemv   (both bit orders, padded tails)
  * kernel/utils.py:116-183  unpack_binary_gemv (including garbage padding bits)
  * modules/linear.py:282-291 NanoQuantLinear._compute_forward, evaluated in float32
  * modules/linear.py:359-433 NanoQuantLinear.state_dict / load_state_dict packing

Inputs come from the splitmix64 generator in oracle/oracle.py, so the tests can
rebuild the large inputs instead of storing them; for the full-size layer only the
SHA-256 of the reference's packed planes and the float32 outputs are stored.
"""
import os
import sys

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")  # the reference packers are @torch.compile'd
HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
# the reference checkout sits beside this repository unless NQ_REFERENCE_SRC says otherwise
sys.path.insert(0, os.environ.get("NQ_REFERENCE_SRC", os.path.join(os.path.dirname(REPO), "reference", "src")))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import torch.nn as nn  # noqa: E402

from nanoquant.kernel.utils import pack_binary_gemv, unpack_binary_gemv  # noqa: E402
from nanoquant.modules.linear import NanoQuantLinear  # noqa: E402

from oracle import oracle as orc  # noqa: E402

PACK_SHAPES = [(1, 1), (3, 5), (5, 7), (7, 3), (4, 32), (4, 33), (2, 64), (17, 100), (33, 65),
               (8, 1126), (3, 2054), (64, 31)]
LAYERS = [  # (name, out, in, rank, batch, dtype, with_mid)
    ("tiny", 7, 5, 3, 1, "f32", False),
    ("odd_mid", 100, 70, 33, 3, "f32", True),
    ("ragged_b8", 130, 96, 47, 8, "f16", True),
    ("attn_small", 256, 512, 160, 2, "bf16", False),
]
FULL = dict(name="cfg0", seed=20260, out=4096, inp=4096, rank=1126, batch=1, dtype="f16")


def ref_pack(signs: np.ndarray, method: str) -> np.ndarray:
    return pack_binary_gemv(torch.from_numpy(signs), method).numpy()


def ref_forward(layer: orc.Layer) -> np.ndarray:
    """Reference dense path in float32 (module built the way the reference loader does)."""
    lin = nn.Linear(layer.in_f, layer.out_f, bias=False)
    lin.__class__ = NanoQuantLinear
    lin.init_for_inference(layer.rank, has_scale_mid=layer.smid is not None)
    f = lambda a: torch.from_numpy(np.asarray(a, dtype=np.float32))  # noqa: E731
    V = f(layer.V.astype(np.float32))
    U = f(layer.U.astype(np.float32))
    s2 = f(layer.s2).reshape(1, -1)
    s1 = f(layer.s1).reshape(1, -1)
    smid = None if layer.smid is None else f(layer.smid).reshape(1, -1)
    with torch.no_grad():
        y = lin._compute_forward(f(layer.x), V, U, s2, smid, s1)
    return y.numpy().astype(np.float32)


def main():
    out = {}
    # 1. packing / unpacking goldens
    for i, (rows, cols) in enumerate(PACK_SHAPES):
        s = orc.random_signs(1000 + i, rows, cols)
        out[f"pack_{rows}x{cols}_signs"] = s
        for m in ("lsb_first", "half2"):
            out[f"pack_{rows}x{cols}_{m}"] = ref_pack(s, m)
        # unpack of words whose padding bits are random (the reference ignores them)
        w = orc.splitmix64(2000 + i, rows * orc.words(cols)).astype(np.uint32).view(np.int32)
        w = w.reshape(rows, orc.words(cols))
        out[f"unpack_{rows}x{cols}_words"] = w
        for m in ("lsb_first", "half2"):
            u = unpack_binary_gemv(torch.from_numpy(w), (rows, cols), m).numpy()
            out[f"unpack_{rows}x{cols}_{m}"] = u

    # 2. small layers: full data
    for (name, o, n, r, b, dt, mid) in LAYERS:
        seed = len(name) * 31 + o
        L = orc.make_layer(seed, o, n, r, b, dt, mid)
        out[f"layer_{name}_meta"] = np.array([o, n, r, b, int(mid), seed], dtype=np.int64)
        out[f"layer_{name}_y"] = ref_forward(L)
        for m in ("lsb_first", "half2"):
            out[f"layer_{name}_V_{m}"] = ref_pack(L.V, m)
            out[f"layer_{name}_U_{m}"] = ref_pack(L.U, m)

    # 3. the full-size config-0 layer: hashes of reference-packed planes + outputs
    F = FULL
    L = orc.make_layer(F["seed"], F["out"], F["inp"], F["rank"], F["batch"], F["dtype"], False)
    for m in ("lsb_first", "half2"):
        out[f"cfg0_V_{m}_sha256"] = np.frombuffer(orc.sha256(ref_pack(L.V, m)).encode(), dtype=np.uint8)
        out[f"cfg0_U_{m}_sha256"] = np.frombuffer(orc.sha256(ref_pack(L.U, m)).encode(), dtype=np.uint8)
    out["cfg0_meta"] = np.array([F["seed"], F["out"], F["inp"], F["rank"], F["batch"]], dtype=np.int64)
    out["cfg0_y"] = ref_forward(L)

    # 4. state_dict round trip of the module (packed checkpoint format, lsb_first)
    lin = nn.Linear(5, 7)
    lin.__class__ = NanoQuantLinear
    lin.init_for_inference(3)
    with torch.no_grad():
        lin.U.copy_(torch.from_numpy(orc.random_signs(77, 7, 3).astype(np.float32)))
        lin.V.copy_(torch.from_numpy(orc.random_signs(78, 3, 5).astype(np.float32)))
        lin.scale_pre.fill_(1)
        lin.scale_post.fill_(1)
    sd = lin.state_dict()
    for k in ("U_packed", "V_packed", "U_shape", "V_shape"):
        out[f"sd_{k}"] = sd[k].numpy()
    out["sd_keys"] = np.array(sorted(sd.keys()))

    path = os.path.join(HERE, "golden_v1.npz")
    np.savez_compressed(path, **out)
    print(f"wrote {path}: {len(out)} arrays, {os.path.getsize(path)} bytes")


if __name__ == "__main__":
    main()
