"""Loader for the committed golden vectors (tests/golden/golden_v1.npz)."""
import os

import numpy as np

from oracle import oracle as orc

_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_v1.npz")
GOLDEN = dict(np.load(_PATH))

PACK_SHAPES = sorted({tuple(int(v) for v in k[len("pack_"):-len("_signs")].split("x"))
                      for k in GOLDEN if k.startswith("pack_") and k.endswith("_signs")})
LAYER_NAMES = sorted(k[len("layer_"):-len("_meta")] for k in GOLDEN if k.startswith("layer_") and k.endswith("_meta"))
_DTYPES = {"tiny": "f32", "odd_mid": "f32", "ragged_b8": "f16", "attn_small": "bf16"}


def layer_from_golden(name: str) -> orc.Layer:
    out_f, in_f, rank, batch, mid, seed = (int(v) for v in GOLDEN[f"layer_{name}_meta"])
    return orc.make_layer(seed, out_f, in_f, rank, batch, _DTYPES[name], bool(mid))
