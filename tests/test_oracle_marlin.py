"""Pins the oracle's Marlin restatement (oracle/oracle.py: pack_marlin, unpack_marlin, the scale
permutations and pack_marlin_fused) to golden vectors produced by the reference's own
pack_binary_marlin / pack_binary_marlin_fused (tests/golden/make_golden_marlin.py): bit-exact."""
import os

import numpy as np
import pytest

from oracle import oracle as orc

G = dict(np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_marlin_v1.npz")))
ONEBIT = sorted({k[len("onebit_"):-len("_signs")] for k in G if k.startswith("onebit_") and k.endswith("_signs")})
FUSED = sorted({k[len("fused_"):-len("_V")] for k in G if k.startswith("fused_") and k.endswith("_V")})


@pytest.mark.parametrize("key", ONEBIT)
def test_marlin_pack_matches_reference(key):
    w = G[f"onebit_{key}_signs"]
    assert np.array_equal(orc.pack_marlin(w), G[f"onebit_{key}_bits"])
    assert np.array_equal(orc.unpack_marlin(G[f"onebit_{key}_bits"], *w.shape), w)
    assert np.array_equal(orc.marlin_perm_in(G[f"onebit_{key}_sin"]), G[f"onebit_{key}_sin_perm"])
    assert np.array_equal(orc.marlin_perm_out(G[f"onebit_{key}_sout"]), G[f"onebit_{key}_sout_perm"])
    assert w.shape[0] // 128 * 32 == int(G[f"onebit_{key}_ws"][0])


@pytest.mark.parametrize("key", FUSED)
def test_marlin_fused_pack_matches_reference(key):
    vb, ub, s1, s2, s3, ws = orc.pack_marlin_fused(G[f"fused_{key}_V"], G[f"fused_{key}_U"], G[f"fused_{key}_sg"],
                                                   G[f"fused_{key}_sl"], G[f"fused_{key}_sh"])
    assert np.array_equal(vb, G[f"fused_{key}_vbits"])
    assert np.array_equal(ub, G[f"fused_{key}_ubits"])
    for a, b in ((s1, "s1"), (s2, "s2"), (s3, "s3")):
        assert np.array_equal(a.astype(np.float32), G[f"fused_{key}_{b}"])
    assert ws == int(G[f"fused_{key}_ws_numel"][0])


def test_marlin_rejects_unaligned_shapes():
    with pytest.raises(ValueError):
        orc.pack_marlin(np.ones((32, 16), dtype=np.int8))


def test_reference_kernels_refuse_a_process_with_this_package():
    """The reference extension registers the same op namespace: it never loads beside this package."""
    import nanoquant_b200  # noqa: F401
    from oracle import ref_kernels as rk
    if not rk._repo_libraries_mapped():
        pytest.skip("this package's libraries are not mapped in this process")
    with pytest.raises(RuntimeError, match="binary_kernels namespace"):
        rk.load()
