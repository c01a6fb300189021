"""Pin the CPU oracle against golden vectors produced by the reference itself
(tests/golden/make_golden.py).  CPU only."""
import numpy as np
import pytest

from oracle import oracle as orc

from .golden_data import GOLDEN, PACK_SHAPES, LAYER_NAMES, layer_from_golden


@pytest.mark.parametrize("shape", PACK_SHAPES)
@pytest.mark.parametrize("method", ["lsb_first", "half2"])
def test_pack_matches_reference(shape, method):
    rows, cols = shape
    signs = GOLDEN[f"pack_{rows}x{cols}_signs"]
    np.testing.assert_array_equal(orc.pack(signs, method), GOLDEN[f"pack_{rows}x{cols}_{method}"])


@pytest.mark.parametrize("shape", PACK_SHAPES)
@pytest.mark.parametrize("method", ["lsb_first", "half2"])
def test_unpack_matches_reference_with_garbage_padding(shape, method):
    rows, cols = shape
    words = GOLDEN[f"unpack_{rows}x{cols}_words"]
    np.testing.assert_array_equal(orc.unpack(words, shape, method), GOLDEN[f"unpack_{rows}x{cols}_{method}"])


def test_pack_rejects_non_sign_values_and_bad_dtype():
    with pytest.raises(ValueError):
        orc.pack(np.array([[1, 0, -1]], dtype=np.int8))
    with pytest.raises(TypeError):
        orc.pack(np.ones((2, 2), dtype=np.int32))
    with pytest.raises(ValueError):
        orc.pack(np.ones((2, 2), dtype=np.int8), "msb_first")
    with pytest.raises(ValueError):
        orc.unpack(np.zeros((2, 3), dtype=np.int32), (2, 33))


@pytest.mark.parametrize("name", LAYER_NAMES)
@pytest.mark.parametrize("method", ["lsb_first", "half2"])
def test_layer_forward_matches_reference(name, method):
    L = layer_from_golden(name)
    np.testing.assert_array_equal(orc.pack(L.V, method), GOLDEN[f"layer_{name}_V_{method}"])
    np.testing.assert_array_equal(orc.pack(L.U, method), GOLDEN[f"layer_{name}_U_{method}"])
    y = L.reference(method)
    # the reference ran in float32; the oracle accumulates in float64
    assert orc.rel_l2(y, GOLDEN[f"layer_{name}_y"]) < 2e-6


def test_config0_full_size_layer_pinned():
    seed, out_f, in_f, rank, batch = (int(v) for v in GOLDEN["cfg0_meta"])
    L = orc.make_layer(seed, out_f, in_f, rank, batch, "f16", False)
    for m in ("lsb_first", "half2"):
        vb, ub = L.packed(m)
        assert orc.sha256(vb) == bytes(GOLDEN[f"cfg0_V_{m}_sha256"]).decode()
        assert orc.sha256(ub) == bytes(GOLDEN[f"cfg0_U_{m}_sha256"]).decode()
    y = L.reference("half2")
    assert orc.rel_l2(y, GOLDEN["cfg0_y"]) < 2e-6


def test_state_dict_packing_format():
    U = orc.random_signs(77, 7, 3)
    V = orc.random_signs(78, 3, 5)
    np.testing.assert_array_equal(orc.pack(U, "lsb_first"), GOLDEN["sd_U_packed"])
    np.testing.assert_array_equal(orc.pack(V, "lsb_first"), GOLDEN["sd_V_packed"])
    np.testing.assert_array_equal(GOLDEN["sd_U_shape"], [7, 3])
    np.testing.assert_array_equal(GOLDEN["sd_V_shape"], [3, 5])


def test_generator_is_deterministic():
    a = orc.random_normal(5, 1000, 3)
    b = orc.random_normal(5, 1000, 3)
    np.testing.assert_array_equal(a, b)
    assert abs(a.mean()) < 0.1 and 0.9 < a.std() < 1.1
    s = orc.random_signs(9, 100, 100)
    assert set(np.unique(s)) == {-1, 1} and abs(s.mean()) < 0.05


@pytest.mark.parametrize("name", LAYER_NAMES)
def test_dense_float64_form_matches_packed_oracle(name):
    L = layer_from_golden(name)
    y = orc.forward_dense(L.x, L.s2, L.V, L.smid, L.U, L.s1)
    assert orc.rel_l2(y, L.reference("lsb_first")) < 1e-12
    assert orc.rel_l2(y, GOLDEN[f"layer_{name}_y"]) < 2e-6
