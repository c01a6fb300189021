"""Sign packing on the GPU: bit-exact against the reference's own outputs (golden
vectors) and the oracle, through the C ABI and through the torch ops."""
import ctypes

import numpy as np
import pytest
import torch

import nanoquant_b200 as nq
from nanoquant_b200 import _lib
from oracle import oracle as orc

from .golden_data import GOLDEN, PACK_SHAPES
from .nq_testutil import ptr, stream_ptr

pytestmark = pytest.mark.gpu
ORDER = {"lsb_first": _lib.NQ_BITS_LSB_FIRST, "half2": _lib.NQ_BITS_HALF2}


def capi_pack(signs: torch.Tensor, method: str, count=None):
    rows, cols = signs.shape
    out = torch.empty(rows, (cols + 31) // 32, dtype=torch.int32, device="cuda")
    _lib.check(_lib.cuda_lib().nq_pack_signs(ptr(signs), rows, cols, ORDER[method], ptr(out), ptr(count),
                                             stream_ptr()))
    return out


@pytest.mark.parametrize("shape", PACK_SHAPES)
@pytest.mark.parametrize("method", ["lsb_first", "half2"])
def test_pack_golden_capi(shape, method):
    rows, cols = shape
    s = torch.from_numpy(GOLDEN[f"pack_{rows}x{cols}_signs"]).cuda()
    out = capi_pack(s, method)
    np.testing.assert_array_equal(out.cpu().numpy(), GOLDEN[f"pack_{rows}x{cols}_{method}"])


@pytest.mark.parametrize("shape", PACK_SHAPES)
@pytest.mark.parametrize("method", ["lsb_first", "half2"])
def test_unpack_golden_with_garbage_padding(shape, method):
    rows, cols = shape
    w = torch.from_numpy(GOLDEN[f"unpack_{rows}x{cols}_words"]).cuda()
    out = nq.unpack_binary_gemv(w, (rows, cols), method)
    np.testing.assert_array_equal(out.cpu().numpy(), GOLDEN[f"unpack_{rows}x{cols}_{method}"])


@pytest.mark.parametrize("method", ["lsb_first", "half2"])
def test_pack_full_size_config0_hash(method):
    seed, out_f, in_f, rank, _ = (int(v) for v in GOLDEN["cfg0_meta"])
    L = orc.make_layer(seed, out_f, in_f, rank, 1, "f16")
    v = nq.pack_binary_gemv(torch.from_numpy(L.V).cuda(), method).cpu().numpy()
    u = nq.pack_binary_gemv(torch.from_numpy(L.U).cuda(), method).cpu().numpy()
    assert orc.sha256(v) == bytes(GOLDEN[f"cfg0_V_{method}_sha256"]).decode()
    assert orc.sha256(u) == bytes(GOLDEN[f"cfg0_U_{method}_sha256"]).decode()


@pytest.mark.parametrize("shape", [(2054, 11008), (11008, 2054), (4096, 1126), (1, 1), (3, 4097), (257, 63)])
def test_pack_unpack_roundtrip_and_oracle(shape):
    rows, cols = shape
    s = orc.random_signs(rows * 7 + cols, rows, cols)
    st = torch.from_numpy(s).cuda()
    for method in ("lsb_first", "half2"):
        p = nq.pack_binary_gemv(st, method)
        np.testing.assert_array_equal(p.cpu().numpy(), orc.pack(s, method))
        back = nq.unpack_binary_gemv(p, shape, method)
        assert torch.equal(back, st)


def test_pack_unaligned_view_uses_scalar_path():
    s = orc.random_signs(5, 9, 77)
    big = torch.from_numpy(np.concatenate([np.ones((9, 3), np.int8), s], axis=1)).cuda()
    view = big[:, 3:]  # non-contiguous view: the op copies it contiguous first
    np.testing.assert_array_equal(nq.pack_binary_gemv(view, "half2").cpu().numpy(), orc.pack(s, "half2"))


def test_pack_counts_invalid_values():
    s = torch.from_numpy(orc.random_signs(3, 4, 40)).cuda()
    s[1, 5] = 0
    s[2, 39] = 3
    count = torch.zeros(1, dtype=torch.int32, device="cuda")
    capi_pack(s, "lsb_first", count)
    torch.cuda.synchronize()
    assert int(count.item()) == 2
    with pytest.raises(ValueError):
        nq.pack_binary_gemv(s, "lsb_first", check=True)


@pytest.mark.parametrize("shape", [(33, 65), (1126, 4096), (7, 1)])
def test_repack_between_orders(shape):
    rows, cols = shape
    s = orc.random_signs(11, rows, cols)
    lsb = torch.from_numpy(orc.pack(s, "lsb_first")).cuda()
    h2 = nq.repack_binary(lsb, cols, "lsb_first", "half2")
    np.testing.assert_array_equal(h2.cpu().numpy(), orc.pack(s, "half2"))
    back = nq.repack_binary(h2, cols, "half2", "lsb_first")
    assert torch.equal(back, lsb)


def test_repack_clears_garbage_padding():
    w = torch.from_numpy(GOLDEN["unpack_33x65_words"]).cuda()
    h2 = nq.repack_binary(w, 65, "lsb_first", "half2")
    expect = orc.pack(GOLDEN["unpack_33x65_lsb_first"], "half2")
    np.testing.assert_array_equal(h2.cpu().numpy(), expect)
