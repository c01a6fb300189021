"""tcgen05 prefill GEMM parity on the GPU.

Tolerance: rel-L2 <= 1e-3 per layer against the float64 oracle rounded to the output
dtype (precise mode: T kept as a bf16 hi/lo pair).  Fast mode rounds T once to bf16, as
the reference's GEMM does with its intermediate; it is checked against the oracle with
the same rounding point applied (orc.forward_dense(round_t="bf16"))."""
import ctypes

import numpy as np
import pytest
import torch

from nanoquant_b200 import _lib
from oracle import oracle as orc

from .golden_data import GOLDEN, layer_from_golden
from .nq_testutil import NQ_DT, DeviceLayer, assert_close_to_oracle, ptr, stream_ptr, workspace_status

pytestmark = pytest.mark.gpu


def capi_gemm(d: DeviceLayer, precise: bool = True):
    lib = _lib.cuda_lib()
    x = d.x
    m, in_f = x.shape
    out_f = d.s1.numel()
    y = torch.empty(m, out_f, dtype=x.dtype, device=x.device)
    wsb = lib.nq_gemm_workspace_bytes(m, d.L.rank)
    ws = torch.zeros(wsb, dtype=torch.uint8, device=x.device)
    st = lib.nq_gemm(NQ_DT[d.dtype], ptr(x), m, in_f, ptr(d.s2), ptr(d.vb), d.L.rank, ptr(d.smid), ptr(d.ub),
                     out_f, ptr(d.s1), 1 if precise else 0, ptr(y), ptr(ws), wsb, stream_ptr())
    _lib.check(st)
    return y, ws


def dense_ref(d: DeviceLayer, round_t=None):
    return orc.forward_dense(d.xr, d.s2r, d.L.V, d.smidr, d.L.U, d.s1r, round_t=round_t)


@pytest.mark.parametrize("name,dtype", [("ragged_b8", "f16"), ("attn_small", "bf16")])
def test_gemm_reference_golden(name, dtype):
    d = DeviceLayer(layer_from_golden(name), dtype)
    y, ws = capi_gemm(d)
    assert_close_to_oracle(y, GOLDEN[f"layer_{name}_y"].astype(np.float64), dtype)
    assert workspace_status(ws) == 0


@pytest.mark.parametrize("shape", [(4096, 4096, 1126), (11008, 4096, 2054), (4096, 11008, 2054)])
@pytest.mark.parametrize("m", [128, 512])
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_gemm_llama_shapes_precise(shape, m, dtype):
    out_f, in_f, rank = shape
    L = orc.make_layer(m + rank, out_f, in_f, rank, m, dtype, with_mid=(m == 128))
    d = DeviceLayer(L, dtype)
    y, ws = capi_gemm(d, precise=True)
    assert_close_to_oracle(y, dense_ref(d), dtype)
    assert workspace_status(ws) == 0


@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_gemm_fast_mode_matches_dtype_intermediate(dtype):
    """Fast mode rounds T once to the layer dtype (the reference's fp16/bf16 intermediate)."""
    L = orc.make_layer(3, 4096, 4096, 1126, 256, dtype)
    d = DeviceLayer(L, dtype)
    y, _ = capi_gemm(d, precise=False)
    assert_close_to_oracle(y, dense_ref(d, round_t=dtype), dtype)
    if dtype == "f16":  # an fp16 intermediate is also within the per-layer bound of the exact result
        assert_close_to_oracle(y, dense_ref(d), dtype)


@pytest.mark.parametrize("shape", [(7, 8, 3, 1), (100, 64, 33, 5), (130, 96, 47, 130), (1000, 200, 96, 77),
                                   (33, 1024, 300, 257), (4096, 11008, 2054, 1),
                                   (1000, 2000, 300, 77)])  # split-K over a ragged K tail
@pytest.mark.parametrize("dtype", ["bf16", "f16"])
def test_gemm_ragged_shapes(shape, dtype):
    out_f, in_f, rank, m = shape
    L = orc.make_layer(sum(shape), out_f, in_f, rank, m, dtype, with_mid=True)
    d = DeviceLayer(L, dtype)
    y, ws = capi_gemm(d, precise=True)
    assert_close_to_oracle(y, dense_ref(d), dtype)
    assert workspace_status(ws) == 0


@pytest.mark.parametrize("shape,dtype,precise", [((4096, 4096, 2054, 2048), "bf16", True),
                                                 ((4096, 4096, 2054, 2048), "f16", False),
                                                 ((4000, 4096, 2050, 2000), "bf16", True)])
def test_gemm_wide_tiles(shape, dtype, precise):
    """Shapes whose output tiles fill the GPU run 256-column tiles in both stages (ragged M and N
    included)."""
    out_f, in_f, rank, m = shape
    L = orc.make_layer(m + rank, out_f, in_f, rank, m, dtype, with_mid=True)
    d = DeviceLayer(L, dtype)
    y, ws = capi_gemm(d, precise=precise)
    assert_close_to_oracle(y, dense_ref(d, round_t=None if precise else dtype), dtype)
    assert workspace_status(ws) == 0


def test_gemm_m2048_full_prefill_shape():
    L = orc.make_layer(2048, 4096, 4096, 1126, 2048, "bf16")
    d = DeviceLayer(L, "bf16")
    y, _ = capi_gemm(d)
    assert_close_to_oracle(y, dense_ref(d), "bf16")


def test_gemm_rejects_unaligned_in_features():
    lib = _lib.cuda_lib()
    fake = ctypes.c_void_p(0x10000)
    st = lib.nq_gemm(0, fake, 4, 70, fake, fake, 16, None, fake, 32, fake, 1, fake, fake, 1 << 20, None)
    assert st == _lib.NQ_ERR_UNSUPPORTED


def test_reference_op_prefill_dispatches_to_gemm():
    """The reference GEMV op called with a prefill-sized x runs the GEMM and agrees with
    the explicit GEMV run on the same rows."""
    L = orc.make_layer(11, 4096, 4096, 1126, 64, "f16", with_mid=True)
    d = DeviceLayer(L, "f16")
    y = torch.ops.binary_kernels.nanoquant_dyn_forward(d.x, d.s2, d.vb, d.smid, d.ub, d.s1, 128, 128, 2, 2, 1, 1,
                                                       8, 8)
    assert_close_to_oracle(y, dense_ref(d), "f16")
    y2 = torch.ops.nq_b200.gemv(d.x, d.s2, d.vb, d.smid, d.ub, d.s1)
    assert orc.rel_l2(y.float().cpu().numpy(), y2.float().cpu().numpy()) < 1e-3
