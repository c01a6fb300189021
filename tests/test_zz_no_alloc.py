"""The allocation-free GEMV entry point (nq_gemv_static), for callers that cannot allocate
device memory -- a plugin interface that passes only input and output buffers, or a process
that must not call cudaMalloc after start-up.  It is checked through the C ABI against the
workspace entry point (nq_gemv) and the oracle, on two calls in a row, with the tolerance of
the other GEMV tests (rel-L2 <= 1e-3).  This file is collected last on purpose."""
import ctypes

import pytest
import torch

from nanoquant_b200 import _lib
from oracle import oracle as orc

from .nq_testutil import NQ_DT, DeviceLayer, assert_close_to_oracle, capi_gemv, ptr, stream_ptr

pytestmark = pytest.mark.gpu
MAX_RANK = 4096  # NQ_GEMV_STATIC_MAX_RANK in include/nq_b200.h


def capi_gemv_static(d: DeviceLayer):
    lib = _lib.cuda_lib()
    batch, in_f = d.x.shape
    out_f = d.s1.numel()
    y = torch.empty(batch, out_f, dtype=d.x.dtype, device="cuda")
    st = lib.nq_gemv_static(NQ_DT[d.dtype], ptr(d.x), batch, in_f, ptr(d.s2), ptr(d.vb), d.L.rank, ptr(d.smid),
                            ptr(d.ub), out_f, ptr(d.s1), ptr(y), stream_ptr())
    _lib.check(st)
    return y


def test_static_entry_point_matches_workspace_entry_point_twice():
    layers = [
        DeviceLayer(orc.make_layer(31, 4096, 4096, 1126, 1, "f16"), "f16"),
        DeviceLayer(orc.make_layer(32, 11008, 4096, 2054, 5, "bf16", with_mid=True), "bf16"),
    ]
    for d in layers:  # two calls in a row, different shapes, sharing the one static scratch
        y_static = capi_gemv_static(d)
        y_ws, _ = capi_gemv(d)
        torch.cuda.synchronize()
        err = orc.rel_l2(y_static.float().cpu().numpy(), y_ws.float().cpu().numpy())
        assert err <= 1e-3, err
        assert_close_to_oracle(y_static, d.oracle(), d.dtype)


def test_static_entry_point_rejects_rank_above_limit():
    lib = _lib.cuda_lib()
    fake = ctypes.c_void_p(0x10000)  # never dereferenced: the size check comes first
    st = lib.nq_gemv_static(0, fake, 1, 64, fake, fake, MAX_RANK + 1, None, fake, 32, fake, fake, None)
    assert st == _lib.NQ_ERR_UNSUPPORTED
    assert b"rank" in lib.nq_last_error_message()
