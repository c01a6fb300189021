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


def static_status() -> int:
    lib = _lib.cuda_lib()
    out = ctypes.c_int(-1)
    _lib.check(lib.nq_gemv_static_status(stream_ptr(), ctypes.byref(out)))
    return out.value


def device_free_bytes() -> int:
    free, _total = torch.cuda.mem_get_info()
    return free


def test_static_entry_point_at_rank_limit_and_beyond_eight_rows():
    # rank == NQ_GEMV_STATIC_MAX_RANK fills the scratch exactly; batch 9 runs two launches that
    # share the one control block (cleared once per call, monotonic barrier counter after that)
    for d in (DeviceLayer(orc.make_layer(33, 1024, 2048, MAX_RANK, 1, "bf16"), "bf16"),
              DeviceLayer(orc.make_layer(34, 2048, 1024, 700, 9, "f16", with_mid=True), "f16")):
        y = capi_gemv_static(d)
        torch.cuda.synchronize()
        assert static_status() == _lib.NQ_OK
        assert_close_to_oracle(y, d.oracle(), d.dtype)


def test_static_entry_point_allocates_nothing():
    d = DeviceLayer(orc.make_layer(35, 4096, 4096, 1126, 1, "f16"), "f16")
    y = torch.empty(1, 4096, dtype=torch.float16, device="cuda")
    lib = _lib.cuda_lib()
    args = (NQ_DT["f16"], ptr(d.x), 1, 4096, ptr(d.s2), ptr(d.vb), 1126, None, ptr(d.ub), 4096, ptr(d.s1), ptr(y),
            stream_ptr())
    _lib.check(lib.nq_gemv_static(*args))  # the first call on the device looks up the scratch address
    torch.cuda.synchronize()
    stats0 = torch.cuda.memory_stats()
    free0 = device_free_bytes()
    for _ in range(3):
        _lib.check(lib.nq_gemv_static(*args))
    torch.cuda.synchronize()
    assert device_free_bytes() == free0, "device memory changed across nq_gemv_static calls"
    stats1 = torch.cuda.memory_stats()
    assert stats1.get("allocation.all.allocated", 0) == stats0.get("allocation.all.allocated", 0)
    assert static_status() == _lib.NQ_OK
    assert_close_to_oracle(y, d.oracle(), "f16")


def test_static_entry_point_rejects_rank_above_limit():
    lib = _lib.cuda_lib()
    fake = ctypes.c_void_p(0x10000)  # never dereferenced: the size check comes first
    st = lib.nq_gemv_static(0, fake, 1, 64, fake, fake, MAX_RANK + 1, None, fake, 32, fake, fake, None)
    assert st == _lib.NQ_ERR_UNSUPPORTED
    assert b"rank" in lib.nq_last_error_message()
