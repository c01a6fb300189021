"""Helpers shared by the GPU parity tests: call the C ABI directly through ctypes on
torch-allocated device buffers, and build torch tensors from oracle layers."""
import ctypes

import numpy as np
import torch

from nanoquant_b200 import _lib
from oracle import oracle as orc

TORCH_DT = {"f16": torch.float16, "bf16": torch.bfloat16}
NQ_DT = {"f16": _lib.NQ_DTYPE_F16, "bf16": _lib.NQ_DTYPE_BF16}


def stream_ptr():
    return ctypes.c_void_p(torch.cuda.current_stream().cuda_stream)


def dev(a: np.ndarray, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a))
    if dtype is not None:
        t = t.to(dtype)
    return t.cuda()


def ptr(t):
    return None if t is None else ctypes.c_void_p(t.data_ptr())


class DeviceLayer:
    """An oracle layer uploaded to the GPU in the kernel layout (half2 planes)."""

    def __init__(self, L: orc.Layer, dtype: str):
        td = TORCH_DT[dtype]
        self.L = L
        self.dtype = dtype
        self.x = dev(L.x, td)
        self.s2 = dev(L.s2, td)
        self.s1 = dev(L.s1, td)
        self.smid = None if L.smid is None else dev(L.smid, td)
        vb, ub = L.packed("half2")
        self.vb = dev(vb)
        self.ub = dev(ub)
        # inputs exactly as the GPU sees them (rounded to dtype), for the oracle
        f = lambda t: None if t is None else t.float().cpu().numpy()  # noqa: E731
        self.xr, self.s2r, self.s1r, self.smidr = f(self.x), f(self.s2), f(self.s1), f(self.smid)

    def oracle(self, x=None):
        x = self.xr if x is None else x
        return orc.forward(x, self.s2r, self.L.packed("half2")[0], self.L.rank, self.smidr,
                           self.L.packed("half2")[1], self.s1r, "half2")


def capi_gemv(d: DeviceLayer, x: torch.Tensor = None, workspace: torch.Tensor = None):
    lib = _lib.cuda_lib()
    x = d.x if x is None else x
    batch, in_f = x.shape
    out_f = d.s1.numel()
    y = torch.empty(batch, out_f, dtype=x.dtype, device=x.device)
    wsb = lib.nq_gemv_workspace_bytes(batch, d.L.rank)
    if workspace is None:
        workspace = torch.zeros(wsb, dtype=torch.uint8, device=x.device)
    st = lib.nq_gemv(NQ_DT[d.dtype], ptr(x), batch, in_f, ptr(d.s2), ptr(d.vb), d.L.rank, ptr(d.smid), ptr(d.ub),
                     out_f, ptr(d.s1), ptr(y), ptr(workspace), workspace.numel(), stream_ptr())
    _lib.check(st)
    return y, workspace


def workspace_status(ws: torch.Tensor) -> int:
    lib = _lib.cuda_lib()
    out = ctypes.c_int(-1)
    _lib.check(lib.nq_workspace_status(ptr(ws), ws.numel(), stream_ptr(), ctypes.byref(out)))
    return out.value


def assert_close_to_oracle(y: torch.Tensor, ref: np.ndarray, dtype: str, tol: float = 1e-3):
    """rel-L2 of the kernel output against the float64 oracle rounded once to the output
    dtype is <= tol (1e-3 per layer); for fp16 outputs the unrounded oracle must meet the
    same bound."""
    yk = y.float().cpu().numpy().astype(np.float64)
    r_round = orc.rel_l2(yk, orc.round_to(ref, dtype))
    assert r_round <= tol, f"rel-L2 vs dtype-rounded oracle {r_round:.3e} > {tol}"
    if dtype == "f16":
        r = orc.rel_l2(yk, ref)
        assert r <= tol, f"rel-L2 vs float64 oracle {r:.3e} > {tol}"
    return r_round
