"""Loading of the in-tree native libraries.

``cuda_lib()`` opens ``_build/libnq_b200.so`` (the C ABI of include/nq_b200.h) with ctypes;
``load_torch_ops()`` registers the ``binary_kernels`` / ``nq_b200`` dispatcher ops from
``_build/libnq_torch.so``.  Both raise ImportError when the library has not been built:
there is no fallback implementation.
"""
from __future__ import annotations

import ctypes
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
BUILD_DIR = os.path.join(HERE, "_build")
CUDA_LIB_PATH = os.path.join(BUILD_DIR, "libnq_b200.so")
TORCH_LIB_PATH = os.path.join(BUILD_DIR, "libnq_torch.so")

NQ_OK = 0
NQ_ERR_INVALID_ARGUMENT = 1
NQ_ERR_UNSUPPORTED = 2
NQ_ERR_WORKSPACE = 3
NQ_ERR_CUDA = 4
NQ_ERR_DEVICE_TIMEOUT = 5
NQ_ERR_NOT_SIGNS = 6
NQ_DTYPE_F16 = 0
NQ_DTYPE_BF16 = 1
NQ_BITS_LSB_FIRST = 0
NQ_BITS_HALF2 = 1


class GemvLayer(ctypes.Structure):
    """nq_gemv_layer of include/nq_b200.h."""
    _fields_ = [("scale_pre", ctypes.c_void_p), ("v_bits", ctypes.c_void_p), ("rank", ctypes.c_int64),
                ("scale_mid", ctypes.c_void_p), ("u_bits", ctypes.c_void_p), ("out_features", ctypes.c_int64),
                ("scale_post", ctypes.c_void_p), ("y", ctypes.c_void_p)]


class GemvInput(ctypes.Structure):
    """nq_gemv_input of include/nq_b200.h."""
    _fields_ = [("x_mode", ctypes.c_int), ("eps", ctypes.c_float), ("x", ctypes.c_void_p), ("x2", ctypes.c_void_p),
                ("norm_weight", ctypes.c_void_p), ("residual_out", ctypes.c_void_p)]


class TpExchange(ctypes.Structure):
    """nq_tp_exchange of include/nq_b200.h."""
    _fields_ = [("regions", ctypes.c_void_p * 8), ("rank", ctypes.c_int), ("world", ctypes.c_int),
                ("max_elems", ctypes.c_int64)]


_lock = threading.Lock()
_cuda = None
_torch_loaded = False

_c = ctypes
_SIGNATURES = {
    "nq_abi_version": (_c.c_int, []),
    "nq_status_string": (_c.c_char_p, [_c.c_int]),
    "nq_last_error_message": (_c.c_char_p, []),
    "nq_pack_signs": (_c.c_int, [_c.c_void_p, _c.c_int64, _c.c_int64, _c.c_int, _c.c_void_p, _c.c_void_p, _c.c_void_p]),
    "nq_unpack_signs": (_c.c_int, [_c.c_void_p, _c.c_int64, _c.c_int64, _c.c_int, _c.c_void_p, _c.c_void_p]),
    "nq_repack_signs": (_c.c_int, [_c.c_void_p, _c.c_int64, _c.c_int64, _c.c_int, _c.c_int, _c.c_void_p,
                                   _c.c_void_p]),
    "nq_gemv_workspace_bytes": (_c.c_size_t, [_c.c_int64, _c.c_int64]),
    "nq_gemv": (_c.c_int, [_c.c_int, _c.c_void_p, _c.c_int64, _c.c_int64, _c.c_void_p, _c.c_void_p, _c.c_int64,
                           _c.c_void_p, _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_void_p, _c.c_void_p,
                           _c.c_size_t, _c.c_void_p]),
    "nq_gemv_group_workspace_bytes": (_c.c_size_t, [_c.c_int, _c.c_void_p]),
    "nq_gemv_group": (_c.c_int, [_c.c_int, _c.c_void_p, _c.c_int64, _c.c_int64, _c.c_int, _c.c_void_p, _c.c_void_p,
                                 _c.c_size_t, _c.c_void_p]),
    "nq_gemv_static": (_c.c_int, [_c.c_int, _c.c_void_p, _c.c_int64, _c.c_int64, _c.c_void_p, _c.c_void_p,
                                  _c.c_int64, _c.c_void_p, _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_void_p,
                                  _c.c_void_p]),
    "nq_gemv_static_status": (_c.c_int, [_c.c_void_p, _c.POINTER(_c.c_int)]),
    "nq_tp_region_bytes": (_c.c_size_t, [_c.c_int, _c.c_int64]),
    "nq_tp_region_alloc": (_c.c_int, [_c.c_int, _c.c_int64, _c.POINTER(_c.c_void_p)]),
    "nq_gemv_group_tp": (_c.c_int, [_c.c_int, _c.c_void_p, _c.c_int64, _c.c_int64, _c.c_int, _c.c_void_p, _c.c_int,
                                    _c.c_void_p, _c.c_int, _c.c_void_p, _c.c_size_t, _c.c_void_p]),
    "nq_tp_pull": (_c.c_int, [_c.c_int, _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_void_p]),
    "nq_gemv_group_ex": (_c.c_int, [_c.c_int, _c.c_void_p, _c.c_int64, _c.c_int64, _c.c_int, _c.c_void_p, _c.c_int,
                                    _c.c_void_p, _c.c_size_t, _c.c_void_p]),
    "nq_gemm_workspace_bytes": (_c.c_size_t, [_c.c_int64, _c.c_int64]),
    "nq_gemm_onebit_workspace_bytes": (_c.c_size_t, []),
    "nq_gemm_onebit": (_c.c_int, [_c.c_int, _c.c_void_p, _c.c_int64, _c.c_int64, _c.c_void_p, _c.c_void_p,
                                  _c.c_int64, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_size_t, _c.c_void_p]),
    "nq_pack_marlin": (_c.c_int, [_c.c_void_p, _c.c_int64, _c.c_int64, _c.c_void_p, _c.c_void_p, _c.c_void_p]),
    "nq_unpack_marlin": (_c.c_int, [_c.c_void_p, _c.c_int64, _c.c_int64, _c.c_void_p, _c.c_void_p]),
    "nq_marlin_to_half2": (_c.c_int, [_c.c_void_p, _c.c_int64, _c.c_int64, _c.c_void_p, _c.c_void_p]),
    "nq_gemm": (_c.c_int, [_c.c_int, _c.c_void_p, _c.c_int64, _c.c_int64, _c.c_void_p, _c.c_void_p, _c.c_int64,
                           _c.c_void_p, _c.c_void_p, _c.c_int64, _c.c_void_p, _c.c_int, _c.c_void_p, _c.c_void_p,
                           _c.c_size_t, _c.c_void_p]),
    "nq_workspace_reset": (_c.c_int, [_c.c_void_p, _c.c_size_t, _c.c_void_p]),
    "nq_workspace_status": (_c.c_int, [_c.c_void_p, _c.c_size_t, _c.c_void_p, _c.POINTER(_c.c_int)]),
    # include/nq_decoder.h
    "nq_rmsnorm": (_c.c_int, [_c.c_int, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_void_p,
                              _c.c_int64, _c.c_int64, _c.c_float, _c.c_void_p]),
    "nq_rope_cache": (_c.c_int, [_c.c_int, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_void_p,
                                 _c.c_void_p, _c.c_void_p, _c.c_int64, _c.c_int64, _c.c_int64, _c.c_int64,
                                 _c.c_int64, _c.c_float, _c.c_void_p]),
    "nq_decode_attention_workspace_bytes": (_c.c_size_t, [_c.c_int64, _c.c_int64, _c.c_int64, _c.c_int64]),
    "nq_decode_attention": (_c.c_int, [_c.c_int, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_void_p,
                                       _c.c_int64, _c.c_int64, _c.c_int64, _c.c_int64, _c.c_int64, _c.c_void_p,
                                       _c.c_size_t, _c.c_void_p]),
    "nq_decode_attention_rope": (_c.c_int, [_c.c_int, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_void_p,
                                            _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_int64, _c.c_int64,
                                            _c.c_int64, _c.c_int64, _c.c_int64, _c.c_float, _c.c_void_p,
                                            _c.c_size_t, _c.c_void_p]),
    "nq_silu_mul": (_c.c_int, [_c.c_int, _c.c_void_p, _c.c_void_p, _c.c_void_p, _c.c_int64, _c.c_void_p]),
    "nq_allreduce_region_bytes": (_c.c_size_t, [_c.c_int, _c.c_int64]),
    "nq_allreduce_region_alloc": (_c.c_int, [_c.c_int, _c.c_int64, _c.POINTER(_c.c_void_p)]),
    "nq_allreduce_region_free": (_c.c_int, [_c.c_void_p]),
    "nq_ipc_handle": (_c.c_int, [_c.c_void_p, _c.c_void_p]),
    "nq_ipc_open": (_c.c_int, [_c.c_void_p, _c.POINTER(_c.c_void_p)]),
    "nq_ipc_close": (_c.c_int, [_c.c_void_p]),
    "nq_allreduce": (_c.c_int, [_c.c_int, _c.c_void_p, _c.c_void_p, _c.c_int64, _c.c_int, _c.c_int, _c.c_void_p,
                                _c.c_int64, _c.c_void_p]),
}


class NQError(RuntimeError):
    """A non-OK status returned by the C ABI."""

    def __init__(self, status: int, message: str):
        super().__init__(f"nq_b200: {message} (status {status})")
        self.status = status


def cuda_lib() -> ctypes.CDLL:
    """ctypes handle on libnq_b200.so with argument types set for every entry point."""
    global _cuda
    with _lock:
        if _cuda is None:
            if not os.path.exists(CUDA_LIB_PATH):
                raise ImportError(f"{CUDA_LIB_PATH} is missing; build it with `python nanoquant_b200/build.py`")
            lib = ctypes.CDLL(CUDA_LIB_PATH)
            for name, (res, args) in _SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _cuda = lib
    return _cuda


def check(status: int):
    """Raise NQError for a non-OK C ABI status."""
    if status != NQ_OK:
        lib = cuda_lib()
        msg = lib.nq_last_error_message().decode(errors="replace") or lib.nq_status_string(status).decode()
        raise NQError(status, msg)


def load_torch_ops() -> None:
    """Register the dispatcher ops (idempotent)."""
    global _torch_loaded
    with _lock:
        if _torch_loaded:
            return
        if not os.path.exists(TORCH_LIB_PATH):
            raise ImportError(f"{TORCH_LIB_PATH} is missing; build it with `python nanoquant_b200/build.py`")
        import torch
        torch.ops.load_library(TORCH_LIB_PATH)
        _torch_loaded = True
