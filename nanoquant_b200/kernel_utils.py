"""GPU counterparts of the reference packing / dispatch helpers.

Mirrors the names, argument meaning and error behaviour of
``src/nanoquant/kernel/utils.py`` for the in-scope functions:

* ``pack_binary_gemv``   (utils.py:51-113)  -> nq_pack_signs CUDA kernel
* ``unpack_binary_gemv`` (utils.py:116-183) -> nq_unpack_signs CUDA kernel
* ``get_kernel_function`` (utils.py:33-48)  -> resolves ``torch.ops.binary_kernels.*``
* ``binary_packer`` / ``binary_unpacker`` aliases (utils.py:503-507)

The kernels need CUDA tensors; a CPU tensor raises instead of being packed on the host.
"""
from __future__ import annotations

from typing import Tuple

import torch

from . import _lib

METHODS = ("lsb_first", "half2")


def _ops():
    _lib.load_torch_ops()
    return torch.ops.nq_b200


def _require_cuda(t: torch.Tensor, what: str):
    if not t.is_cuda:
        raise RuntimeError(f"{what}: nanoquant_b200 runs on CUDA devices only (got a {t.device} tensor)")


def pack_binary_gemv(tensor: torch.Tensor, method: str = "lsb_first", check: bool = False) -> torch.Tensor:
    """Pack a {-1,+1} int8 matrix [rows, cols] into int32 words [rows, ceil(cols/32)].

    +1 -> bit 0, -1 -> bit 1, columns padded with +1; ``method`` selects the bit order
    ('lsb_first': column j -> bit j; 'half2': column j -> bit 15 - j//2 + 16*(j%2)).
    Raises TypeError for a non-int8 input and ValueError for an unknown method, like the
    reference.  With ``check=True`` values other than +-1 raise ValueError (the
    reference packs them into carried garbage).
    """
    if tensor.dtype != torch.int8:
        raise TypeError("Input tensor must be int8.")
    if method not in METHODS:
        raise ValueError(f"Unsupported method: '{method}'. Supported methods are 'lsb_first', 'half2'.")
    _require_cuda(tensor, "pack_binary_gemv")
    return _ops().pack_signs(tensor, method, check)


def unpack_binary_gemv(packed_tensor: torch.Tensor, original_shape: Tuple[int, int],
                       method: str = "lsb_first") -> torch.Tensor:
    """Inverse of pack_binary_gemv: int32 [rows, ceil(cols/32)] -> int8 +-1 [rows, cols]."""
    if packed_tensor.dim() != 2:
        raise ValueError(
            f"Unsupported packed tensor format. Expected 2D tensor, got {packed_tensor.dim()} dimensions.")
    n_rows, n_cols = (int(v) for v in original_shape)
    words = (n_cols + 31) // 32
    if tuple(packed_tensor.shape) != (n_rows, words):
        raise ValueError(
            f"Unsupported packed tensor shape. Expected ({n_rows}, {words}), got {packed_tensor.shape}.")
    if method not in METHODS:
        raise ValueError(f"Unsupported method: '{method}'. Supported methods are 'lsb_first', 'half2'.")
    _require_cuda(packed_tensor, "unpack_binary_gemv")
    return _ops().unpack_signs(packed_tensor.contiguous(), n_rows, n_cols, method)


def repack_binary(packed: torch.Tensor, n_cols: int, src_method: str, dst_method: str) -> torch.Tensor:
    """Convert sign planes between bit orders on the GPU (no dense round trip)."""
    _require_cuda(packed, "repack_binary")
    if src_method == dst_method:
        return packed.contiguous()
    return _ops().repack_signs(packed.contiguous(), int(n_cols), src_method, dst_method)


binary_packer = pack_binary_gemv
binary_unpacker = unpack_binary_gemv


def get_kernel_function(namespace: str, dtype: torch.dtype, kernel_type: str):
    """Resolve ``torch.ops.binary_kernels.<namespace>[_dyn]_forward`` like the reference."""
    try:
        _lib.load_torch_ops()
    except Exception as exc:  # same message shape as the reference
        raise ImportError("Could not import `binary_kernels`. Did you build the extension?\n"
                          f"Original error: {exc}") from exc
    mid = "_dyn" if kernel_type != "fixed" else ""
    op_name = f"{namespace}{mid}_forward"
    try:
        return getattr(torch.ops.binary_kernels, op_name)
    except AttributeError as exc:
        have = dir(torch.ops.binary_kernels) if hasattr(torch.ops, "binary_kernels") else []
        raise AttributeError(f"Dispatcher op `{namespace}::{op_name}` not found. "
                             f"Available in torch.ops.binary_kernels: {have}") from exc
