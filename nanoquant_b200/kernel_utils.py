"""GPU counterparts of the reference packing / dispatch helpers.

Mirrors the names, argument meaning and error behaviour of
``src/nanoquant/kernel/utils.py`` for the in-scope functions:

* ``pack_binary_gemv``   (utils.py:51-113)  -> nq_pack_signs CUDA kernel
* ``unpack_binary_gemv`` (utils.py:116-183) -> nq_unpack_signs CUDA kernel
* ``get_kernel_function`` (utils.py:33-48)  -> resolves ``torch.ops.binary_kernels.*``
* ``pack_binary_marlin`` (utils.py:186-214), ``pack_binary_marlin_fused`` (utils.py:217-284)
  -> nq_pack_marlin CUDA kernel + the reference's scale permutations
* ``binary_packer`` / ``binary_unpacker`` / ``marlin_onebit_packer`` / ``marlin_nanoquant_packer``
  aliases (utils.py:503-507)

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


MARLIN_MIN_MAX_PAR = 32  # the reference's lower bound for parallel column slices (kernel/utils.py:21)


def _perm_in(s: torch.Tensor) -> torch.Tensor:
    return s.reshape(s.numel() // 16, 2, 4, 2).permute(0, 2, 1, 3).reshape(-1).contiguous()


def _perm_out(s: torch.Tensor) -> torch.Tensor:
    return s.reshape(s.numel() // 32, 4, 4, 2).permute(0, 2, 1, 3).reshape(-1).contiguous()


def pack_binary_marlin(weight: torch.Tensor, scale_in: torch.Tensor, scale_out: torch.Tensor):
    """Marlin packing of a {-1,+1} weight [n_out, k_red] (kernel/utils.py:186-214), on the GPU.

    Returns (words int32 [k_red/16, n_out/2], scale_in permuted, scale_out permuted,
    workspace size) exactly as the reference; the sign words come from the nq_pack_marlin
    CUDA kernel, the scale permutations are the reference's reshape / permute."""
    _require_cuda(weight, "pack_binary_marlin")
    n_out, k_red = weight.shape
    if n_out % 64 or k_red % 16:
        raise RuntimeError(f"shape {tuple(weight.shape)} is invalid for the Marlin layout "
                           "(needs rows % 64 == 0 and columns % 16 == 0)")
    words = _ops().pack_marlin(weight.to(torch.int8).contiguous(), False)
    workspace_size = scale_out.numel() // 128 * MARLIN_MIN_MAX_PAR
    return words, _perm_in(scale_in), _perm_out(scale_out), workspace_size


def pack_binary_marlin_fused(V_sign: torch.Tensor, U_sign: torch.Tensor, scale_g: torch.Tensor,
                             scale_l: torch.Tensor, scale_h: torch.Tensor):
    """Both factors of a layer for the Marlin GEMM (kernel/utils.py:217-284), on the GPU.

    V_sign [N, R] and U_sign [R, M] are the module's V.T and U.T; the rank is padded to a
    multiple of 256 with +1 signs (V columns, U rows) and zero scale_l, as the reference does
    (which, like it, needs R % 32 == 0: utils.py:251-262 rounds only a local copy of R).
    Returns (V_bits, U_bits, scale_g_marlin, scale_l_marlin, scale_h_marlin, workspace)."""
    dev = V_sign.device
    N = scale_g.shape[0]
    R = scale_l.shape[0] if scale_l is not None else U_sign.shape[0]
    M = scale_h.shape[0]
    p = 32
    if N % p != 0:
        N = ((N // p) + 1) * p
    if R % p != 0:
        R = ((R // p) + 1) * p
    if M % p != 0:
        M = ((M // p) + 1) * p
    rank_marlin = (R + 255) // 256 * 256
    if rank_marlin > R:
        pad = rank_marlin - R
        V_sign = torch.cat([V_sign, torch.ones(N, pad, device=dev, dtype=torch.int8)], dim=1)
        U_sign = torch.cat([U_sign, torch.ones(pad, M, device=dev, dtype=torch.int8)], dim=0)
        if scale_l is not None:
            scale_l = torch.cat([scale_l, torch.zeros(pad, device=dev, dtype=scale_l.dtype)], dim=0)
    V_bits, scale_g_m, scale_l_m, ws_v = pack_binary_marlin(V_sign.T, scale_g, scale_l)
    U_bits, _, scale_h_m, ws_u = pack_binary_marlin(U_sign.T, scale_l, scale_h)
    workspace = torch.zeros(max(ws_v, ws_u), device=dev, dtype=torch.int32)
    return V_bits.contiguous(), U_bits.contiguous(), scale_g_m, scale_l_m, scale_h_m, workspace


def unpack_binary_marlin(words: torch.Tensor, n_out: int, k_red: int) -> torch.Tensor:
    """Inverse of the Marlin sign packing: int32 words -> int8 +-1 [n_out, k_red] (GPU)."""
    _require_cuda(words, "unpack_binary_marlin")
    return _ops().unpack_marlin(words.contiguous(), int(n_out), int(k_red))


binary_packer = pack_binary_gemv
binary_unpacker = unpack_binary_gemv
marlin_onebit_packer = pack_binary_marlin
marlin_nanoquant_packer = pack_binary_marlin_fused


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
