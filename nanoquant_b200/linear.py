"""Inference form of the reference ``NanoQuantLinear`` running on the B200 kernels.

Mirrors ``src/nanoquant/modules/linear.py``: attribute names (``V`` [rank, in], ``U``
[out, rank], ``scale_pre`` (1, in), ``scale_post`` (1, out), optional ``scale_mid``
(1, rank), ``bias``), ``init_for_inference`` (:116-129), ``_prepare_kernel`` (:186-238),
the kernel branch of ``forward`` (:141-175), ``_compute_forward`` (:282-291) and the packed
checkpoint format of ``state_dict`` / ``_load_from_state_dict`` (:359-433: ``<name>_packed``
int32 [rows, ceil(cols/32)] in lsb_first order plus ``<name>_shape`` int64 [2]).

Differences, all deliberate:
* a packed checkpoint is kept packed: ``V_packed`` / ``U_packed`` buffers are repacked to
  the kernel's bit order on the GPU, never expanded to dense +-1 tensors;
* ``forward`` always runs the CUDA kernels (an unprepared module prepares itself with
  ``kernel_type="b200"`` on first use); there is no dense or CPU fallback;
* ``bias`` is added on the kernel path too (the reference's kernel branch drops it,
  linear.py:155-166, while its dense branch adds it, linear.py:182-183).
"""
from __future__ import annotations

from typing import Optional

import torch
import torch.nn as nn

from . import _lib
from .kernel_utils import get_kernel_function, pack_binary_gemv, repack_binary, unpack_binary_gemv

KERNEL_TYPES = ("gemv", "gemm", "b200")

# launch knobs the reference passes to the GEMV op (linear.py:210-219); accepted and
# validated by this build's op, which picks its own launch shape
REFERENCE_GEMV_KWARGS = {
    "num_thread_stage1": 128,
    "num_thread_stage2": 128,
    "num_row_per_warp_stage1": 2,
    "num_row_per_warp_stage2": 2,
    "num_acc_stage1": 1,
    "num_acc_stage2": 1,
    "num_pipeline_stage1": 8,
    "num_pipeline_stage2": 8,
}


class NanoQuantLinear(nn.Module):
    """y = ((x * scale_pre) @ V^T * scale_mid) @ U^T * scale_post (+ bias), V/U in {+-1}."""

    def __init__(self, in_features: int, out_features: int, rank: int, bias: bool = False,
                 has_scale_mid: bool = False, packed: bool = True, device=None, dtype=torch.bfloat16):
        super().__init__()
        self.in_features = int(in_features)
        self.out_features = int(out_features)
        if bias:
            self.bias = nn.Parameter(torch.zeros(out_features, device=device, dtype=dtype), requires_grad=False)
        else:
            self.register_parameter("bias", None)
        self.init_for_inference(rank, has_scale_mid=has_scale_mid, packed=packed, device=device)

    # ------------------------------------------------------------------ construction
    def init_for_inference(self, rank: int, has_scale_mid: bool = False, packed: bool = False, device=None):
        """Allocate empty inference parameters (linear.py:116-129).

        ``packed=False`` allocates dense bf16 ``V``/``U`` like the reference; ``packed=True``
        allocates the lsb_first planes ``V_packed``/``U_packed`` instead.
        """
        self.rank = int(rank)
        self.do_train = False
        self._binarized = True
        self.dtype = torch.bfloat16
        self.do_kernel_inference = False
        if device is None:
            device = self.bias.device if self.bias is not None else torch.device("cpu")
        for name in ("V", "U", "V_packed", "U_packed", "V_int8", "U_int8", "scale_mid"):
            if hasattr(self, name):
                delattr(self, name)
        p = lambda *shape: nn.Parameter(torch.empty(*shape, device=device, dtype=self.dtype),  # noqa: E731
                                        requires_grad=False)
        self.scale_pre = p(1, self.in_features)
        self.scale_post = p(1, self.out_features)
        if has_scale_mid:
            self.scale_mid = p(1, self.rank)
        else:
            self.scale_mid = None
        if packed:
            self.register_buffer("V_packed", torch.zeros(self.rank, (self.in_features + 31) // 32,
                                                         device=device, dtype=torch.int32))
            self.register_buffer("U_packed", torch.zeros(self.out_features, (self.rank + 31) // 32,
                                                         device=device, dtype=torch.int32))
        else:
            self.V = p(self.rank, self.in_features)
            self.U = p(self.out_features, self.rank)

    @classmethod
    def from_linear(cls, linear: nn.Linear, rank: int, has_scale_mid: bool = False, packed: bool = True):
        """Replace an nn.Linear's geometry (and bias) the way the reference loader does
        (src/nanoquant/utils/load_utils.py:457-469)."""
        m = cls(linear.in_features, linear.out_features, rank, bias=linear.bias is not None,
                has_scale_mid=has_scale_mid, packed=packed, device=linear.weight.device)
        if linear.bias is not None:
            with torch.no_grad():
                m.bias.copy_(linear.bias.to(m.bias.dtype))
        return m

    @classmethod
    def from_factors(cls, V: torch.Tensor, U: torch.Tensor, scale_pre: torch.Tensor, scale_post: torch.Tensor,
                     scale_mid: Optional[torch.Tensor] = None, bias: Optional[torch.Tensor] = None):
        """Build from dense +-1 factors V [rank, in], U [out, rank] (CUDA tensors)."""
        rank, in_f = V.shape
        out_f = U.shape[0]
        m = cls(in_f, out_f, rank, bias=bias is not None, has_scale_mid=scale_mid is not None, packed=True,
                device=V.device)
        with torch.no_grad():
            m.V_packed.copy_(pack_binary_gemv(V.to(torch.int8), "lsb_first", check=True))
            m.U_packed.copy_(pack_binary_gemv(U.to(torch.int8), "lsb_first", check=True))
            m.scale_pre.copy_(scale_pre.reshape(1, -1).to(m.dtype))
            m.scale_post.copy_(scale_post.reshape(1, -1).to(m.dtype))
            if scale_mid is not None:
                m.scale_mid.copy_(scale_mid.reshape(1, -1).to(m.dtype))
            if bias is not None:
                m.bias.copy_(bias.to(m.bias.dtype))
        return m

    # ------------------------------------------------------------------ kernels
    def _planes_half2(self):
        """(V planes, U planes) in half2 order, built on the GPU from whatever is held."""
        if hasattr(self, "V_int8") and self.V_int8 is not None:
            return self.V_int8, self.U_int8
        if getattr(self, "V_packed", None) is not None:
            v = repack_binary(self.V_packed, self.in_features, "lsb_first", "half2")
            u = repack_binary(self.U_packed, self.rank, "lsb_first", "half2")
            return v, u
        v = pack_binary_gemv(self.V.detach().to(torch.int8), "half2", check=True)
        u = pack_binary_gemv(self.U.detach().to(torch.int8), "half2", check=True)
        return v, u

    def _prepare_kernel(self, kernel_type: str = "gemv", dtype: torch.dtype = torch.float16):
        """Convert scales to 1-D ``dtype`` and the factors to half2 planes (linear.py:186-238).

        kernel_type: "gemv" -> torch.ops.binary_kernels.nanoquant_dyn_forward (reference op);
        "gemm" -> the reference's Marlin path: marlin_nanoquant_packer on V.T / U.T (rank padded
        to 256) and torch.ops.binary_kernels.marlin_nanoquant_forward (linear.py:220-236), whose
        CUDA implementation here runs the tcgen05 GEMM (the GEMV for <= 32 rows);
        "b200" -> torch.ops.nq_b200.linear (GEMV for <= 32 rows, GEMM above).
        The reference's "gemlite" backend (third-party Triton) is not provided.
        """
        if kernel_type == "gemlite":
            raise NotImplementedError("the gemlite (Triton) backend is not part of nanoquant_b200")
        if kernel_type not in KERNEL_TYPES:
            raise ValueError("kernel_type must be one of ['gemv', 'gemm', 'b200'].")
        if dtype not in (torch.float16, torch.bfloat16):
            raise ValueError("dtype must be torch.float16 or torch.bfloat16")
        if not self.scale_pre.is_cuda:
            raise RuntimeError("move the module to a CUDA device before _prepare_kernel")
        _lib.load_torch_ops()
        v, u = self._planes_half2()
        if kernel_type == "gemm":
            self._prepare_marlin(v, u, dtype)
            return
        self.V_int8, self.U_int8 = v.contiguous(), u.contiguous()
        for name in ("V", "U", "V_packed", "U_packed"):
            if name in self._parameters or name in self._buffers:
                delattr(self, name)
        self.scale_pre = nn.Parameter(self.scale_pre.detach().to(dtype).reshape(-1), requires_grad=False)
        self.scale_post = nn.Parameter(self.scale_post.detach().to(dtype).reshape(-1), requires_grad=False)
        if self.scale_mid is not None:
            self.scale_mid = nn.Parameter(self.scale_mid.detach().to(dtype).reshape(-1), requires_grad=False)
        self.dtype = dtype
        self.kernel_type = kernel_type
        self.do_kernel_inference = True
        if kernel_type == "gemv":
            self.kernel_forward = get_kernel_function("nanoquant", dtype, kernel_type="dynamic")
            self.kernel_kwargs = dict(REFERENCE_GEMV_KWARGS)
        else:
            self.kernel_forward = torch.ops.nq_b200.linear
            self.kernel_kwargs = {}

    def _prepare_marlin(self, v_planes: torch.Tensor, u_planes: torch.Tensor, dtype: torch.dtype):
        """The reference's gemm branch (linear.py:220-236): scales in ``dtype`` (scale_mid ones if
        absent), marlin_nanoquant_packer(V.T, U.T, ...), the op marlin_nanoquant_forward."""
        from .kernel_utils import marlin_nanoquant_packer
        V = unpack_binary_gemv(v_planes, (self.rank, self.in_features), "half2")
        U = unpack_binary_gemv(u_planes, (self.out_features, self.rank), "half2")
        s_pre = self.scale_pre.detach().to(dtype).reshape(-1)
        s_post = self.scale_post.detach().to(dtype).reshape(-1)
        s_mid = (self.scale_mid.detach().to(dtype).reshape(-1) if self.scale_mid is not None
                 else torch.ones(self.rank, device=s_pre.device, dtype=dtype))
        (self.V_int8, self.U_int8, self.s1, self.s2, self.s3,
         self.workspace) = marlin_nanoquant_packer(V.T, U.T, s_pre, s_mid, s_post)
        for name in ("V", "U", "V_packed", "U_packed", "scale_pre", "scale_mid", "scale_post"):
            if name in self._parameters or name in self._buffers or hasattr(self, name):
                delattr(self, name)
        self.scale_mid = None
        self.dtype = dtype
        self.kernel_type = "gemm"
        self.do_kernel_inference = True
        self.kernel_forward = getattr(torch.ops.binary_kernels, "marlin_nanoquant_forward")
        self.kernel_kwargs = {}

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        if not getattr(self, "do_kernel_inference", False):
            self._prepare_kernel("b200", x.dtype if x.dtype in (torch.float16, torch.bfloat16) else torch.bfloat16)
        orig_dtype = x.dtype
        if x.dtype != self.dtype:
            x = x.to(self.dtype)
        original_shape = None
        if x.ndim == 3:
            original_shape = x.shape
            x = x.contiguous().view(-1, x.size(-1))
        elif x.ndim == 2:
            x = x.contiguous()
        else:
            raise ValueError(f"Expected 2D or 3D input tensor, got {x.ndim}D")
        if self.kernel_type == "gemm":
            y = self.kernel_forward(x, self.V_int8, self.U_int8, self.s1, self.s2, self.s3, self.workspace)
        else:
            y = self.kernel_forward(x, self.scale_pre, self.V_int8, self.scale_mid, self.U_int8, self.scale_post,
                                    **self.kernel_kwargs)
        if self.bias is not None:
            y = y + self.bias.to(y.dtype)
        if original_shape is not None:
            y = y.view(original_shape[0], original_shape[1], -1)
        return y.to(orig_dtype) if y.dtype != orig_dtype else y

    # ------------------------------------------------------------------ dense reference math
    def _compute_forward(self, x, V, U, scale_pre, scale_mid, scale_post):
        """The reference dense math (linear.py:282-291), kept for API parity; not used by forward()."""
        y = torch.nn.functional.linear(x * scale_pre, V)
        if scale_mid is not None:
            y = y * scale_mid
        y = torch.nn.functional.linear(y, U)
        return y * scale_post

    # ------------------------------------------------------------------ checkpoint format
    def _lsb_planes(self):
        if getattr(self, "V_packed", None) is not None:
            return self.V_packed, self.U_packed
        if hasattr(self, "V_int8"):
            return (repack_binary(self.V_int8, self.in_features, "half2", "lsb_first"),
                    repack_binary(self.U_int8, self.rank, "half2", "lsb_first"))
        return (pack_binary_gemv(self.V.detach().to(torch.int8), "lsb_first", check=True),
                pack_binary_gemv(self.U.detach().to(torch.int8), "lsb_first", check=True))

    def state_dict(self, *args, destination=None, prefix="", keep_vars=False):
        """Packed checkpoint entries (linear.py:359-394): <prefix>{V,U}_packed / _shape, scales, bias."""
        out = destination if destination is not None else {}
        vp, up = self._lsb_planes()
        out[prefix + "V_packed"] = vp.detach().cpu()
        out[prefix + "V_shape"] = torch.tensor([self.rank, self.in_features], dtype=torch.long)
        out[prefix + "U_packed"] = up.detach().cpu()
        out[prefix + "U_shape"] = torch.tensor([self.out_features, self.rank], dtype=torch.long)
        out[prefix + "scale_pre"] = self.scale_pre.detach().reshape(1, -1).cpu()
        out[prefix + "scale_post"] = self.scale_post.detach().reshape(1, -1).cpu()
        if self.scale_mid is not None:
            out[prefix + "scale_mid"] = self.scale_mid.detach().reshape(1, -1).cpu()
        if self.bias is not None:
            out[prefix + "bias"] = self.bias.detach().cpu()
        return out

    def _load_from_state_dict(self, state_dict, prefix, local_metadata, strict, missing_keys, unexpected_keys,
                              error_msgs):
        """Accept the packed format (linear.py:396-433) without expanding it to dense factors."""
        dev = self.scale_pre.device
        for name, rows, cols in (("V", self.rank, self.in_features), ("U", self.out_features, self.rank)):
            pk, sk = prefix + f"{name}_packed", prefix + f"{name}_shape"
            if pk in state_dict:
                if sk not in state_dict:
                    error_msgs.append(f"Packed factor {pk} is missing its shape key {sk}")
                    continue
                shape = tuple(int(v) for v in state_dict[sk].tolist())
                packed = state_dict[pk]
                if shape != (rows, cols) or packed.dtype != torch.int32 or tuple(packed.shape) != (rows, (cols + 31) // 32):
                    error_msgs.append(f"Invalid packed factor {pk}: shape {tuple(packed.shape)} for {shape}")
                    continue
                for stale in (name, f"{name}_int8"):
                    if stale in self._parameters or stale in self._buffers or hasattr(self, stale):
                        delattr(self, stale)
                self.register_buffer(f"{name}_packed", packed.to(device=dev, dtype=torch.int32).contiguous())
            elif strict and getattr(self, f"{name}_packed", None) is not None:
                missing_keys.append(pk)
        self.do_kernel_inference = False
        has_mid = (prefix + "scale_mid") in state_dict
        for name in ("scale_pre", "scale_post", "scale_mid"):
            key = prefix + name
            if key in state_dict:
                val = state_dict[key].to(device=dev, dtype=torch.bfloat16).reshape(1, -1)
                setattr(self, name, nn.Parameter(val, requires_grad=False))
            elif name != "scale_mid" and strict:
                missing_keys.append(key)
        if not has_mid:
            self.scale_mid = None
        if self.bias is not None:
            key = prefix + "bias"
            if key in state_dict:
                with torch.no_grad():
                    self.bias.copy_(state_dict[key].to(self.bias.dtype))
            elif strict:
                missing_keys.append(key)
        known = {prefix + k for k in ("V_packed", "V_shape", "U_packed", "U_shape", "scale_pre", "scale_post",
                                      "scale_mid", "bias")}
        if strict:
            for k in state_dict:
                if k.startswith(prefix) and k not in known and "." not in k[len(prefix):]:
                    unexpected_keys.append(k)

    def extra_repr(self):
        return f"in_features={self.in_features}, out_features={self.out_features}, rank={self.rank}"


def unpack_checkpoint_factor(packed: torch.Tensor, shape, dtype=torch.bfloat16) -> torch.Tensor:
    """Dense +-1 factor from a packed checkpoint entry (load_utils.py:392), on the GPU."""
    return unpack_binary_gemv(packed, tuple(shape), "lsb_first").to(dtype)
