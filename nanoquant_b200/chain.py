"""GEMV chains: several grouped decode GEMVs in one cooperative launch (``nq_gemv_chain``).

A phase is a group of 1-3 NanoQuant layers that read the same input x', formed on the fly from
what earlier phases wrote: x' = x (PLAIN), RMSNorm(x) * weight (RMSNORM), silu(x) * x2
(SILU_MUL) or x * x2 (MUL); a single-layer phase may add a residual to its output, in place, and
`act` puts chosen layers' outputs through SiLU (a SwiGLU gate, then consumed with MUL).  A decoder block's
o-projection, MLP and the next block's q/k/v form one chain, so the block costs two launches
(chain + attention) instead of eight.  The reference runs each of these as its own call
(src/nanoquant/modules/linear.py:155-164 per linear, HF modules around them).
"""
from __future__ import annotations

import ctypes
from typing import List, Optional, Sequence

import torch

from . import _lib

PLAIN, RMSNORM, SILU_MUL, MUL = 0, 1, 2, 3
MAX_PHASES = 4
_DT = {torch.float16: 0, torch.bfloat16: 1}


def _ptr(t: Optional[torch.Tensor]):
    return t.data_ptr() if t is not None else None


class Phase:
    """One chain phase.  `layers`: objects with s2, vb, smid, ub, s1 (QuantLinearShard);
    `out`: optional output tensors (one per layer), allocated when omitted."""

    def __init__(self, layers: Sequence, x: torch.Tensor, mode: int = PLAIN, x2: Optional[torch.Tensor] = None,
                 norm_weight: Optional[torch.Tensor] = None, eps: float = 1e-5,
                 residual: Optional[torch.Tensor] = None, out: Optional[Sequence[torch.Tensor]] = None,
                 act: int = 0):
        self.layers, self.x, self.mode, self.x2, self.act = list(layers), x, mode, x2, act
        self.norm_weight, self.eps, self.residual = norm_weight, eps, residual
        self.out = list(out) if out is not None else None


def _struct(phases: Sequence[Phase], batch: int, alloc: bool):
    arr = (_lib.ChainPhase * len(phases))()
    outs: List[List[torch.Tensor]] = []
    for i, ph in enumerate(phases):
        c = arr[i]
        c.n_layers = len(ph.layers)
        c.x_mode = ph.mode
        c.act = ph.act
        c.in_features = ph.layers[0].s2.numel()
        c.x, c.x2, c.norm_weight = _ptr(ph.x), _ptr(ph.x2), _ptr(ph.norm_weight)
        c.eps = ph.eps
        c.residual = _ptr(ph.residual)
        ys = ph.out
        if ys is None:
            ys = [torch.empty(batch, L.s1.numel(), dtype=ph.x.dtype, device=ph.x.device) if alloc else None
                  for L in ph.layers]
        for l, L in enumerate(ph.layers):
            g = c.layers[l]
            g.scale_pre, g.v_bits, g.rank = L.s2.data_ptr(), L.vb.data_ptr(), L.vb.shape[0]
            g.scale_mid, g.u_bits = _ptr(L.smid), L.ub.data_ptr()
            g.out_features, g.scale_post = L.s1.numel(), L.s1.data_ptr()
            g.y = _ptr(ys[l]) if ys[l] is not None else 16  # planning only: any aligned address
        outs.append(ys)
    return arr, outs


def workspace_bytes(phases: Sequence[Phase], batch: int) -> int:
    """Workspace of a chain, 0 when it cannot run (too large for shared memory, batch > 2, ...)."""
    arr, _ = _struct(phases, batch, alloc=False)
    return int(_lib.cuda_lib().nq_gemv_chain_workspace_bytes(_DT[phases[0].x.dtype], batch, len(phases),
                                                             ctypes.addressof(arr)))


def why_not() -> str:
    return _lib.cuda_lib().nq_last_error_message().decode()


def run(phases: Sequence[Phase], workspace: torch.Tensor) -> List[List[torch.Tensor]]:
    """Launch the chain on the current stream; returns each phase's outputs.  `workspace`: a
    zero-initialised uint8 tensor of at least workspace_bytes(), used by one chain at a time."""
    x = phases[0].x
    if not x.is_cuda:
        raise RuntimeError("nq_gemv_chain needs CUDA tensors")
    batch = x.shape[0]
    arr, outs = _struct(phases, batch, alloc=True)
    lib = _lib.cuda_lib()
    st = lib.nq_gemv_chain(_DT[x.dtype], batch, len(phases), ctypes.addressof(arr), workspace.data_ptr(),
                           workspace.numel(), torch.cuda.current_stream(x.device).cuda_stream)
    _lib.check(st)
    return outs
