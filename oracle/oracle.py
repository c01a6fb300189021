"""CPU oracle for the NanoQuant quantized-linear path (TEST INFRASTRUCTURE ONLY).

Only ``tests/``, ``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py``
may import this module; the product package ``nanoquant_b200`` never does.

It wraps ``nq_oracle.c`` (a plain-C restatement of the reference packers and dense
forward) through ctypes and adds the seeded input generator shared by tests and the
benchmark.  Reference behaviour restated here:

* ``pack``      -> ``src/nanoquant/kernel/utils.py:51-113``  (``pack_binary_gemv``)
* ``unpack``    -> ``src/nanoquant/kernel/utils.py:116-183`` (``unpack_binary_gemv``)
* ``forward``   -> ``src/nanoquant/modules/linear.py:282-291`` (``_compute_forward``)
  evaluated in float64 on the packed planes.
* ``dense_forward_torch`` -> the same ``_compute_forward`` as the reference's CPU path
  runs it after ``load_compressed_model`` has unpacked every factor to dense +-1
  tensors (``src/nanoquant/utils/load_utils.py:372-392``): two dense matmuls.

Pinning: ``tests/test_oracle.py`` checks every function here against golden vectors
that ``tests/golden/make_golden.py`` produced by importing the reference itself.
"""
from __future__ import annotations

import ctypes
import hashlib
import os
import subprocess
from dataclasses import dataclass
from typing import Optional

import numpy as np

ORDERS = {"lsb_first": 0, "half2": 1}
_HERE = os.path.dirname(os.path.abspath(__file__))
_SO = os.path.join(_HERE, "_build", "libnq_oracle.so")
_lib = None


def build(force: bool = False) -> str:
    """Compile nq_oracle.c with gcc into oracle/_build/libnq_oracle.so."""
    src = os.path.join(_HERE, "nq_oracle.c")
    if force or not os.path.exists(_SO) or os.path.getmtime(_SO) < os.path.getmtime(src):
        os.makedirs(os.path.dirname(_SO), exist_ok=True)
        subprocess.check_call(["gcc", "-O2", "-fPIC", "-shared", "-o", _SO, src])
    return _SO


def _load():
    global _lib
    if _lib is None:
        lib = ctypes.CDLL(build())
        lib.nqo_pack.restype = ctypes.c_long
        lib.nqo_pack.argtypes = [ctypes.c_void_p, ctypes.c_long, ctypes.c_long, ctypes.c_int, ctypes.c_void_p]
        lib.nqo_unpack.restype = ctypes.c_int
        lib.nqo_unpack.argtypes = [ctypes.c_void_p, ctypes.c_long, ctypes.c_long, ctypes.c_int, ctypes.c_void_p]
        lib.nqo_forward.restype = ctypes.c_int
        lib.nqo_forward.argtypes = [ctypes.c_void_p, ctypes.c_long, ctypes.c_long, ctypes.c_void_p,
                                    ctypes.c_void_p, ctypes.c_long, ctypes.c_void_p, ctypes.c_void_p,
                                    ctypes.c_long, ctypes.c_void_p, ctypes.c_int, ctypes.c_void_p,
                                    ctypes.c_void_p]
        _lib = lib
    return _lib


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data


def words(cols: int) -> int:
    return (cols + 31) // 32


def pack(signs: np.ndarray, method: str = "lsb_first") -> np.ndarray:
    """int8 +-1 [rows, cols] -> int32 [rows, ceil(cols/32)] (utils.py:51-113)."""
    if signs.dtype != np.int8:
        raise TypeError("Input tensor must be int8.")
    if method not in ORDERS:
        raise ValueError(f"Unsupported method: '{method}'.")
    s = np.ascontiguousarray(signs)
    rows, cols = s.shape
    out = np.empty((rows, words(cols)), dtype=np.int32)
    bad = _load().nqo_pack(_ptr(s), rows, cols, ORDERS[method], _ptr(out))
    if bad:
        raise ValueError(f"{bad} entries are not exactly +1 or -1")
    return out


def unpack(packed: np.ndarray, shape, method: str = "lsb_first") -> np.ndarray:
    """int32 planes -> int8 +-1 (utils.py:116-183); padding bits are ignored."""
    rows, cols = int(shape[0]), int(shape[1])
    if packed.ndim != 2 or packed.shape != (rows, words(cols)):
        raise ValueError(f"Unsupported packed tensor shape {packed.shape} for {shape}")
    p = np.ascontiguousarray(packed, dtype=np.int32)
    out = np.empty((rows, cols), dtype=np.int8)
    if _load().nqo_unpack(_ptr(p), rows, cols, ORDERS[method], _ptr(out)) != 0:
        raise ValueError(f"Unsupported method: '{method}'.")
    return out


# ---------------------------------------------------------------------------------------------
# Marlin layout (kernel/utils.py:186-284): the reference's prefill-GEMM packing.
# For a weight [n_out, k_red] (output rows, reduction columns), element (o, r) with
#   o = ((tile_out * 4 + o16) * 2 + o8) * 8 + o1,  r = ((tile_red * 2 + r8) * 4 + r2) * 2 + r1
# sits in word [tile_red, tile_out * 32 + o1 * 4 + r2] at bit 15 - (2 * o8 + r8) + 16 * r1 - 4 * o16
# (utils.py:191-205: the reshape / permute and the exponent table), bit set for -1.
def marlin_positions(n_out: int, k_red: int):
    """(word row, word column, bit) of every element of an [n_out, k_red] weight."""
    if n_out % 64 or k_red % 16:
        raise ValueError("the Marlin layout needs n_out % 64 == 0 and k_red % 16 == 0")
    o = np.arange(n_out)[:, None]
    r = np.arange(k_red)[None, :]
    tile_out, o16, o8, o1 = o // 64, (o % 64) // 16, (o % 16) // 8, o % 8
    tile_red, r8, r2, r1 = r // 16, (r % 16) // 8, (r % 8) // 2, r % 2
    row = np.broadcast_to(tile_red, (n_out, k_red))
    col = tile_out * 32 + o1 * 4 + r2
    bit = 15 - (2 * o8 + r8) + 16 * r1 - 4 * o16
    return row, np.broadcast_to(col, (n_out, k_red)), bit


def pack_marlin(signs: np.ndarray) -> np.ndarray:
    """int8 +-1 weight [n_out, k_red] -> int32 Marlin words [k_red / 16, n_out / 2].

    The 32 bits of word [tile_red, tile_out * 32 + o1 * 4 + r2] are the elements with
    (o16, o8, r8, r1) running over 4 x 2 x 2 x 2 (marlin_positions), so the weight is viewed as
    [tile_out, o16, o8, o1, tile_red, r8, r2, r1] and each word is a weighted sum over those axes."""
    n_out, k_red = signs.shape
    if n_out % 64 or k_red % 16:
        raise ValueError("the Marlin layout needs n_out % 64 == 0 and k_red % 16 == 0")
    neg = (np.asarray(signs) < 0).astype(np.uint64).reshape(n_out // 64, 4, 2, 8, k_red // 16, 2, 4, 2)
    o16 = np.arange(4).reshape(1, 4, 1, 1, 1, 1, 1, 1)
    o8 = np.arange(2).reshape(1, 1, 2, 1, 1, 1, 1, 1)
    r8 = np.arange(2).reshape(1, 1, 1, 1, 1, 2, 1, 1)
    r1 = np.arange(2).reshape(1, 1, 1, 1, 1, 1, 1, 2)
    weight = np.left_shift(np.uint64(1), (15 - (2 * o8 + r8) + 16 * r1 - 4 * o16).astype(np.uint64))
    w = (neg * weight).sum(axis=(1, 2, 5, 7))              # [tile_out, o1, tile_red, r2]
    w = w.transpose(2, 0, 1, 3).reshape(k_red // 16, n_out // 2)
    return w.astype(np.uint32).view(np.int32)


def unpack_marlin(words: np.ndarray, n_out: int, k_red: int) -> np.ndarray:
    """Inverse of pack_marlin: int32 words -> int8 +-1 [n_out, k_red]."""
    row, col, bit = marlin_positions(n_out, k_red)
    w = np.asarray(words).view(np.uint32).astype(np.uint64)
    b = (w[row, col] >> bit.astype(np.uint64)) & np.uint64(1)
    return (1 - 2 * b.astype(np.int8)).astype(np.int8)


def marlin_perm_in(s: np.ndarray) -> np.ndarray:
    """Input-scale order of the Marlin GEMM (utils.py:207-208)."""
    return np.asarray(s).reshape(-1, 2, 4, 2).transpose(0, 2, 1, 3).reshape(-1)


def marlin_perm_out(s: np.ndarray) -> np.ndarray:
    """Output-scale order of the Marlin GEMM (utils.py:209-210)."""
    return np.asarray(s).reshape(-1, 4, 4, 2).transpose(0, 2, 1, 3).reshape(-1)


def pack_marlin_fused(V: np.ndarray, U: np.ndarray, sg, sl, sh):
    """pack_binary_marlin_fused (utils.py:217-284) for a module's V [rank, in] and U [out, rank]
    (the reference passes V.T and U.T): rank padded to a multiple of 256 with +1 signs and zero
    scale_mid; returns (V words, U words, s1, s2, s3, workspace elements)."""
    r = V.shape[0]
    rp = (r + 255) // 256 * 256
    Vp = np.concatenate([V, np.ones((rp - r, V.shape[1]), dtype=np.int8)], 0)
    Up = np.concatenate([U, np.ones((U.shape[0], rp - r), dtype=np.int8)], 1)
    slp = np.concatenate([np.asarray(sl, dtype=np.float32), np.zeros(rp - r, dtype=np.float32)])
    ws = max(rp // 128 * 32, U.shape[0] // 128 * 32)
    return (pack_marlin(Vp), pack_marlin(Up), marlin_perm_in(sg), marlin_perm_out(slp), marlin_perm_out(sh), ws)


def forward(x, s2, v_bits, rank, smid, u_bits, s1, method: str = "lsb_first", return_interm=False):
    """float64 y = s1 * (U (smid * (V (s2 * x)))) from packed planes (linear.py:282-291).

    x: float32 [batch, in]; s2: [in]; v_bits: int32 [rank, ceil(in/32)];
    smid: [rank] or None; u_bits: int32 [out, ceil(rank/32)]; s1: [out].
    """
    x = np.ascontiguousarray(np.atleast_2d(x), dtype=np.float32)
    batch, in_f = x.shape
    out_f = int(np.asarray(s1).size)
    s2 = np.ascontiguousarray(s2, dtype=np.float32).reshape(-1)
    s1 = np.ascontiguousarray(s1, dtype=np.float32).reshape(-1)
    sm = None if smid is None else np.ascontiguousarray(smid, dtype=np.float32).reshape(-1)
    vb = np.ascontiguousarray(v_bits, dtype=np.int32)
    ub = np.ascontiguousarray(u_bits, dtype=np.int32)
    assert vb.shape == (rank, words(in_f)) and ub.shape == (out_f, words(rank))
    y = np.empty((batch, out_f), dtype=np.float64)
    t = np.empty((batch, rank), dtype=np.float64) if return_interm else None
    rc = _load().nqo_forward(_ptr(x), batch, in_f, _ptr(s2), _ptr(vb), rank, _ptr(sm), _ptr(ub),
                             out_f, _ptr(s1), ORDERS[method], _ptr(y), _ptr(t))
    if rc != 0:
        raise ValueError(method)
    return (y, t) if return_interm else y


def forward_dense(x, s2, V, smid, U, s1, round_t: Optional[str] = None):
    """float64 BLAS form of the same math on dense +-1 factors V [rank, in], U [out, rank]
    (linear.py:282-291), for large batches.  ``round_t`` rounds the intermediate
    t = smid * (V (s2 * x)) to "bf16"/"f16" first, emulating a kernel that stores it at
    that precision (the reference's own fp16/bf16 intermediate, gemm.cpp:119)."""
    x = np.atleast_2d(np.asarray(x, dtype=np.float64))
    t = (x * np.asarray(s2, dtype=np.float64).reshape(1, -1)) @ np.asarray(V, dtype=np.float64).T
    if smid is not None:
        t = t * np.asarray(smid, dtype=np.float64).reshape(1, -1)
    if round_t is not None:
        t = round_to(t.astype(np.float32), round_t).astype(np.float64)
    y = t @ np.asarray(U, dtype=np.float64).T
    return y * np.asarray(s1, dtype=np.float64).reshape(1, -1)


def dense_forward_torch(x, s2, V, smid, U, s1):
    """The reference CPU path: _compute_forward on dense +-1 factors (linear.py:282-291)."""
    import torch.nn.functional as F
    y = F.linear(x * s2, V)
    if smid is not None:
        y = y * smid
    y = F.linear(y, U)
    return y * s1


# --------------------------------------------------------------------------------------
# Seeded synthetic inputs (same stream on every machine: splitmix64, no library RNG)
# --------------------------------------------------------------------------------------
_GOLD = np.uint64(0x9E3779B97F4A7C15)


def splitmix64(seed: int, n: int, stream: int = 0) -> np.ndarray:
    """n uint64 values of the splitmix64 sequence for (seed, stream)."""
    with np.errstate(over="ignore"):
        base = np.uint64((seed * 0x100000001B3 + stream * 0xC2B2AE3D27D4EB4F) & 0xFFFFFFFFFFFFFFFF)
        z = base + (np.arange(1, n + 1, dtype=np.uint64) * _GOLD)
        z = (z ^ (z >> np.uint64(30))) * np.uint64(0xBF58476D1CE4E5B9)
        z = (z ^ (z >> np.uint64(27))) * np.uint64(0x94D049BB133111EB)
        return z ^ (z >> np.uint64(31))


def random_signs(seed: int, rows: int, cols: int, stream: int = 0) -> np.ndarray:
    u = splitmix64(seed, rows * cols, stream)
    return (1 - 2 * (u >> np.uint64(63)).astype(np.int8)).reshape(rows, cols).astype(np.int8)


def random_normal(seed: int, n: int, stream: int = 0) -> np.ndarray:
    """float64 N(0,1) via Box-Muller on two splitmix64 streams."""
    u1 = ((splitmix64(seed, n, 2 * stream + 101) >> np.uint64(11)).astype(np.float64) + 1.0) * 2.0 ** -53
    u2 = (splitmix64(seed, n, 2 * stream + 102) >> np.uint64(11)).astype(np.float64) * 2.0 ** -53
    return np.sqrt(-2.0 * np.log(u1)) * np.cos(2.0 * np.pi * u2)


def f32_to_bf16_bits(a: np.ndarray) -> np.ndarray:
    """Round-to-nearest-even float32 -> bfloat16 bit patterns (uint16)."""
    b = np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)
    rounding = ((b >> np.uint32(16)) & np.uint32(1)) + np.uint32(0x7FFF)
    with np.errstate(over="ignore"):
        out = ((b + rounding) >> np.uint32(16)).astype(np.uint16)
    nan = np.isnan(np.asarray(a, dtype=np.float32))
    out[nan] = 0x7FC0
    return out


def bf16_bits_to_f32(bits: np.ndarray) -> np.ndarray:
    return (np.asarray(bits, dtype=np.uint16).astype(np.uint32) << np.uint32(16)).view(np.float32)


def round_to(a: np.ndarray, dtype: str) -> np.ndarray:
    """Round float values to fp16/bf16 and return them as float32."""
    if dtype == "f16":
        return np.asarray(a, dtype=np.float32).astype(np.float16).astype(np.float32)
    if dtype == "bf16":
        return bf16_bits_to_f32(f32_to_bf16_bits(np.asarray(a, dtype=np.float32)))
    if dtype == "f32":
        return np.asarray(a, dtype=np.float32)
    raise ValueError(dtype)


@dataclass
class Layer:
    """One seeded NanoQuant layer, values already rounded to ``dtype`` (held as float32)."""
    out_f: int
    in_f: int
    rank: int
    V: np.ndarray        # int8 [rank, in]   (module layout, linear.py:99)
    U: np.ndarray        # int8 [out, rank]  (module layout, linear.py:100)
    s2: np.ndarray       # scale_pre  [in]
    s1: np.ndarray       # scale_post [out]
    smid: Optional[np.ndarray]  # scale_mid [rank] or None
    x: np.ndarray        # [batch, in]
    dtype: str

    def packed(self, method="lsb_first"):
        return pack(self.V, method), pack(self.U, method)

    def reference(self, method="lsb_first"):
        vb, ub = self.packed(method)
        return forward(self.x, self.s2, vb, self.rank, self.smid, ub, self.s1, method)


def make_layer(seed: int, out_f: int, in_f: int, rank: int, batch: int = 1, dtype: str = "f16",
               with_mid: bool = False, s1_std: float = 0.02) -> Layer:
    """Synthetic layer with the distributions of the benchmark configs:
    signs i.i.d. +-1; s1 = |N(0, 0.02)|; s2 = |N(0, 1)|; smid = |N(0, 1)|; x = N(0, 1)."""
    V = random_signs(seed, rank, in_f, stream=1)
    U = random_signs(seed, out_f, rank, stream=2)
    s1 = round_to(np.abs(random_normal(seed, out_f, 3)) * s1_std, dtype)
    s2 = round_to(np.abs(random_normal(seed, in_f, 4)), dtype)
    smid = round_to(np.abs(random_normal(seed, rank, 5)), dtype) if with_mid else None
    x = round_to(random_normal(seed, batch * in_f, 6).reshape(batch, in_f), dtype)
    return Layer(out_f, in_f, rank, V, U, s2, s1, smid, x, dtype)


def rel_l2(a, b) -> float:
    a = np.asarray(a, dtype=np.float64)
    b = np.asarray(b, dtype=np.float64)
    return float(np.linalg.norm(a - b) / max(np.linalg.norm(b), 1e-300))


def sha256(a: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(a).tobytes()).hexdigest()
