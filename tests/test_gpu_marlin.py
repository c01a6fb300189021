"""The reference's Marlin (prefill GEMM) path on the GPU.

* packing: pack_binary_marlin / pack_binary_marlin_fused (nq_pack_marlin CUDA kernel + the
  reference's scale permutations) bit-exact against golden vectors produced by the reference's
  own packers (tests/golden/make_golden_marlin.py), including the rank padding to 256;
* nq_marlin_to_half2 equals packing the same signs in HALF2 order directly;
* torch.ops.binary_kernels.marlin_onebit_forward / marlin_nanoquant_forward (the reference
  schemas, pybind.cpp:93-104) against the float64 oracle, rel-L2 <= 1e-3 (nq_testutil);
* the reference's _prepare_kernel("gemm") sequence (modules/linear.py:220-236) replayed through
  this package's NanoQuantLinear, for GEMV-sized and GEMM-sized inputs.
For fp16 layers the GEMM rounds the intermediate once to fp16, the reference's own rounding point
(gemm.cpp:119); those outputs are also compared with the oracle given that rounding."""
import os

import numpy as np
import pytest
import torch

import nanoquant_b200 as nq
from nanoquant_b200 import kernel_utils as ku
from oracle import oracle as orc

from .nq_testutil import assert_close_to_oracle

pytestmark = pytest.mark.gpu
G = dict(np.load(os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "golden_marlin_v1.npz")))
ONEBIT = sorted({k[len("onebit_"):-len("_signs")] for k in G if k.startswith("onebit_") and k.endswith("_signs")})
FUSED = sorted({k[len("fused_"):-len("_V")] for k in G if k.startswith("fused_") and k.endswith("_V")})


def cu(a, dtype=None):
    t = torch.from_numpy(np.ascontiguousarray(a)).cuda()
    return t.to(dtype) if dtype is not None else t


@pytest.mark.parametrize("key", ONEBIT)
def test_pack_binary_marlin_matches_reference(key):
    w = G[f"onebit_{key}_signs"]
    words, si, so, ws = ku.pack_binary_marlin(cu(w), cu(G[f"onebit_{key}_sin"]), cu(G[f"onebit_{key}_sout"]))
    assert np.array_equal(words.cpu().numpy(), G[f"onebit_{key}_bits"])
    assert np.array_equal(si.cpu().numpy(), G[f"onebit_{key}_sin_perm"])
    assert np.array_equal(so.cpu().numpy(), G[f"onebit_{key}_sout_perm"])
    assert ws == int(G[f"onebit_{key}_ws"][0])
    back = ku.unpack_binary_marlin(words, *w.shape)
    assert np.array_equal(back.cpu().numpy(), w)
    # Marlin words -> HALF2 planes equals packing the signs in HALF2 order directly
    h2 = torch.ops.nq_b200.marlin_to_half2(words, w.shape[0], w.shape[1])
    assert torch.equal(h2, nq.pack_binary_gemv(cu(w), "half2"))


@pytest.mark.parametrize("key", FUSED)
def test_pack_binary_marlin_fused_matches_reference(key):
    V, U = G[f"fused_{key}_V"], G[f"fused_{key}_U"]
    vb, ub, s1, s2, s3, ws = ku.marlin_nanoquant_packer(cu(V).T, cu(U).T, cu(G[f"fused_{key}_sg"]),
                                                        cu(G[f"fused_{key}_sl"]), cu(G[f"fused_{key}_sh"]))
    assert np.array_equal(vb.cpu().numpy(), G[f"fused_{key}_vbits"])
    assert np.array_equal(ub.cpu().numpy(), G[f"fused_{key}_ubits"])
    for t, name in ((s1, "s1"), (s2, "s2"), (s3, "s3")):
        assert np.array_equal(t.cpu().numpy(), G[f"fused_{key}_{name}"])
    assert ws.numel() == int(G[f"fused_{key}_ws_numel"][0]) and ws.dtype == torch.int32


@pytest.mark.parametrize("m", [1, 7, 200])
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_marlin_onebit_forward_matches_oracle(m, dtype):
    td = torch.float16 if dtype == "f16" else torch.bfloat16
    n, k = 256, 1024
    w = orc.random_signs(51 + m, n, k)
    s_in = orc.round_to(np.abs(orc.random_normal(52, k)), dtype)
    s_out = orc.round_to(np.abs(orc.random_normal(53, n)) * 0.02, dtype)
    x = orc.round_to(orc.random_normal(54 + m, m * k).reshape(m, k), dtype)
    words, si, so, wsn = ku.marlin_onebit_packer(cu(w), cu(s_in, td), cu(s_out, td))
    ws = torch.zeros(max(wsn, 1), dtype=torch.int32, device="cuda")
    y = torch.ops.binary_kernels.marlin_onebit_forward(cu(x, td), words, si, so, ws)
    ref = ((x.astype(np.float64) * s_in[None, :]) @ w.astype(np.float64).T) * s_out[None, :]
    assert_close_to_oracle(y, ref, dtype)


@pytest.mark.parametrize("shape,m,dtype", [
    ((4096, 4096, 1088), 1, "f16"),      # 7B attention shape at the planner rank: GEMV path
    ((4096, 4096, 1088), 128, "f16"),    # GEMM path, T rounded to fp16 like the reference
    ((256, 512, 96), 300, "bf16"),       # rank padded 96 -> 256; bf16 keeps T as hi/lo
    ((192, 1024, 512), 5, "bf16"),
])
def test_prepare_kernel_gemm_replays_reference_sequence(shape, m, dtype):
    out_f, in_f, rank = shape
    td = torch.float16 if dtype == "f16" else torch.bfloat16
    L = orc.make_layer(rank + m, out_f, in_f, rank, m, dtype, with_mid=True)
    mod = nq.NanoQuantLinear(in_f, out_f, rank, has_scale_mid=True, packed=False, device="cuda")
    with torch.no_grad():
        mod.V.copy_(cu(L.V).float())
        mod.U.copy_(cu(L.U).float())
        mod.scale_pre.copy_(cu(L.s2).reshape(1, -1))
        mod.scale_post.copy_(cu(L.s1).reshape(1, -1))
        mod.scale_mid.copy_(cu(L.smid).reshape(1, -1))
    mod._prepare_kernel("gemm", td)
    assert mod.kernel_forward is torch.ops.binary_kernels.marlin_nanoquant_forward
    assert mod.V_int8.shape == (in_f // 16, ((rank + 255) // 256 * 256) // 2)
    x = cu(L.x, td)
    y = mod(x)
    # the module keeps its scales in bf16 (reference init_for_inference), then casts to dtype
    rr = lambda a: orc.round_to(orc.round_to(a, "bf16"), dtype)  # noqa: E731
    s2, s1, smid = rr(L.s2), rr(L.s1), rr(L.smid)
    xr = x.float().cpu().numpy()
    exact = orc.forward_dense(xr, s2, L.V, smid, L.U, s1)
    assert_close_to_oracle(y, exact, dtype)
    if dtype == "f16" and m > 32:  # the GEMM's fp16 intermediate: also match that rounding point
        assert_close_to_oracle(y, orc.forward_dense(xr, s2, L.V, smid, L.U, s1, round_t="f16"), dtype)


def test_marlin_ops_reject_like_the_reference():
    x = torch.zeros(4, 64, dtype=torch.float16, device="cuda")
    w = torch.zeros(3, 64, dtype=torch.int32, device="cuda")  # k = 48 != 64
    ws = torch.zeros(64, dtype=torch.int32, device="cuda")
    with pytest.raises(RuntimeError, match="k dimension mismatch"):
        torch.ops.binary_kernels.marlin_onebit_forward(x, w, None, None, ws)
    w = torch.zeros(4, 256, dtype=torch.int32, device="cuda")  # n = 512 needs 4 * 32 workspace ints
    with pytest.raises(RuntimeError, match="workspace too small"):
        torch.ops.binary_kernels.marlin_onebit_forward(x, w, None, None, ws[:10])
    with pytest.raises(RuntimeError, match="Unsupported dtype"):
        torch.ops.binary_kernels.marlin_onebit_forward(x.float(), w, None, None, ws)
