"""Fused decode GEMV parity on the GPU against the reference goldens and the float64
oracle.  Tolerance (written in nq_testutil.assert_close_to_oracle): rel-L2 <= 1e-3 per
layer against the oracle rounded to the output dtype, and for fp16 also against the
unrounded float64 oracle."""
import numpy as np
import pytest
import torch

import nanoquant_b200 as nq
from oracle import oracle as orc

from .golden_data import GOLDEN, layer_from_golden
from .nq_testutil import DeviceLayer, assert_close_to_oracle, capi_gemv, stream_ptr, workspace_status

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("name,dtype", [("ragged_b8", "f16"), ("attn_small", "bf16")])
def test_gemv_reference_golden(name, dtype):
    d = DeviceLayer(layer_from_golden(name), dtype)
    y, ws = capi_gemv(d)
    torch.cuda.synchronize()
    assert_close_to_oracle(y, GOLDEN[f"layer_{name}_y"].astype(np.float64), dtype)
    assert workspace_status(ws) == 0


def test_gemv_config0_reference_golden():
    seed, out_f, in_f, rank, batch = (int(v) for v in GOLDEN["cfg0_meta"])
    d = DeviceLayer(orc.make_layer(seed, out_f, in_f, rank, batch, "f16"), "f16")
    y, _ = capi_gemv(d)
    assert_close_to_oracle(y, GOLDEN["cfg0_y"].astype(np.float64), "f16")


SHAPES = [  # (out, in, rank): Llama-2-7B layers at the benchmark ranks and the reference-formula ranks
    (4096, 4096, 1126), (11008, 4096, 2054), (4096, 11008, 2054), (4096, 4096, 1088), (11008, 4096, 1600),
]


@pytest.mark.parametrize("shape", SHAPES)
@pytest.mark.parametrize("batch", [1, 8])
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_gemv_llama_shapes(shape, batch, dtype):
    out_f, in_f, rank = shape
    L = orc.make_layer(out_f + rank + batch, out_f, in_f, rank, batch, dtype, with_mid=(batch == 8))
    d = DeviceLayer(L, dtype)
    y, ws = capi_gemv(d)
    assert_close_to_oracle(y, d.oracle(), dtype)
    assert workspace_status(ws) == 0


@pytest.mark.parametrize("batch", [2, 3, 4, 5])
def test_gemv_batch_sizes(batch):
    L = orc.make_layer(batch, 4096, 4096, 1126, batch, "f16", with_mid=True)
    d = DeviceLayer(L, "f16")
    y, _ = capi_gemv(d)
    assert_close_to_oracle(y, d.oracle(), "f16")


@pytest.mark.parametrize("shape", [(1, 1, 1), (7, 5, 3), (100, 70, 33), (33, 130, 17), (17, 8, 40), (1000, 200, 96),
                                   (130, 96, 47)])
@pytest.mark.parametrize("dtype", ["f16", "bf16"])
def test_gemv_ragged_shapes(shape, dtype):
    out_f, in_f, rank = shape
    L = orc.make_layer(sum(shape), out_f, in_f, rank, 3, dtype, with_mid=True)
    d = DeviceLayer(L, dtype)
    y, _ = capi_gemv(d)
    assert_close_to_oracle(y, d.oracle(), dtype)


def test_gemv_batch_above_eight_runs_in_chunks():
    L = orc.make_layer(21, 1024, 512, 200, 19, "bf16", with_mid=False)
    d = DeviceLayer(L, "bf16")
    y, _ = capi_gemv(d)
    assert_close_to_oracle(y, d.oracle(), "bf16")


def test_gemv_split_mode_for_large_layer():
    """70B down-projection geometry exceeds the fused shared-memory budget and runs as
    two launches; results must be identical in quality."""
    L = orc.make_layer(70, 8192, 28672, 3488, 1, "bf16")
    d = DeviceLayer(L, "bf16")
    y, ws = capi_gemv(d)
    assert_close_to_oracle(y, d.oracle(), "bf16")
    assert workspace_status(ws) == 0


def test_gemv_deterministic_and_workspace_reusable():
    L = orc.make_layer(5, 11008, 4096, 2054, 2, "f16")
    d = DeviceLayer(L, "f16")
    y1, ws = capi_gemv(d)
    outs = [capi_gemv(d, workspace=ws)[0] for _ in range(5)]
    for y in outs:
        assert torch.equal(y, y1)
    assert workspace_status(ws) == 0


def test_gemv_fp16_clamp_matches_reference():
    """Outputs beyond the fp16 range clamp to +-64504 (reference cuda_utils.cuh:80-86)."""
    L = orc.make_layer(9, 64, 256, 32, 1, "f16", s1_std=1.0)
    L.s1[:] = 60000.0
    d = DeviceLayer(L, "f16")
    y, _ = capi_gemv(d)
    ref = d.oracle()
    yk = y.float().cpu().numpy()
    big = np.abs(ref) > 64504
    assert big.any()
    # clamp to +-64504 then round to fp16, which lands on 64512 (fp16 spacing is 32 there)
    np.testing.assert_array_equal(np.abs(yk[big]), float(np.float16(64504.0)))
    assert np.isfinite(yk).all()


def test_reference_op_and_module_drop_in():
    """torch.ops.binary_kernels.nanoquant_dyn_forward with the reference's argument order
    and knobs, and the module's gemv / b200 kernel types."""
    L = orc.make_layer(3, 4096, 4096, 1126, 4, "f16", with_mid=True)
    d = DeviceLayer(L, "f16")
    y = torch.ops.binary_kernels.nanoquant_dyn_forward(d.x, d.s2, d.vb, d.smid, d.ub, d.s1, 128, 128, 2, 2, 1, 1,
                                                       8, 8)
    ref = d.oracle()
    assert_close_to_oracle(y, ref, "f16")
    with pytest.raises(ValueError):  # the reference's own schema default num_acc=4 is outside its sweep
        torch.ops.binary_kernels.nanoquant_dyn_forward(d.x, d.s2, d.vb, d.smid, d.ub, d.s1)
    # 1-D input -> 1-D output, like the reference
    y1 = torch.ops.binary_kernels.nanoquant_dyn_forward(d.x[0], d.s2, d.vb, d.smid, d.ub, d.s1, 128, 128, 2, 2, 1,
                                                        1, 8, 8)
    assert y1.shape == (4096,)
    # the module keeps its scales in bf16 (reference init_for_inference, linear.py:106/120),
    # so its fp16 kernels see scales rounded bf16 -> fp16
    rr = lambda a: orc.round_to(orc.round_to(a, "bf16"), "f16")  # noqa: E731
    vb, ub = L.packed("half2")
    ref_mod = orc.forward(d.xr, rr(d.s2r), vb, L.rank, rr(d.smidr), ub, rr(d.s1r), "half2")
    for kt in ("gemv", "b200"):
        m2 = nq.NanoQuantLinear.from_factors(torch.from_numpy(L.V).cuda().float(),
                                             torch.from_numpy(L.U).cuda().float(), d.s2.float(), d.s1.float(),
                                             d.smid.float())
        m2._prepare_kernel(kt, torch.float16)
        y3 = m2(d.x.view(2, 2, -1))
        assert y3.shape == (2, 2, 4096)
        assert_close_to_oracle(y3.view(4, -1), ref_mod, "f16")


@pytest.mark.parametrize("batch", [1, 3])
def test_gemv_unaligned_vectors(batch):
    """x, s2 and s1 given as views at a 2-byte offset (only 2-byte alignment is required):
    the kernel must take its plain-load paths instead of the bulk copies."""
    L = orc.make_layer(77 + batch, 1000, 512, 200, batch, "f16", with_mid=True)
    d = DeviceLayer(L, "f16")

    def shifted(t):
        buf = torch.empty(t.numel() + 1, dtype=t.dtype, device=t.device)
        v = buf[1:1 + t.numel()].view(t.shape)
        v.copy_(t)
        assert v.data_ptr() % 16 != 0
        return v

    d.x, d.s2, d.s1 = shifted(d.x), shifted(d.s2), shifted(d.s1)
    y, ws = capi_gemv(d)
    assert_close_to_oracle(y, d.oracle(), "f16")
    assert workspace_status(ws) == 0


def _capi_group(ds, x):
    from nanoquant_b200 import _lib as L
    import ctypes as C
    lib = L.cuda_lib()
    batch, in_f = x.shape
    descs = (L.GemvLayer * len(ds))()
    ys = []
    for i, d in enumerate(ds):
        y = torch.empty(batch, d.s1.numel(), dtype=x.dtype, device="cuda")
        ys.append(y)
        descs[i] = L.GemvLayer(d.s2.data_ptr(), d.vb.data_ptr(), d.L.rank,
                               d.smid.data_ptr() if d.smid is not None else None, d.ub.data_ptr(), d.s1.numel(),
                               d.s1.data_ptr(), y.data_ptr())
    ranks = (C.c_int64 * len(ds))(*[d.L.rank for d in ds])
    wsb = lib.nq_gemv_group_workspace_bytes(len(ds), ranks)
    ws = torch.zeros(wsb, dtype=torch.uint8, device="cuda")
    L.check(lib.nq_gemv_group(0 if x.dtype == torch.float16 else 1, C.c_void_p(x.data_ptr()), batch, in_f, len(ds),
                              descs, C.c_void_p(ws.data_ptr()), wsb, stream_ptr()))
    return ys, ws


@pytest.mark.parametrize("shapes,batch,dtype", [
    ([(4096, 1126), (4096, 1126), (4096, 1126)], 1, "f16"),            # 7B q/k/v
    ([(11008, 2054), (11008, 2054)], 1, "f16"),                        # 7B gate/up
    ([(1024, 552), (128, 120), (128, 120)], 2, "bf16"),                # 70B-like q/k/v (GQA), scaled down
    ([(500, 200), (130, 33), (77, 96)], 5, "bf16"),                    # ragged, no folding (batch 5)
])
def test_gemv_group_matches_single_layers(shapes, batch, dtype):
    in_f = 4096 if shapes[0][0] >= 4096 else 1024
    ds = []
    x_np = None
    for i, (out_f, rank) in enumerate(shapes):
        L = orc.make_layer(100 + i, out_f, in_f, rank, batch, dtype, with_mid=(i == 1))
        if x_np is None:
            x_np = L.x
        L.x = x_np  # every member reads the same input
        ds.append(DeviceLayer(L, dtype))
    x = ds[0].x
    ys, ws = _capi_group(ds, x)
    for d, y in zip(ds, ys):
        assert_close_to_oracle(y, d.oracle(), dtype)
    assert workspace_status(ws) == 0
    # and through the torch op used by the decoder
    ys2 = torch.ops.nq_b200.gemv_group(x, [d.s2 for d in ds], [d.vb for d in ds], [d.smid for d in ds],
                                       [d.ub for d in ds], [d.s1 for d in ds])
    for y, y2 in zip(ys, ys2):
        assert torch.equal(y, y2)


def _ex_layers(shapes, dt, seed):
    from nanoquant_b200.decoder import QuantLinearShard, _random_planes
    out = []
    for i, (o, n, r) in enumerate(shapes):
        g = torch.Generator(device="cuda")
        g.manual_seed(seed + i)
        vb, ub = _random_planes(g, r, n, "cuda"), _random_planes(g, o, r, "cuda")
        s2 = (torch.rand(n, generator=g, device="cuda") + 0.5).to(dt) / n ** 0.5
        s1 = (torch.rand(o, generator=g, device="cuda") + 0.5).to(dt) / r ** 0.5
        out.append(QuantLinearShard(vb, ub, s2, None, s1))
    return out


def _lists(Ls):
    return [L.s2 for L in Ls], [L.vb for L in Ls], [L.smid for L in Ls], [L.ub for L in Ls], [L.s1 for L in Ls]


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("batch", [1, 2, 5])
def test_group_ex_input_modes_match_separate_kernels(dt, batch):
    """nq_gemv_group_ex: x' formed in the prologue.  SILU_MUL and MUL give the bits of
    silu_mul / a multiply followed by the grouped GEMV; RMSNORM matches rmsnorm followed by
    the grouped GEMV to rel-L2 1e-3 (the mean is summed in another order) and writes the same
    residual bits; act puts the chosen outputs through SiLU."""
    ops = torch.ops.nq_b200
    Ls = _ex_layers([(1000, 4096, 300), (512, 4096, 160)], dt, 7)
    lists = _lists(Ls)
    g = torch.Generator(device="cuda")
    g.manual_seed(batch)
    x = torch.randn(batch, 4096, generator=g, device="cuda").to(dt)
    x2 = torch.randn(batch, 4096, generator=g, device="cuda").to(dt)
    w = (torch.rand(4096, generator=g, device="cuda") + 0.5).to(dt)
    # SILU_MUL and MUL: bit-identical to the separate kernels
    got = ops.gemv_group_ex(x, x2, None, 0.0, 2, None, 0, *lists)
    want = ops.gemv_group(ops.silu_mul(x, x2), *lists)
    for a, b in zip(got, want):
        assert torch.equal(a, b)
    got = ops.gemv_group_ex(x, x2, None, 0.0, 3, None, 0, *lists)
    want = ops.gemv_group((x.float() * x2.float()).to(dt), *lists)
    for a, b in zip(got, want):
        assert torch.equal(a, b)
    # RMSNORM with and without the residual
    for res_in in (x2, None):
        res_out = torch.empty_like(x)
        got = ops.gemv_group_ex(x, res_in, w, 1e-5, 1, res_out, 0, *lists)
        xn, r = ops.rmsnorm(x, res_in, w, 1e-5)
        want = ops.gemv_group(xn, *lists)
        assert torch.equal(res_out, r)
        for a, b in zip(got, want):
            assert orc.rel_l2(a.float().cpu().numpy(), b.float().cpu().numpy()) <= 1e-3
    # act on the first member only
    got = ops.gemv_group_ex(x, None, None, 0.0, 0, None, 1, *lists)
    want = ops.gemv_group(x, *lists)
    gate = want[0].float()
    assert orc.rel_l2(got[0].float().cpu().numpy(), (gate / (1 + torch.exp(-gate))).cpu().numpy()) <= 2e-3
    assert torch.equal(got[1], want[1])


def test_decoder_fused_prologues_match_separate_kernels():
    """The decode step with the neighbours in the GEMV prologues/epilogue decodes the same
    tokens as the step with separate RMSNorm / SiLU kernels."""
    from nanoquant_b200.decoder import TINY, Decoder
    prompt = torch.randint(0, TINY.vocab, (29,), generator=torch.Generator().manual_seed(4)).cuda()
    runs = []
    for fused in (True, False):
        dec = Decoder(TINY, max_seq=80, seed=5, device="cuda")
        dec.fuse_neighbours = fused
        dec.prefill(prompt)
        logits = dec.step_logits().float()
        dec.tokens.fill_(int(torch.argmax(logits[0])))
        dec.pos.add_(1)
        dec.seq_len.add_(1)
        runs.append((logits.cpu(), [int(dec.step()[0]) for _ in range(8)]))
    assert orc.rel_l2(runs[0][0].numpy(), runs[1][0].numpy()) <= 1e-2
    assert runs[0][1] == runs[1][1]
