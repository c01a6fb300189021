"""Parity of the Llama-3-70B layer shapes on the GPU: every projection's
decode GEMV at batch 1 and 8, its tensor-parallel shards at TP 2/4/8 exactly as the decoder
cuts them (nanoquant_b200.decoder._make_layer), and the prefill GEMM at M = 128 and 2048.

Ranks: the reference planner at 0.55 bpw (src/nanoquant/utils/utils.py:273-289): q/o 2208,
k/v 480, gate/up/down 3488.  Tolerance as in the other kernel tests: rel-L2 <= 1e-3 per layer
against the float64 oracle (nq_testutil.assert_close_to_oracle).  At M = 2048 the GEMM's
output rows are independent, so a seeded sample of 64 rows is compared with the oracle (the
float64 oracle of the whole 28672 x 8192 layer at M = 2048 would take minutes)."""
import numpy as np
import pytest
import torch

from nanoquant_b200.decoder import LLAMA3_70B, PROJ, _make_layer
from oracle import oracle as orc

from .nq_testutil import DeviceLayer, assert_close_to_oracle, capi_gemv, workspace_status
from .test_gpu_gemm import capi_gemm

pytestmark = pytest.mark.gpu

SHAPES_70B = {p: (*LLAMA3_70B.io(p), LLAMA3_70B.ranks[p]) for p in ("q", "k", "o", "gate", "down")}


@pytest.mark.parametrize("proj", list(SHAPES_70B))
@pytest.mark.parametrize("batch,dtype", [(1, "f16"), (8, "bf16")])
def test_gemv_llama3_70b_shapes(proj, batch, dtype):
    out_f, in_f, rank = SHAPES_70B[proj]
    L = orc.make_layer(700 + PROJ.index(proj) + batch, out_f, in_f, rank, batch, dtype, with_mid=(batch == 8))
    d = DeviceLayer(L, dtype)
    y, ws = capi_gemv(d)
    assert_close_to_oracle(y, d.oracle(), dtype)
    assert workspace_status(ws) == 0


@pytest.mark.parametrize("tp", [2, 4, 8])
@pytest.mark.parametrize("proj", list(PROJ))
def test_gemv_llama3_70b_tp_shards(tp, proj):
    """The last rank's shard of every projection (column-parallel: U rows of its outputs;
    row-parallel o/down: V columns of its input slice), as the decoder builds it."""
    dt = torch.float16
    q = _make_layer(LLAMA3_70B, proj, 3, 0, tp - 1, tp, dt, "cuda")
    g = torch.Generator(device="cuda")
    g.manual_seed(tp * 10 + PROJ.index(proj))
    x = torch.randn(2, q.in_features, generator=g, device="cuda").to(dt)
    y = q.gemv(x)
    f = lambda t: None if t is None else t.float().cpu().numpy()  # noqa: E731
    ref = orc.forward(f(x), f(q.s2), q.vb.cpu().numpy(), q.rank, f(q.smid), q.ub.cpu().numpy(), f(q.s1), "half2")
    assert_close_to_oracle(y, ref, "f16")


@pytest.mark.parametrize("proj", ["q", "k", "gate", "down"])
def test_gemm_llama3_70b_shapes_m128(proj):
    out_f, in_f, rank = SHAPES_70B[proj]
    L = orc.make_layer(800 + PROJ.index(proj), out_f, in_f, rank, 128, "bf16", with_mid=(proj == "k"))
    d = DeviceLayer(L, "bf16")
    y, ws = capi_gemm(d, precise=True)
    ref = orc.forward_dense(d.xr, d.s2r, L.V, d.smidr, L.U, d.s1r)
    assert_close_to_oracle(y, ref, "bf16")
    assert workspace_status(ws) == 0


@pytest.mark.parametrize("proj", ["o", "gate", "down"])
def test_gemm_llama3_70b_shapes_m2048_sampled_rows(proj):
    out_f, in_f, rank = SHAPES_70B[proj]
    L = orc.make_layer(900 + PROJ.index(proj), out_f, in_f, rank, 2048, "bf16")
    d = DeviceLayer(L, "bf16")
    y, ws = capi_gemm(d, precise=True)
    rows = np.sort(np.random.default_rng(proj.encode()[0]).choice(2048, 64, replace=False))
    ref = orc.forward_dense(d.xr[rows], d.s2r, L.V, d.smidr, L.U, d.s1r)
    assert_close_to_oracle(y[torch.as_tensor(rows, device=y.device)], ref, "bf16")
    assert workspace_status(ws) == 0


@pytest.mark.parametrize("tp,batch,fits", [(2, 1, True), (8, 1, True), (2, 8, False)])
def test_exchange_plan_check_on_70b_shards(tp, batch, fits):
    """NQ_TP_CHECK plans the exchange launches without running them (no peers, no regions).  At
    TP8 every exchange GEMV has its single-launch plan; at TP2 the gate/up shard needs the
    two-launch GEMV, whose stage-1 launch runs one CTA per SM and pulls; at TP2 batch 8 that
    launch needs one CTA per tile (436), which the check reports, so the decoder keeps NCCL sums."""
    import dataclasses

    from nanoquant_b200.decoder import Decoder
    cfg = dataclasses.replace(LLAMA3_70B, layers=1)
    dec = Decoder(cfg, max_seq=64, batch=batch, tp_rank=0, tp=tp, tp_exchange=False, dtype=torch.float16,
                  device="cuda")
    assert dec._exchange_fits() is fits
