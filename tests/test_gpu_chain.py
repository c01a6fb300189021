"""GEMV chains on the GPU (nq_gemv_chain through the C ABI).

* A single PLAIN phase computes exactly what nq_gemv / nq_gemv_group compute: same bits.
* The 7B decoder-block chain (o + residual, gate/up from RMSNorm, down from SiLU(gate) * up
  + residual, next q/k/v from RMSNorm) against the same steps as separate launches
  (nq_b200.gemv / gemv_group / rmsnorm / silu_mul): rel-L2 <= 1e-3 per output.  The only
  difference is the summation order of the RMSNorm mean, so most values agree to the bit.
* A whole decoder decodes the same tokens with and without chains."""
import pytest
import torch

from nanoquant_b200 import chain
from nanoquant_b200.decoder import TINY, Decoder, QuantLinearShard, _random_planes
from oracle import oracle as orc

pytestmark = pytest.mark.gpu


def layer(out_f, in_f, r, dt, seed, with_mid=False):
    g = torch.Generator(device="cuda")
    g.manual_seed(seed)
    vb = _random_planes(g, r, in_f, "cuda")
    ub = _random_planes(g, out_f, r, "cuda")
    s2 = (torch.randn(in_f, generator=g, device="cuda").abs() / in_f ** 0.5).to(dt)
    s1 = (torch.randn(out_f, generator=g, device="cuda").abs() / r ** 0.5).to(dt)
    smid = (torch.randn(r, generator=g, device="cuda").abs() + 0.5).to(dt) if with_mid else None
    return QuantLinearShard(vb, ub, s2, smid, s1)


def ws_for(phases, batch=1):
    n = chain.workspace_bytes(phases, batch)
    assert n, chain.why_not()
    return torch.zeros(n, dtype=torch.uint8, device="cuda")


def rel(a, b):
    return orc.rel_l2(a.float().cpu().numpy(), b.float().cpu().numpy())


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
@pytest.mark.parametrize("shape", [(4096, 4096, 1126, 1), (11008, 4096, 2054, 2), (4096, 11008, 2054, 1),
                                   (1000, 520, 200, 3)])
def test_single_plain_phase_matches_gemv_bitwise(shape, dt):
    out_f, in_f, r, n = shape
    Ls = [layer(out_f, in_f, r, dt, 10 + i, with_mid=(i == 1)) for i in range(n)]
    x = torch.randn(1, in_f, device="cuda").to(dt)
    ph = [chain.Phase(Ls, x)]
    got = chain.run(ph, ws_for(ph))[0]
    if n == 1:
        want = [Ls[0].gemv(x)]
    else:
        want = torch.ops.nq_b200.gemv_group(x, [L.s2 for L in Ls], [L.vb for L in Ls], [L.smid for L in Ls],
                                            [L.ub for L in Ls], [L.s1 for L in Ls])
    for a, b in zip(got, want):
        assert torch.equal(a, b)


@pytest.mark.parametrize("gate_act", [False, True])
@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_decoder_block_chain_matches_separate_launches(dt, gate_act):
    _block_chain(dt, gate_act)


def _block_chain(dt, gate_act):
    """Runs the o / MLP / next-q/k/v chain against the separate launches (asserting as it goes)
    and returns the residual stream and the next block's q/k/v."""
    hid, ffn, ra, rm = 4096, 11008, 1126, 2054
    o = layer(hid, hid, ra, dt, 1)
    gate, up = layer(ffn, hid, rm, dt, 2), layer(ffn, hid, rm, dt, 3)
    down = layer(hid, ffn, rm, dt, 4)
    q, k, v = (layer(hid, hid, ra, dt, 5 + i) for i in range(3))
    gen = torch.Generator(device="cuda")
    gen.manual_seed(0)
    post_w = (torch.rand(hid, generator=gen, device="cuda") + 0.5).to(dt)
    in_w = (torch.rand(hid, generator=gen, device="cuda") + 0.5).to(dt)
    a = torch.randn(1, hid, generator=gen, device="cuda").to(dt)
    h0 = torch.randn(1, hid, generator=gen, device="cuda").to(dt)
    eps = 1e-5
    # separate launches
    o_out = o.gemv(a)
    xg, h1 = torch.ops.nq_b200.rmsnorm(o_out, h0, post_w, eps)
    g_out, u_out = torch.ops.nq_b200.gemv_group(xg, [gate.s2, up.s2], [gate.vb, up.vb], [None, None],
                                                [gate.ub, up.ub], [gate.s1, up.s1])
    act = torch.ops.nq_b200.silu_mul(g_out, u_out)
    d_out = down.gemv(act)
    xq, h2 = torch.ops.nq_b200.rmsnorm(d_out, h1, in_w, eps)
    want_qkv = torch.ops.nq_b200.gemv_group(xq, [m.s2 for m in (q, k, v)], [m.vb for m in (q, k, v)],
                                            [None] * 3, [m.ub for m in (q, k, v)], [m.s1 for m in (q, k, v)])
    # one chain
    h = h0.clone()
    g_buf, u_buf = torch.empty(1, ffn, device="cuda", dtype=dt), torch.empty(1, ffn, device="cuda", dtype=dt)
    ph = [chain.Phase([o], a, residual=h, out=[h]),
          chain.Phase([gate, up], h, chain.RMSNORM, norm_weight=post_w, eps=eps, out=[g_buf, u_buf],
                      act=1 if gate_act else 0),
          chain.Phase([down], g_buf, chain.MUL if gate_act else chain.SILU_MUL, x2=u_buf, residual=h, out=[h]),
          chain.Phase([q, k, v], h, chain.RMSNORM, norm_weight=in_w, eps=eps)]
    ws = ws_for(ph)
    outs = chain.run(ph, ws)
    torch.cuda.synchronize()
    if gate_act:  # the gate buffer holds dtype(silu(gate))
        g_out = (g_out.float() / (1 + torch.exp(-g_out.float()))).to(dt)
    assert rel(g_buf, g_out) <= 1e-3 and rel(u_buf, u_out) <= 1e-3
    assert rel(h, h2) <= 1e-3
    for got, want in zip(outs[3], want_qkv):
        assert rel(got, want) <= 1e-3
    # the same chain again on the same workspace (barrier counter and status carry over)
    h.copy_(h0)
    outs2 = chain.run(ph, ws)
    for got, again in zip(outs[3], outs2[3]):
        assert torch.equal(got, again)
    assert int(ws[8:12].view(torch.int32).cpu()[0]) == 0  # control block status word
    return h.clone(), [t.clone() for t in outs[3]]


@pytest.mark.parametrize("dt", [torch.float16, torch.bfloat16])
def test_gate_silu_then_mul_equals_silu_mul_bitwise(dt):
    """act on the gate + MUL computes the same bits as SILU_MUL on the raw gate."""
    h_a, qkv_a = _block_chain(dt, False)
    h_b, qkv_b = _block_chain(dt, True)
    assert torch.equal(h_a, h_b)
    for a, b in zip(qkv_a, qkv_b):
        assert torch.equal(a, b)


def test_decoder_with_and_without_chains_agree():
    prompt = torch.randint(0, TINY.vocab, (33,), generator=torch.Generator().manual_seed(5)).cuda()
    runs = []
    for use_chain in (True, False):
        dec = Decoder(TINY, max_seq=96, seed=11, device="cuda", chain=use_chain)
        assert (dec.chain_ws is not None) == use_chain
        first = int(dec.prefill(prompt)[0])
        logits = dec.step_logits().float()
        dec.tokens.fill_(int(torch.argmax(logits[0])))
        dec.pos.add_(1)
        dec.seq_len.add_(1)
        toks = [int(dec.step()[0]) for _ in range(8)]
        runs.append((first, logits.cpu(), toks))
    assert runs[0][0] == runs[1][0]
    assert rel(runs[0][1], runs[1][1]) <= 1e-2
    assert runs[0][2] == runs[1][2]
