"""Whole-decoder checks on one GPU: prefill + decode logits against the float32 reference
decoder (oracle/decoder_ref.py), graph replay identical to eager steps.

Tolerance: rel-L2 of the logits <= 2e-2 (fp16 activations and KV cache through every layer)."""
import numpy as np
import pytest
import torch

from nanoquant_b200.decoder import TINY, Decoder
from oracle import decoder_ref as ref
from oracle import oracle as orc

pytestmark = pytest.mark.gpu
TOL = 2e-2


def make(with_mid=False, max_seq=96):
    return Decoder(TINY, max_seq=max_seq, batch=1, seed=7, dtype=torch.float16, device="cuda", with_mid=with_mid)


@pytest.mark.parametrize("with_mid", [False, True])
def test_prefill_and_decode_match_reference(with_mid):
    dec = make(with_mid)
    W = ref.extract(dec)
    prompt = torch.randint(0, TINY.vocab, (45,), generator=torch.Generator().manual_seed(3))
    first = dec.prefill(prompt.cuda())
    want = ref.logits(TINY, W, prompt.tolist())[-1]
    assert int(first[0]) == int(torch.argmax(want))
    seq = prompt.tolist() + [int(first[0])]
    for _ in range(6):
        got = dec.step_logits().float().cpu()[0]
        want = ref.logits(TINY, W, seq)[-1]
        assert orc.rel_l2(got.numpy(), want.numpy()) <= TOL
        nxt = int(torch.argmax(got))
        seq.append(nxt)
        dec.tokens.fill_(nxt)
        dec.pos.add_(1)
        dec.seq_len.add_(1)


def test_graph_replay_matches_eager_steps():
    prompt = torch.randint(0, TINY.vocab, (33,), generator=torch.Generator().manual_seed(4)).cuda()
    a, b = make(), make()
    a.prefill(prompt)
    b.prefill(prompt)
    eager = [int(a.step()[0]) for _ in range(8)]
    g = b.capture(warmup=2)
    graphed = [int(g.replay()[0]) for _ in range(8)]
    assert eager == graphed
    assert torch.equal(a.k_cache, b.k_cache) and torch.equal(a.v_cache, b.v_cache)
    host_in = torch.tensor([graphed[-1]], dtype=torch.long).pin_memory()
    host_out = torch.empty(1, dtype=torch.long).pin_memory()
    nxt = int(g.generate(host_in, host_out)[0])
    assert nxt == int(a.step()[0])
    g.release()


def test_decode_attention_against_reference():
    """Split-KV attention (several chunks, GQA group 4) against float32 softmax attention."""
    B, hq, hkv, D, S = 2, 8, 2, 128, 700
    g = torch.Generator().manual_seed(0)
    q = torch.randn(B, hq, D, generator=g).half()
    kc = torch.randn(B, hkv, S, D, generator=g).half()
    vc = torch.randn(B, hkv, S, D, generator=g).half()
    L = torch.tensor([700, 257], dtype=torch.int32)
    out = torch.ops.nq_b200.decode_attention(q.cuda(), kc.cuda(), vc.cuda(), L.cuda()).float().cpu()
    for b in range(B):
        n = int(L[b])
        k = kc[b, :, :n].float().repeat_interleave(hq // hkv, 0)
        v = vc[b, :, :n].float().repeat_interleave(hq // hkv, 0)
        w = torch.softmax((q[b].float()[:, None, :] @ k.transpose(1, 2))[:, 0] / np.sqrt(D), -1)
        want = (w[:, None, :] @ v)[:, 0]
        assert orc.rel_l2(out[b].numpy(), want.numpy()) < 2e-3


def test_rmsnorm_and_silu_against_torch():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(3, 4096, generator=g).half().cuda()
    r = torch.randn(3, 4096, generator=g).half().cuda()
    w = (torch.rand(4096, generator=g) + 0.5).half().cuda()
    out, res = torch.ops.nq_b200.rmsnorm(x, r, w, 1e-5)
    h = (x + r)
    assert torch.equal(res, h)
    hf = h.float()
    want = (w.float() * (hf * torch.rsqrt(hf.pow(2).mean(-1, keepdim=True) + 1e-5)).half().float())
    assert orc.rel_l2(out.float().cpu().numpy(), want.cpu().numpy()) < 1e-3
    a = torch.ops.nq_b200.silu_mul(x, r)
    want = (torch.nn.functional.silu(x.float()).half().float() * r.float())
    assert orc.rel_l2(a.float().cpu().numpy(), want.cpu().numpy()) < 1e-3
