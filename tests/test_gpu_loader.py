"""The packed-checkpoint loader on the GPU: a checkpoint exported by the reference's own packer
(tests/golden/make_checkpoint.py: HF Llama whose linears are the reference's NanoQuantLinear) is
loaded with its planes kept packed (lsb_first -> half2 on the device) into the decoder, whose
prefill + decode logits must match the reference model's own float32 logits for the same tokens.
Tolerance as in the other decoder tests: rel-L2 <= 2e-2 (fp16 activations and KV cache)."""
import os

import pytest
import torch

from nanoquant_b200 import loader
from oracle import oracle as orc

pytestmark = pytest.mark.gpu
CKPT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "tiny_llama_nq.pt")
TOL = 2e-2


def test_loaded_decoder_matches_reference_model():
    fx = torch.load(CKPT, weights_only=True)
    tokens, golden = fx["tokens"], fx["logits"]
    dec = loader.load_compressed_decoder(fx["config"], CKPT, max_seq=64, dtype=torch.float16, device="cuda")
    assert dec.layers[1]["down"].smid is not None and dec.layers[0]["q"].smid is None
    P = 36
    first = int(dec.prefill(torch.tensor(tokens[:P]).cuda())[0])
    want = golden[P - 1]
    top2 = torch.topk(want, 2).values
    if float(top2[0] - top2[1]) > 4 * TOL * float(want.pow(2).mean().sqrt()):
        assert first == int(torch.argmax(want))
    for p in range(P, len(tokens)):
        dec.tokens.fill_(tokens[p])
        got = dec.step_logits().float().cpu()[0]
        assert orc.rel_l2(got.numpy(), golden[p].numpy()) <= TOL, p
        dec.pos.add_(1)
        dec.seq_len.add_(1)
