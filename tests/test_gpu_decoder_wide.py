"""The decoder at the benchmark models' own widths against the float32 decoder oracle
(oracle/decoder_ref.py, itself pinned to HF LlamaForCausalLM by tests/test_decoder_ref_hf.py):

* Llama-2-7B width (hidden 4096, 32 heads, FFN 11008, ranks 1126 / 2054, vocab 32000), 2 layers,
  a 2048-token prompt -- the shapes bench.py times, with the layer count cut so the float32
  CPU oracle stays affordable;
* Llama-3-70B width (hidden 8192, 64 query / 8 KV heads, FFN 28672, ranks 2208 / 480 / 3488),
  1 layer, a 256-token prompt, vocabulary cut to 4096 (the lm_head's width is not under test).

The oracle is fed the GPU's own greedy tokens (teacher forcing), so both sides see the same
sequence.  Checks per decode step: logits rel-L2 <= 2e-2 (fp16 activations and KV cache through
every layer, as in tests/test_gpu_decoder.py), and the same argmax wherever the oracle's top-2
margin exceeds the observed logit error by 4x (a closer margin is a tie at fp16 precision)."""
import numpy as np
import pytest
import torch

from nanoquant_b200.configs import LLAMA2_7B, LLAMA3_70B, DecoderConfig
from nanoquant_b200.decoder import Decoder
from oracle import decoder_ref as ref
from oracle import oracle as orc

pytestmark = pytest.mark.gpu
TOL = 2e-2

W7B = DecoderConfig("llama2-7b-2l", LLAMA2_7B.vocab, 4096, 2, 32, 32, 128, 11008, dict(LLAMA2_7B.ranks))
W70B = DecoderConfig("llama3-70b-1l", 4096, 8192, 1, 64, 8, 128, 28672, dict(LLAMA3_70B.ranks),
                     rope_theta=LLAMA3_70B.rope_theta)


def check_argmax(got: torch.Tensor, want: torch.Tensor):
    top2 = torch.topk(want, 2).values
    margin = float(top2[0] - top2[1])
    err = float((got - want).abs().max())
    if margin > 4 * err:
        assert int(torch.argmax(got)) == int(torch.argmax(want)), (margin, err)


@pytest.mark.parametrize("cfg,prompt_len,steps", [(W7B, 2048, 4), (W70B, 256, 3)], ids=["7b-width", "70b-width"])
def test_wide_decoder_matches_oracle(cfg, prompt_len, steps):
    torch.manual_seed(0)
    dec = Decoder(cfg, max_seq=prompt_len + steps + 8, batch=1, seed=21, dtype=torch.float16, device="cuda")
    W = ref.extract(dec)
    prompt = torch.randint(0, cfg.vocab, (prompt_len,), generator=torch.Generator().manual_seed(9))
    oracle = ref.Incremental(cfg, W)
    want = oracle.feed(prompt.tolist())
    first = int(dec.prefill(prompt.cuda())[0])
    # prefill returns only the token: compare it where the oracle's top-2 margin is clear of the
    # logit error the decode steps tolerate (TOL x the rms logit, x4)
    top2 = torch.topk(want, 2).values
    if float(top2[0] - top2[1]) > 4 * TOL * float(want.pow(2).mean().sqrt()):
        assert first == int(torch.argmax(want))
    tok = first
    for _ in range(steps):
        got = dec.step_logits().float().cpu()[0]
        want = oracle.feed([tok])
        assert orc.rel_l2(got.numpy(), want.numpy()) <= TOL
        check_argmax(got, want)
        tok = int(torch.argmax(got))
        dec.tokens.fill_(tok)
        dec.pos.add_(1)
        dec.seq_len.add_(1)
    assert np.isfinite(got.numpy()).all()
