"""Pins the float32 decoder oracle (oracle/decoder_ref.py) to HF transformers' LlamaForCausalLM,
the model the reference's decode harness runs (src/nanoquant/kernel/test_decode.py), on the
same weights: every NanoQuant factorisation multiplied out into the dense projection weight
diag(s1) U diag(smid) V^T diag(s2) that HF's nn.Linear holds.  Both run in float32 on the
CPU; they differ only in summation order (rel-L2 well below 1e-5).  Also checks that the
oracle's KV-cached incremental mode equals its whole-sequence form."""
import numpy as np
import pytest
import torch

from nanoquant_b200.configs import DecoderConfig
from oracle import decoder_ref as ref
from oracle import oracle as orc

transformers = pytest.importorskip("transformers")

CFGS = [
    DecoderConfig("hf-pin-gqa", 300, 256, 2, 4, 2, 64, 384,
                  {"q": 96, "k": 40, "v": 40, "o": 96, "gate": 130, "up": 130, "down": 130}),
    DecoderConfig("hf-pin-mha", 200, 128, 1, 2, 2, 64, 256,
                  {"q": 50, "k": 50, "v": 50, "o": 50, "gate": 70, "up": 70, "down": 70}, rope_theta=500000.0),
]


def random_weights(cfg, seed):
    g = torch.Generator().manual_seed(seed)
    sign = lambda r, c: (torch.randint(0, 2, (r, c), generator=g) * 2 - 1).float()  # noqa: E731
    layers = []
    for _ in range(cfg.layers):
        L = {}
        for p in ("q", "k", "v", "o", "gate", "up", "down"):
            out_f, in_f = cfg.io(p)
            r = cfg.ranks[p]
            L[p] = {"V": sign(r, in_f), "U": sign(out_f, r),
                    "s2": torch.rand(in_f, generator=g) / in_f ** 0.5 + 0.01,
                    "s1": torch.rand(out_f, generator=g) / r ** 0.5 + 0.01,
                    "smid": torch.rand(r, generator=g) + 0.5 if p in ("k", "down") else None}
        L["in_norm"] = torch.rand(cfg.hidden, generator=g) + 0.5
        L["post_norm"] = torch.rand(cfg.hidden, generator=g) + 0.5
        layers.append(L)
    return {"layers": layers, "embed": torch.randn(cfg.vocab, cfg.hidden, generator=g),
            "lm_head": torch.randn(cfg.vocab, cfg.hidden, generator=g) * 0.05,
            "final_norm": torch.rand(cfg.hidden, generator=g) + 0.5}


def dense(w):
    """The projection weight [out, in] of one factorisation (linear.py:282-291 multiplied out)."""
    mid = w["smid"] if w["smid"] is not None else torch.ones(w["V"].shape[0])
    return (w["s1"][:, None] * w["U"] * mid[None, :]) @ (w["V"] * w["s2"][None, :])


def hf_model(cfg, W):
    conf = transformers.LlamaConfig(
        vocab_size=cfg.vocab, hidden_size=cfg.hidden, intermediate_size=cfg.ffn, num_hidden_layers=cfg.layers,
        num_attention_heads=cfg.heads, num_key_value_heads=cfg.kv_heads, head_dim=cfg.head_dim,
        rms_norm_eps=cfg.rms_eps, rope_parameters={"rope_type": "default", "rope_theta": cfg.rope_theta},
        max_position_embeddings=4096, tie_word_embeddings=False, attention_bias=False, mlp_bias=False)
    conf._attn_implementation = "eager"
    m = transformers.LlamaForCausalLM(conf).float().eval()
    with torch.no_grad():
        m.model.embed_tokens.weight.copy_(W["embed"])
        m.lm_head.weight.copy_(W["lm_head"])
        m.model.norm.weight.copy_(W["final_norm"])
        for lay, L in zip(m.model.layers, W["layers"]):
            a, f = lay.self_attn, lay.mlp
            for name, mod in (("q", a.q_proj), ("k", a.k_proj), ("v", a.v_proj), ("o", a.o_proj),
                              ("gate", f.gate_proj), ("up", f.up_proj), ("down", f.down_proj)):
                mod.weight.copy_(dense(L[name]))
            lay.input_layernorm.weight.copy_(L["in_norm"])
            lay.post_attention_layernorm.weight.copy_(L["post_norm"])
    return m


@pytest.mark.parametrize("cfg", CFGS, ids=lambda c: c.name)
def test_decoder_oracle_matches_hf_llama(cfg):
    W = random_weights(cfg, 3)
    tokens = torch.randint(0, cfg.vocab, (37,), generator=torch.Generator().manual_seed(5))
    want = hf_model(cfg, W)(tokens[None]).logits[0].detach()
    got = ref.logits(cfg, W, tokens.tolist())
    assert got.shape == want.shape
    assert orc.rel_l2(got.numpy(), want.numpy()) <= 1e-5


@pytest.mark.parametrize("cfg", CFGS, ids=lambda c: c.name)
def test_incremental_oracle_matches_whole_sequence(cfg):
    W = random_weights(cfg, 4)
    tokens = torch.randint(0, cfg.vocab, (30,), generator=torch.Generator().manual_seed(6)).tolist()
    whole = ref.logits(cfg, W, tokens)
    inc = ref.Incremental(cfg, W)
    got = [inc.feed(tokens[:25])]
    for t in tokens[25:]:
        got.append(inc.feed([t]))
    for i, g in enumerate(got):
        np.testing.assert_allclose(g.numpy(), whole[24 + i].numpy(), rtol=1e-4, atol=1e-5)
