"""Generate a small packed NanoQuant checkpoint with the reference's own code, and its logits.

Run once in a container that has the reference checkout; the output is committed next to this
script (tiny_llama_nq.pt):

    NQ_REFERENCE_SRC=<reference>/src python tests/golden/make_checkpoint.py

What it does, with the reference's functions (paths inside the reference project):
  * builds a random-init HF LlamaForCausalLM (hidden 256, 2 layers, 2 query / 1 KV heads,
    head_dim 128, FFN 512, vocab 512) and turns every nn.Linear but lm_head into the reference's
    NanoQuantLinear the way its loader does (modules/linear.py init_for_inference, as in
    utils/load_utils.py:457-469), with seeded +-1 factors and scales (some layers with scale_mid);
  * exports the packed checkpoint as utils/load_utils.py:304-321 get_compressed_state_dict does:
    for a model without linearized blocks its body is model.state_dict(), which runs the reference
    NanoQuantLinear's packer (lsb_first int32 planes + shapes, modules/linear.py:359-433); the
    function itself is not imported because load_utils pulls in the reference's training and
    evaluation stack (cut_cross_entropy, lm_eval), which is not installed;
  * records the reference model's own float32 logits (dense factors, _compute_forward) for a
    fixed token sequence.
"""
import os
import sys

os.environ.setdefault("TORCHDYNAMO_DISABLE", "1")
HERE = os.path.dirname(os.path.abspath(__file__))
REPO = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, REPO)
sys.path.insert(0, os.environ.get("NQ_REFERENCE_SRC", os.path.join(os.path.dirname(REPO), "reference", "src")))

import numpy as np  # noqa: E402
import torch  # noqa: E402
import transformers  # noqa: E402

from nanoquant.modules.linear import NanoQuantLinear  # noqa: E402

from oracle import oracle as orc  # noqa: E402

RANKS = {"q_proj": 96, "k_proj": 40, "v_proj": 40, "o_proj": 96, "gate_proj": 130, "up_proj": 130, "down_proj": 130}
WITH_MID = {"k_proj", "down_proj"}
TOKENS = [int(t) for t in orc.splitmix64(77, 40) % np.uint64(512)]


def main():
    conf = transformers.LlamaConfig(
        vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=2, num_attention_heads=2,
        num_key_value_heads=1, head_dim=128, rms_norm_eps=1e-5,
        rope_parameters={"rope_type": "default", "rope_theta": 10000.0}, max_position_embeddings=1024,
        tie_word_embeddings=False, attention_bias=False, mlp_bias=False)
    conf._attn_implementation = "eager"
    torch.manual_seed(0)
    model = transformers.LlamaForCausalLM(conf).bfloat16().eval()
    seed = 5000
    with torch.no_grad():
        model.model.embed_tokens.weight.copy_(torch.from_numpy(orc.random_normal(seed, 512 * 256).reshape(512, 256)) * 0.5)
        model.lm_head.weight.copy_(torch.from_numpy(orc.random_normal(seed + 1, 512 * 256).reshape(512, 256)) * 0.05)
        model.model.norm.weight.copy_(torch.from_numpy(np.abs(orc.random_normal(seed + 2, 256)) + 0.5))
        for li, layer in enumerate(model.model.layers):
            layer.input_layernorm.weight.copy_(torch.from_numpy(np.abs(orc.random_normal(seed + 10 + li, 256)) + 0.5))
            layer.post_attention_layernorm.weight.copy_(
                torch.from_numpy(np.abs(orc.random_normal(seed + 20 + li, 256)) + 0.5))
            mods = dict(layer.self_attn.named_children())
            mods.update(dict(layer.mlp.named_children()))
            for j, (name, lin) in enumerate(sorted(mods.items())):
                if name not in RANKS:
                    continue
                r = RANKS[name]
                out_f, in_f = lin.out_features, lin.in_features
                lin.__class__ = NanoQuantLinear
                lin.init_for_inference(r, has_scale_mid=name in WITH_MID)
                s = seed + 100 * (li + 1) + j
                lin.V.copy_(torch.from_numpy(orc.random_signs(s, r, in_f, 1).astype(np.float32)))
                lin.U.copy_(torch.from_numpy(orc.random_signs(s, out_f, r, 2).astype(np.float32)))
                lin.scale_pre.copy_(torch.from_numpy(np.abs(orc.random_normal(s, in_f, 3)) / np.sqrt(in_f)).reshape(1, -1))
                lin.scale_post.copy_(torch.from_numpy(np.abs(orc.random_normal(s, out_f, 4)) / np.sqrt(r)).reshape(1, -1))
                if name in WITH_MID:
                    lin.scale_mid.copy_(torch.from_numpy(np.abs(orc.random_normal(s, r, 5)) + 0.5).reshape(1, -1))
    # the checkpoint in bf16 like the reference's own exports (NanoQuantLinear keeps bf16 scales);
    # the golden logits from the same bf16-rounded weights, evaluated in float32
    model = model.bfloat16()
    assert not any(isinstance(m, NanoQuantLinear) and m.do_train for m in model.modules())
    sd = {k: v.clone() for k, v in model.state_dict().items()}
    with torch.no_grad():
        logits = model.float()(torch.tensor([TOKENS])).logits[0].float().numpy()
    path = os.path.join(HERE, "tiny_llama_nq.pt")
    torch.save({"config": conf.to_dict(), "state_dict": sd, "tokens": TOKENS, "logits": torch.from_numpy(logits)},
               path)
    print(f"wrote {path}: {len(sd)} tensors, {os.path.getsize(path)} bytes; "
          f"packed keys {sum(k.endswith('_packed') for k in sd)}")


if __name__ == "__main__":
    main()
