"""Host side of the packed-checkpoint loader (nanoquant_b200/loader.py): the reference's file
handling and consistency checks (src/nanoquant/utils/load_utils.py:324-402), on the checkpoint that
tests/golden/make_checkpoint.py exported with the reference's own packer."""
import os
import shutil

import pytest
import torch

from nanoquant_b200 import loader

CKPT = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "tiny_llama_nq.pt")


def fixture():
    return torch.load(CKPT, weights_only=True)


def test_read_file_and_directory(tmp_path):
    sd = loader.read_state_dict(CKPT)
    assert sum(k.endswith("_packed") for k in sd) == 28
    d = tmp_path / "nq"
    d.mkdir()
    torch.save(fixture()["state_dict"], d / "model_state.pt")
    assert set(loader.read_state_dict(str(d))) == set(sd)
    with pytest.raises(FileNotFoundError):
        loader.read_state_dict(str(tmp_path / "missing"))
    empty = tmp_path / "empty"
    empty.mkdir()
    with pytest.raises(FileNotFoundError, match="model.safetensors or model_state.pt"):
        loader.read_state_dict(str(empty))


def test_check_packed_keeps_planes_packed():
    factors, rest = loader.check_packed(fixture()["state_dict"])
    assert len(factors) == 28
    plane, shape = factors["model.layers.0.self_attn.q_proj.V"]
    assert plane.dtype == torch.int32 and shape == (96, 256) and tuple(plane.shape) == (96, 8)
    assert "model.layers.1.mlp.down_proj.scale_mid" in rest and "model.embed_tokens.weight" in rest


def test_check_packed_errors_match_reference():
    sd = fixture()["state_dict"]
    key = "model.layers.0.self_attn.q_proj"
    bad = dict(sd)
    del bad[key + ".V_shape"]
    with pytest.raises(ValueError, match="missing its shape key"):
        loader.check_packed(bad)
    bad = dict(sd)
    bad[key + ".V"] = torch.ones(96, 256)
    with pytest.raises(ValueError, match="both packed and unpacked"):
        loader.check_packed(bad)
    bad = dict(sd)
    bad[key + ".V_shape"] = torch.tensor([96, 0])
    with pytest.raises(ValueError, match="Invalid shape"):
        loader.check_packed(bad)
    bad = dict(sd)
    bad[key + ".V_packed"] = sd[key + ".V_packed"].long()
    with pytest.raises(ValueError, match="must be int32"):
        loader.check_packed(bad)
    bad = dict(sd)
    del bad[key + ".U_packed"]
    with pytest.raises(ValueError, match="Shape metadata without packed factors"):
        loader.check_packed(bad)


def test_config_from_hf():
    cfg = loader.config_from_hf(fixture()["config"])
    assert (cfg.vocab, cfg.hidden, cfg.layers, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn) == \
        (512, 256, 2, 2, 1, 128, 512)
    assert cfg.rope_theta == 10000.0 and cfg.rms_eps == 1e-5
