"""Loading packed NanoQuant checkpoints onto the GPU with no dense unpack.

The reference loader (src/nanoquant/utils/load_utils.py) reads a checkpoint written by
get_compressed_state_dict (:304-321) -- every NanoQuant factor as an lsb_first int32 plane
``<prefix>.V_packed`` / ``U_packed`` plus ``<prefix>.V_shape`` / ``U_shape`` (modules/linear.py:359-433),
scales and every other weight as plain tensors -- and expands each plane into a dense bf16 +-1 matrix
on the CPU (``_load_and_process_state_dict``, :324-402) before building an HF model whose linears
become NanoQuantLinear (``load_compressed_model``, :405-527).

Here the planes stay packed end to end: they are copied to the GPU as they are (4 bytes per 32
signs) and converted to the kernels' half2 bit order there (nq_repack_signs), then handed to the
Llama decoder of this package, sharded for tensor parallelism.

* ``read_state_dict``         the reference's file handling: a file, or a directory holding
                              ``model.safetensors`` or ``model_state.pt``; torch.load with mmap and
                              weights_only when available;
* ``check_packed``            the reference's consistency checks on packed factors (same errors),
                              without the unpack;
* ``config_from_hf``          a DecoderConfig from an HF Llama config (dict or object);
* ``load_compressed_decoder`` the decoder for one tensor-parallel rank.
"""
from __future__ import annotations

import inspect
import os
from pathlib import Path
from typing import Any, Dict, Optional, Tuple

import torch

from . import _lib
from .configs import PROJ, DecoderConfig

HF_PROJ = {"q": "self_attn.q_proj", "k": "self_attn.k_proj", "v": "self_attn.v_proj", "o": "self_attn.o_proj",
           "gate": "mlp.gate_proj", "up": "mlp.up_proj", "down": "mlp.down_proj"}


def read_state_dict(checkpoint_path: str) -> Dict[str, Any]:
    """The state dict of a checkpoint file or NanoQuant directory (load_utils.py:324-371)."""
    if not os.path.exists(checkpoint_path):
        raise FileNotFoundError(f"Could not find model weights at {checkpoint_path}")
    path = Path(checkpoint_path)
    if path.is_dir():
        st, pt = path / "model.safetensors", path / "model_state.pt"
        if st.is_file():
            try:
                from safetensors.torch import load_file
            except ImportError as error:
                raise ImportError("Loading this NanoQuant directory requires safetensors") from error
            sd = load_file(str(st), device="cpu")
            path = None
        elif pt.is_file():
            path = pt
        else:
            raise FileNotFoundError(
                f"No model.safetensors or model_state.pt found in NanoQuant directory {checkpoint_path}")
    if path is not None:
        sig = inspect.signature(torch.load)
        kwargs = {"map_location": "cpu"}
        if "mmap" in sig.parameters:
            kwargs["mmap"] = True
        if "weights_only" in sig.parameters:
            kwargs["weights_only"] = True
        try:
            sd = torch.load(path, **kwargs)
        except Exception:
            if not kwargs.get("weights_only", False):
                raise
            kwargs["weights_only"] = False  # only for a trusted checkpoint, as the reference does
            sd = torch.load(path, **kwargs)
    if isinstance(sd, dict) and "state_dict" in sd and isinstance(sd["state_dict"], dict):
        sd = sd["state_dict"]
    if not isinstance(sd, dict):
        raise TypeError(f"Expected a state_dict dict from {checkpoint_path}, got {type(sd)}")
    return sd


def check_packed(sd: Dict[str, Any]) -> Tuple[Dict[str, Tuple[torch.Tensor, Tuple[int, int]]], Dict[str, Any]]:
    """Split a state dict into packed factors {"<prefix>.<V|U>": (int32 plane, (rows, cols))} and
    the rest, with the reference's checks and messages (load_utils.py:379-399)."""
    packed = {k: v for k, v in sd.items() if k.endswith("_packed")}
    shapes = {k: v for k, v in sd.items() if k.endswith("_shape")}
    rest = {k: v for k, v in sd.items() if not (k.endswith("_packed") or k.endswith("_shape"))}
    factors = {}
    for pk, pv in packed.items():
        prefix, packed_name = pk.rsplit(".", 1)
        base = packed_name[:-7]
        sk = f"{prefix}.{base}_shape"
        st = shapes.get(sk, None)
        if st is None:
            raise ValueError(f"Packed factor {pk} is missing its shape key {sk}")
        if f"{prefix}.{base}" in rest:
            raise ValueError(f"Checkpoint contains both packed and unpacked factors for {prefix}.{base}")
        shape = tuple(int(x) for x in (st.tolist() if isinstance(st, torch.Tensor) else st))
        if len(shape) != 2 or any(size <= 0 for size in shape):
            raise ValueError(f"Invalid shape for {pk}: {shape}")
        if pv.dtype != torch.int32:
            raise ValueError(f"Packed factor {pk} must be int32, got {pv.dtype}")
        if tuple(pv.shape) != (shape[0], (shape[1] + 31) // 32):
            raise ValueError(f"Packed factor {pk} has shape {tuple(pv.shape)}, expected "
                             f"({shape[0]}, {(shape[1] + 31) // 32}) for {shape}")
        factors[f"{prefix}.{base}"] = (pv, shape)
    orphan = [key for key in shapes if key[:-6] + "_packed" not in packed]
    if orphan:
        raise ValueError(f"Shape metadata without packed factors: {orphan[:10]}")
    return factors, rest


def config_from_hf(conf, name: str = "checkpoint", ranks: Optional[Dict[str, int]] = None) -> DecoderConfig:
    """DecoderConfig of an HF Llama config (a dict or a config object)."""
    c = conf if isinstance(conf, dict) else conf.to_dict()
    heads = int(c["num_attention_heads"])
    head_dim = int(c.get("head_dim") or c["hidden_size"] // heads)
    rope = c.get("rope_parameters") or {}
    theta = float(rope.get("rope_theta", c.get("rope_theta", 10000.0)))
    return DecoderConfig(name, int(c["vocab_size"]), int(c["hidden_size"]), int(c["num_hidden_layers"]), heads,
                         int(c.get("num_key_value_heads") or heads), head_dim, int(c["intermediate_size"]),
                         dict(ranks or {}), rms_eps=float(c.get("rms_norm_eps", 1e-5)), rope_theta=theta)


def _half2(plane: torch.Tensor, cols: int, device) -> torch.Tensor:
    """An lsb_first plane, copied to the device as it is and reordered to half2 there."""
    p = plane.to(device=device, dtype=torch.int32, non_blocking=False).contiguous()
    return torch.ops.nq_b200.repack_signs(p, int(cols), "lsb_first", "half2")


def gpu_weights(sd: Dict[str, Any], cfg: DecoderConfig, device, prefix: str = "model.") -> dict:
    """The decoder's weights from a packed state dict, planes in half2 order on ``device``."""
    _lib.load_torch_ops()
    factors, rest = check_packed(sd)

    def get(key):
        if key not in rest:
            raise RuntimeError(f"Checkpoint does not match the model: missing weight {key}")
        return rest[key]

    out = {"embed": get(f"{prefix}embed_tokens.weight"), "final_norm": get(f"{prefix}norm.weight")}
    out["lm_head"] = rest.get("lm_head.weight", out["embed"])  # a tied head may be absent (load_utils.py:505-509)
    layers = []
    for li in range(cfg.layers):
        lp = f"{prefix}layers.{li}."
        w = {"in_norm": get(lp + "input_layernorm.weight"), "post_norm": get(lp + "post_attention_layernorm.weight")}
        for p in PROJ:
            base = lp + HF_PROJ[p]
            missing = [k for k in (base + ".V", base + ".U") if k not in factors]
            missing += [base + "." + k for k in ("scale_pre", "scale_post") if base + "." + k not in rest]
            if missing:
                raise RuntimeError(f"Incomplete compressed layer {base}; missing weights: {missing}")
            (vp, (r, in_f)), (up, (out_f, r2)) = factors[base + ".V"], factors[base + ".U"]
            if r != r2 or (out_f, in_f) != cfg.io(p):
                raise RuntimeError(f"{base}: factor shapes V {(r, in_f)} / U {(out_f, r2)} do not fit {cfg.io(p)}")
            w[p] = (_half2(vp, in_f, device), _half2(up, r, device), rest[base + ".scale_pre"],
                    rest.get(base + ".scale_mid"), rest[base + ".scale_post"])
        layers.append(w)
    out["layers"] = layers
    return out


def load_compressed_decoder(model_config, checkpoint_path: str, max_seq: int, batch: int = 1, tp_rank: int = 0,
                            tp: int = 1, group=None, dtype=torch.float16, device=None, **decoder_kwargs):
    """The Llama decoder of one tensor-parallel rank, loaded from a packed NanoQuant checkpoint
    (load_compressed_model, load_utils.py:405-527, without the dense unpack).  ``model_config``:
    an HF Llama config (dict or object) or a DecoderConfig."""
    from .decoder import Decoder
    cfg = model_config if isinstance(model_config, DecoderConfig) else config_from_hf(model_config)
    dev = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
    sd = read_state_dict(checkpoint_path)
    if "lm_head.weight" in sd or "model.embed_tokens.weight" in sd:
        prefix = "model."
    else:
        prefix = ""
    weights = gpu_weights(sd, cfg, dev, prefix)
    ranks = {p: int(weights["layers"][0][p][0].shape[0]) for p in PROJ}
    cfg = DecoderConfig(cfg.name, cfg.vocab, cfg.hidden, cfg.layers, cfg.heads, cfg.kv_heads, cfg.head_dim, cfg.ffn,
                        ranks, rms_eps=cfg.rms_eps, rope_theta=cfg.rope_theta)
    return Decoder(cfg, max_seq=max_seq, batch=batch, tp_rank=tp_rank, tp=tp, group=group, dtype=dtype, device=dev,
                   weights=weights, **decoder_kwargs)
