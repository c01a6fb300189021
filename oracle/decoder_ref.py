"""float32 PyTorch reference of the decoder in nanoquant_b200/decoder.py (TEST INFRASTRUCTURE ONLY).

The quantized linears are evaluated as the reference's dense path does it
(src/nanoquant/modules/linear.py:282-291 on factors unpacked by the C oracle), the rest as
HF's Llama modules compute it (RMSNorm in float32, rotate-half RoPE with theta, causal SDPA
with GQA, SwiGLU), all in float32 on the CPU, over the whole sequence without a cache.
"""
from __future__ import annotations

import numpy as np
import torch
import torch.nn.functional as F

from . import oracle as orc


def dense_factors(q) -> dict:
    """Dense float32 +-1 factors and scales of one QuantLinearShard (half2 planes)."""
    vb = q.vb.detach().cpu().numpy()
    ub = q.ub.detach().cpu().numpy()
    r, in_f, out_f = q.rank, q.in_features, q.out_features
    V = torch.from_numpy(orc.unpack(vb, (r, in_f), "half2").astype(np.float32))
    U = torch.from_numpy(orc.unpack(ub, (out_f, r), "half2").astype(np.float32))
    f = lambda t: None if t is None else t.detach().float().cpu()  # noqa: E731
    return {"V": V, "U": U, "s2": f(q.s2), "s1": f(q.s1), "smid": f(q.smid)}


def linear(x, w):
    return orc.dense_forward_torch(x, w["s2"], w["V"], w["smid"], w["U"], w["s1"])


def extract(dec) -> dict:
    layers = []
    for lay in dec.layers:
        d = {p: dense_factors(lay[p]) for p in ("q", "k", "v", "o", "gate", "up", "down")}
        d["in_norm"] = lay["in_norm"].float().cpu()
        d["post_norm"] = lay["post_norm"].float().cpu()
        layers.append(d)
    return {"layers": layers, "embed": dec.embed.float().cpu(), "lm_head": dec.lm_head.float().cpu(),
            "final_norm": dec.final_norm.float().cpu()}


def rope(x, pos, theta):
    """x [T, H, D]; rotate-half pairs (i, i + D/2)."""
    D = x.shape[-1]
    inv = 1.0 / (theta ** (torch.arange(0, D, 2, dtype=torch.float64) / D))
    ang = pos.double()[:, None] * inv[None, :]
    cos = torch.cat([ang.cos(), ang.cos()], -1).float()[:, None, :]
    sin = torch.cat([ang.sin(), ang.sin()], -1).float()[:, None, :]
    x1, x2 = x[..., : D // 2], x[..., D // 2:]
    rot = torch.cat([-x2, x1], -1)
    return x * cos + rot * sin


def rmsnorm(x, w, eps):
    return w * (x * torch.rsqrt(x.pow(2).mean(-1, keepdim=True) + eps))


class Incremental:
    """The same float32 decoder fed a few tokens at a time with a KV cache, as HF's generate
    loop runs it: ``feed(tokens)`` appends tokens and returns the logits of the last one.
    Equal to ``logits(...)[-1]`` of the whole sequence up to float32 summation order."""

    def __init__(self, cfg, W: dict):
        self.cfg, self.W = cfg, W
        self.k = [None] * len(W["layers"])
        self.v = [None] * len(W["layers"])
        self.n = 0

    @torch.no_grad()
    def feed(self, tokens) -> torch.Tensor:
        cfg, W = self.cfg, self.W
        t = torch.as_tensor(tokens, dtype=torch.long).reshape(-1)
        T, D, n = t.numel(), cfg.head_dim, self.n
        pos = torch.arange(n, n + T)
        # query i (position n + i) sees keys 0 .. n + i
        mask = torch.arange(n + T)[None, :] <= pos[:, None]
        rep = cfg.heads // cfg.kv_heads
        h = W["embed"][t]
        for li, L in enumerate(W["layers"]):
            x = rmsnorm(h, L["in_norm"], cfg.rms_eps)
            q = rope(linear(x, L["q"]).view(T, cfg.heads, D), pos, cfg.rope_theta)
            k = rope(linear(x, L["k"]).view(T, cfg.kv_heads, D), pos, cfg.rope_theta)
            v = linear(x, L["v"]).view(T, cfg.kv_heads, D)
            self.k[li] = k if self.k[li] is None else torch.cat([self.k[li], k])
            self.v[li] = v if self.v[li] is None else torch.cat([self.v[li], v])
            a = F.scaled_dot_product_attention(q.transpose(0, 1),
                                               self.k[li].transpose(0, 1).repeat_interleave(rep, 0),
                                               self.v[li].transpose(0, 1).repeat_interleave(rep, 0), attn_mask=mask)
            h = h + linear(a.transpose(0, 1).reshape(T, -1), L["o"])
            x = rmsnorm(h, L["post_norm"], cfg.rms_eps)
            h = h + linear(F.silu(linear(x, L["gate"])) * linear(x, L["up"]), L["down"])
        self.n += T
        return (rmsnorm(h[-1:], W["final_norm"], cfg.rms_eps) @ W["lm_head"].t())[0]


@torch.no_grad()
def logits(cfg, W: dict, tokens) -> torch.Tensor:
    """float32 logits [T, vocab] of the whole token sequence."""
    t = torch.as_tensor(tokens, dtype=torch.long)
    T, D = t.numel(), cfg.head_dim
    pos = torch.arange(T)
    h = W["embed"][t]
    for L in W["layers"]:
        x = rmsnorm(h, L["in_norm"], cfg.rms_eps)
        q = rope(linear(x, L["q"]).view(T, cfg.heads, D), pos, cfg.rope_theta)
        k = rope(linear(x, L["k"]).view(T, cfg.kv_heads, D), pos, cfg.rope_theta)
        v = linear(x, L["v"]).view(T, cfg.kv_heads, D)
        rep = cfg.heads // cfg.kv_heads
        a = F.scaled_dot_product_attention(q.transpose(0, 1), k.transpose(0, 1).repeat_interleave(rep, 0),
                                           v.transpose(0, 1).repeat_interleave(rep, 0), is_causal=True)
        h = h + linear(a.transpose(0, 1).reshape(T, -1), L["o"])
        x = rmsnorm(h, L["post_norm"], cfg.rms_eps)
        h = h + linear(F.silu(linear(x, L["gate"])) * linear(x, L["up"]), L["down"])
    return rmsnorm(h, W["final_norm"], cfg.rms_eps) @ W["lm_head"].t()
