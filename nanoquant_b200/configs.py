"""Model configurations of the benchmark decoders (plain data: importing this file loads no
native library, so the CPU reference arm of bench.py can read it by path without mapping
this package's kernels).

Ranks: Llama-2-7B at the benchmark's ~0.55 bpw ranks (q/k/v/o 1126, gate/up/down 2054);
Llama-3-70B from the reference rank planner at 0.55 bpw (src/nanoquant/utils/utils.py:273-289).
"""
from __future__ import annotations

from dataclasses import dataclass, field
from typing import Dict

PROJ = ("q", "k", "v", "o", "gate", "up", "down")


@dataclass(frozen=True)
class DecoderConfig:
    name: str
    vocab: int
    hidden: int
    layers: int
    heads: int
    kv_heads: int
    head_dim: int
    ffn: int
    ranks: Dict[str, int] = field(hash=False)
    rms_eps: float = 1e-5
    rope_theta: float = 10000.0

    def io(self, proj: str):
        """(out_features, in_features) of a projection."""
        h, d = self.hidden, self.head_dim
        return {"q": (self.heads * d, h), "k": (self.kv_heads * d, h), "v": (self.kv_heads * d, h),
                "o": (h, self.heads * d), "gate": (self.ffn, h), "up": (self.ffn, h), "down": (h, self.ffn)}[proj]

    def packed_bytes_per_token(self) -> int:
        """Sign-plane + scale bytes of every quantized linear (one decode token, TP=1)."""
        tot = 0
        for p in PROJ:
            out_f, in_f = self.io(p)
            r = self.ranks[p]
            tot += 4 * r * ((in_f + 31) // 32) + 4 * out_f * ((r + 31) // 32) + 2 * (in_f + out_f)
        return tot * self.layers


def uniform_rank(bits: float, out_f: int, in_f: int) -> int:
    """The reference rank planner: floor((bits*a*b/(a+b) - 16) / 32) * 32 (src/nanoquant/utils/utils.py:273-289)."""
    return int(((bits * out_f * in_f / (out_f + in_f)) - 16) // 32 * 32)


LLAMA2_7B = DecoderConfig("llama2-7b", 32000, 4096, 32, 32, 32, 128, 11008,
                          {"q": 1126, "k": 1126, "v": 1126, "o": 1126, "gate": 2054, "up": 2054, "down": 2054})
LLAMA3_70B = DecoderConfig("llama3-70b", 128256, 8192, 80, 64, 8, 128, 28672,
                           {"q": 2208, "k": 480, "v": 480, "o": 2208, "gate": 3488, "up": 3488, "down": 3488},
                           rope_theta=500000.0)
TINY = DecoderConfig("tiny", 512, 256, 2, 2, 1, 128, 512,
                     {"q": 96, "k": 40, "v": 40, "o": 96, "gate": 130, "up": 130, "down": 130})
CONFIGS = {c.name: c for c in (LLAMA2_7B, LLAMA3_70B, TINY)}
