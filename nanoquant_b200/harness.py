"""Decode benchmark harness with the reference's metric and CSV rows.

The reference measures decode in src/nanoquant/kernel/test_decode.py: ``generate`` (:474-690) runs
the prompt, then a decode loop for tokens 2..N, and reports ``tps_total = batch * (N - 1) / wall``
(the loop's wall-clock time, :685); the sweep writes one CSV row per measured iteration with
``decode_tps_total``, ``decode_tokens_total``, ``decode_time_s``, ... (:971-1003) and an
aggregate row per configuration (:781-803).  This module reproduces that measurement on this
package's decoder: greedy decoding through the CUDA-graph step, token ids fed back from the host
every step like the reference's loop, prompts of random token ids (no tokenizer or dataset),
random weights or a packed checkpoint (nanoquant_b200.loader).

    python -m nanoquant_b200.harness --model llama2-7b --batch_size 1 --prompt_tokens 128 \
        --max_new_tokens 32,128,256 --iters 2 --output_csv decode.csv
"""
from __future__ import annotations

import argparse
import csv
import time
from typing import Dict, List, Optional

import torch

# the reference's per-iteration row fields that this harness fills (test_decode.py:971-1003); the
# energy fields (Zeus) are left blank as the reference leaves them without a monitor
ROW_FIELDS = ["iter", "model_name", "qmodel_ckpt", "batch_size", "prompt_tokens_target", "seqlen_prompt",
              "max_new_tokens", "decode_tokens_per_seq", "decode_tokens_total", "decode_time_s", "decode_tps_total",
              "decode_tps_per_seq", "top_k", "temperature", "dtype", "compiled", "use_quant_kernels",
              "quant_kernel_type", "prefill_time_s_zeus", "prefill_energy_j", "prefill_energy_per_prompt_token_j",
              "decode_time_s_zeus", "decode_energy_j", "decode_energy_per_token_j", "gpu_mem_peak_alloc_bytes",
              "gpu_mem_peak_reserved_bytes", "gpu_mem_peak_alloc_increase_bytes",
              "gpu_mem_peak_reserved_increase_bytes"]


@torch.no_grad()
def generate(dec, prompt_ids: torch.Tensor, max_new_tokens: int, graphed=None):
    """Greedy generation of ``max_new_tokens`` tokens after ``prompt_ids`` [batch, T] (test_decode.py
    generate, :474-690, greedy): token 1 from the prefill, tokens 2..N from the CUDA-graph step with
    the token ids copied host -> device -> host every step.  Returns (ids [batch, T + N],
    tps_total = batch * (N - 1) / decode wall-clock seconds, profile dict)."""
    dev = dec.device
    if prompt_ids.dim() == 1:
        prompt_ids = prompt_ids[None]
    B, T = prompt_ids.shape
    prof: Dict[str, float] = {}
    torch.cuda.synchronize(dev)
    alloc0, res0 = torch.cuda.memory_allocated(dev), torch.cuda.memory_reserved(dev)
    torch.cuda.reset_peak_memory_stats(dev)
    t0 = time.perf_counter()
    first = dec.prefill(prompt_ids.to(dev))
    torch.cuda.synchronize(dev)
    prof["prefill_time_s"] = time.perf_counter() - t0
    g = graphed if graphed is not None else dec.capture(warmup=1)
    host_in = first.cpu().pin_memory()
    host_out = torch.empty(B, dtype=torch.long).pin_memory()
    out = [first.cpu()]
    torch.cuda.synchronize(dev)
    t1 = time.perf_counter()
    for _ in range(max(max_new_tokens - 1, 0)):
        g.generate(host_in, host_out)
        out.append(host_out.clone())
        host_in.copy_(host_out)
    torch.cuda.synchronize(dev)
    wall = time.perf_counter() - t1
    tokens_in_loop = max(max_new_tokens - 1, 0)
    tps_total = float(B * tokens_in_loop) / max(wall, 1e-9)
    prof.update({"decode_time_s": wall, "decode_tokens_total": B * tokens_in_loop,
                 "gpu_mem_peak_alloc_bytes": torch.cuda.max_memory_allocated(dev),
                 "gpu_mem_peak_reserved_bytes": torch.cuda.max_memory_reserved(dev)})
    prof["gpu_mem_peak_alloc_increase_bytes"] = max(0, prof["gpu_mem_peak_alloc_bytes"] - alloc0)
    prof["gpu_mem_peak_reserved_increase_bytes"] = max(0, prof["gpu_mem_peak_reserved_bytes"] - res0)
    if graphed is None:
        g.release()
    ids = torch.cat([prompt_ids.cpu(), torch.stack(out, dim=1)], dim=1)
    return ids, tps_total, prof


def make_row(it: int, model_name: str, ckpt: str, bs: int, pt: int, new: int, tps_total: float, prof: dict,
             dtype: str) -> Dict[str, object]:
    """One measured iteration as the reference writes it (test_decode.py:966-1003)."""
    tokens_in_loop = max(int(new) - 1, 0)
    total = int(bs * tokens_in_loop)
    decode_time_s = float(total) / max(float(tps_total), 1e-12) if total > 0 else 0.0
    row = {k: "" for k in ROW_FIELDS}
    row.update({"iter": it, "model_name": model_name, "qmodel_ckpt": ckpt, "batch_size": bs,
                "prompt_tokens_target": pt, "seqlen_prompt": pt, "max_new_tokens": new,
                "decode_tokens_per_seq": tokens_in_loop, "decode_tokens_total": total,
                "decode_time_s": f"{decode_time_s:.6f}",
                "decode_tps_total": f"{float(tps_total):.6f}" if total > 0 else "",
                "decode_tps_per_seq": f"{(float(tps_total) / bs):.6f}" if total > 0 else "",
                "top_k": 1, "temperature": 0.0, "dtype": dtype, "compiled": 1, "use_quant_kernels": 1,
                "quant_kernel_type": "b200"})
    for k in ("gpu_mem_peak_alloc_bytes", "gpu_mem_peak_reserved_bytes", "gpu_mem_peak_alloc_increase_bytes",
              "gpu_mem_peak_reserved_increase_bytes"):
        if k in prof:
            row[k] = f"{int(prof[k])}"
    return row


def aggregate(rows: List[Dict[str, object]]) -> Dict[str, object]:
    """The per-configuration row (test_decode.py:781-803): tokens and time summed,
    decode_tps_total = their ratio, peaks maxed, other numeric fields averaged."""
    agg = dict(rows[0])
    agg["iter"] = "AVG"
    tok = sum(float(r["decode_tokens_total"]) for r in rows)
    sec = sum(float(r["decode_time_s"]) for r in rows)
    if tok > 0 and sec > 0:
        agg["decode_tokens_total"] = f"{tok:.0f}"
        agg["decode_time_s"] = f"{sec:.6f}"
        agg["decode_tps_total"] = f"{tok / sec:.6f}"
        agg["decode_tps_per_seq"] = f"{tok / sec / float(rows[0]['batch_size']):.6f}"
    for k in ("gpu_mem_peak_alloc_bytes", "gpu_mem_peak_reserved_bytes", "gpu_mem_peak_alloc_increase_bytes",
              "gpu_mem_peak_reserved_increase_bytes"):
        vals = [float(r[k]) for r in rows if r.get(k) not in ("", None)]
        if vals:
            agg[k] = f"{max(vals):.0f}"
    return agg


def write_csv(rows: List[Dict[str, object]], path: str) -> None:
    with open(path, "w", newline="") as f:
        w = csv.DictWriter(f, fieldnames=list(rows[0].keys()))
        w.writeheader()
        w.writerows(rows)


def main(argv: Optional[List[str]] = None):
    from .configs import CONFIGS
    from .decoder import Decoder
    ap = argparse.ArgumentParser(description=__doc__.split("\n\n")[0])
    ap.add_argument("--model", default="llama2-7b", help="a configuration name, or an HF config.json with --checkpoint")
    ap.add_argument("--checkpoint", default="", help="packed NanoQuant checkpoint (file or directory)")
    ap.add_argument("--batch_size", default="1")
    ap.add_argument("--prompt_tokens", default="128")
    ap.add_argument("--max_new_tokens", default="32,128,256")
    ap.add_argument("--iters", type=int, default=2)
    ap.add_argument("--warmup_iters", type=int, default=1)
    ap.add_argument("--output_csv", default="decode_b200.csv")
    args = ap.parse_args(argv)
    ints = lambda s: [int(v) for v in str(s).split(",") if v]  # noqa: E731
    dev = torch.device("cuda", torch.cuda.current_device())
    rows = []
    for bs in ints(args.batch_size):
        for pt in ints(args.prompt_tokens):
            max_seq = pt + max(ints(args.max_new_tokens)) + 8
            if args.checkpoint:
                import json

                from .loader import load_compressed_decoder
                with open(args.model) as f:
                    hf = json.load(f)
                dec = load_compressed_decoder(hf, args.checkpoint, max_seq=max_seq, batch=bs, device=dev)
                name = hf.get("_name_or_path", "checkpoint")
            else:
                dec = Decoder(CONFIGS[args.model], max_seq=max_seq, batch=bs, seed=0, device=dev)
                name = args.model
            gen = torch.Generator().manual_seed(0)
            prompt = torch.randint(0, dec.cfg.vocab, (bs, pt), generator=gen)
            for new in ints(args.max_new_tokens):
                cfg_rows = []
                for it in range(args.warmup_iters + args.iters):
                    _, tps, prof = generate(dec, prompt, new)
                    if it >= args.warmup_iters:
                        cfg_rows.append(make_row(it - args.warmup_iters, name, args.checkpoint, bs, pt, new, tps,
                                                 prof, "float16"))
                agg = aggregate(cfg_rows)
                print(f"bs={bs} pt={pt} new={new}: decode_tps_total {agg['decode_tps_total']}", flush=True)
                rows.extend(cfg_rows + [agg])
            del dec
            torch.cuda.empty_cache()
    write_csv(rows, args.output_csv)
    print(f"wrote {args.output_csv}")


if __name__ == "__main__":
    main()
