"""Benchmark: batch-1 greedy decode tokens/s of a Llama-2-7B-architecture decoder whose
every linear is a NanoQuant layer at the benchmark ranks (~0.55 bpw), after a 2048-token
random-id prompt, tensor-parallel over N GPUs (one process per GPU; the per-block sums run
inside the GEMVs over NVLink, or through NCCL where a shard cannot).  Also reports the fused
decode GEMV against the HBM roofline and the reference's CPU path on this host.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl nq|reference] [--model NAME]

For N > 1 run under torch.distributed.run (one rank per GPU).  Rank 0 prints one JSON line.
"""
from __future__ import annotations

import argparse
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

import torch  # noqa: E402

METRIC = "batch-1 decode tokens/s (7B shape, 0.55 bpw)"

# Under torchrun, native libraries (NCCL prints its version banner on rank 0) may write to
# stdout; main() points file descriptor 1 at stderr and keeps the original stdout here for
# the one JSON line.
_JSON_FD = None


def emit(line: dict) -> None:
    text = json.dumps(line) + "\n"
    if _JSON_FD is None:
        sys.stdout.write(text)
        sys.stdout.flush()
    else:
        os.write(_JSON_FD, text.encode())


def parse():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=256)
    ap.add_argument("--warmup", type=int, default=8)
    ap.add_argument("--impl", default="nq", choices=["nq", "reference"])
    ap.add_argument("--model", default="llama2-7b")
    ap.add_argument("--prompt", type=int, default=2048)
    ap.add_argument("--batch", type=int, default=1)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--cpu-seconds", type=float, default=12.0, help="CPU-baseline sample length")
    ap.add_argument("--layer", default=None,
                    help="per-layer GEMV instead of whole-model decode: out,in,rank (e.g. 11008,4096,2054); "
                         "prints that layer's GB/s over --copies weight copies cycled through the timed loop")
    ap.add_argument("--copies", type=int, default=40, help="--layer: distinct weight copies (past L2)")
    ap.add_argument("--attention", type=int, default=None, metavar="L",
                    help="the fused decode attention (RoPE + cache write + split-KV attention) of --model at "
                         "sequence length L instead of whole-model decode: KV-cache GB/s over 8 caches cycled")
    ap.add_argument("--attention-tp", type=int, default=1,
                    help="--attention: the heads of one tensor-parallel rank of --model (heads / N, kv heads / N)")
    ap.add_argument("--max-seq", type=int, default=None,
                    help="--attention: KV-cache capacity in positions (default L + 64 rounded up to a multiple of 64); "
                         "the kernel's chunking and the cache layout follow it")
    ap.add_argument("--gemm", default=None, metavar="M,OUT,IN,RANK",
                    help="the prefill GEMM of one layer instead of whole-model decode (e.g. 2048,11008,4096,2054): "
                         "TFLOP/s counting the two rank-r contractions, 2*M*r*(in+out), over --copies weight copies")
    ap.add_argument("--fast-gemm", action="store_true",
                    help="--gemm: the reference-rounding mode (T rounded once to bf16) instead of precise")
    ap.add_argument("--gemv-trace", action="store_true",
                    help="phase timeline of every fused GEMV launch of one decode step (rank 0; needs the library "
                         "built with NQ_NVCC_EXTRA=-DNQ_GEMV_TRACE): per launch kind, the median over the step's "
                         "launches of the median and slowest CTA's time at each phase boundary")
    ap.add_argument("--no-exchange", action="store_true",
                    help="N > 1: per-block sums through NCCL instead of inside the GEMVs (the default exchange)")
    ap.add_argument("--peer-allreduce", action="store_true",
                    help="N > 1: sum the blocks' partial outputs through peer memory (nq_allreduce) instead of NCCL")
    return ap.parse_args()


def dist_setup(args):
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != args.gpus:
        raise SystemExit(f"--gpus {args.gpus} but WORLD_SIZE={world}")
    if world > 1:
        import datetime
        torch.cuda.set_device(local)
        torch.distributed.init_process_group("nccl", timeout=datetime.timedelta(seconds=180),
                                             device_id=torch.device("cuda", local))
    elif torch.cuda.is_available():
        torch.cuda.set_device(0)
    return world, rank, local


def peaks():
    p = os.path.join(ROOT, "MEASURED_PEAKS.json")
    if os.path.exists(p):
        d = json.load(open(p))
        return float(d["hbm_gbs"]), "measured"
    return 6650.0, "fallback"


def profile_traffic(alg_bytes_per_launch: float):
    """DRAM bytes per GEMV launch: the committed ncu summary's measured DRAM/algorithmic byte
    ratio (one full capture of a gate/up-shaped launch) applied to this run's average
    algorithmic bytes per launch, since traffic grows in proportion to the planes read."""
    p = os.path.join(ROOT, "profiles", "gemv_llama2_7b_decode.txt")
    if not os.path.exists(p):
        return None
    for line in open(p):
        if line.startswith("dram_per_alg_byte:"):
            return round(float(line.split(":", 1)[1]) * alg_bytes_per_launch, 1)
    return None


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while the timed region runs."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu: int):
        self.gpu, self.lines, self.proc = gpu, [], None
        self.first = threading.Event()

    def __enter__(self):
        """Start nvidia-smi and wait (up to 5 s) for its first sample, so that samples cover the
        timed region even when it lasts well under a second (nvidia-smi takes a while to start,
        longer when several ranks start one each)."""
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "100", "-i", str(self.gpu)], stdout=subprocess.PIPE,
                                         stderr=subprocess.DEVNULL, text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            self.first.wait(timeout=5.0)
        except OSError:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())
            self.first.set()

    def __exit__(self, *exc):
        if self.proc is not None:
            n0, t0 = len(self.lines), time.time()
            while len(self.lines) <= n0 and time.time() - t0 < 1.0:  # one sample at the end of the region
                time.sleep(0.02)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            f = [x.strip() for x in ln.split(",")]
            if len(f) < 9:
                continue
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except ValueError:
                continue
            for n, v in zip(names, f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(n)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


# --------------------------------------------------------------------------------------
# CPU baseline: the reference's CPU path (dense +-1 factors, _compute_forward) on this host
# --------------------------------------------------------------------------------------
def cpu_reference_token_time(cfg, context: int, seconds: float):
    """Seconds per decode token of the reference CPU path, from a bounded sample: one decoder
    layer (7 dense-factor NanoQuant linears in float32 via oracle.dense_forward_torch, the
    reference's _compute_forward, plus attention over `context` cached positions and the
    norms) timed repeatedly for ~`seconds`, scaled by the layer count, plus the fp32 lm_head."""
    from oracle import oracle as orc
    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    g = torch.Generator().manual_seed(0)
    sign = lambda r, c: (torch.randint(0, 2, (r, c), generator=g, dtype=torch.int8) * 2 - 1).float()  # noqa: E731
    lin = {}
    for p in ("q", "k", "v", "o", "gate", "up", "down"):
        out_f, in_f = cfg.io(p)
        r = cfg.ranks[p]
        lin[p] = (sign(r, in_f), sign(out_f, r), torch.rand(in_f, generator=g), torch.rand(out_f, generator=g))
    kc = torch.randn(cfg.kv_heads, context, cfg.head_dim, generator=g)
    vc = torch.randn(cfg.kv_heads, context, cfg.head_dim, generator=g)
    lm = torch.randn(cfg.vocab, cfg.hidden, generator=g) * 0.02
    x0 = torch.randn(1, cfg.hidden, generator=g)
    rep = cfg.heads // cfg.kv_heads

    def layer(x):
        def f(p, v):
            V, U, s2, s1 = lin[p]
            return orc.dense_forward_torch(v, s2, V, None, U, s1)
        h = torch.nn.functional.rms_norm(x, (cfg.hidden,))
        q = f("q", h).view(cfg.heads, 1, cfg.head_dim)
        f("k", h), f("v", h)
        a = torch.nn.functional.scaled_dot_product_attention(q, kc.repeat_interleave(rep, 0),
                                                             vc.repeat_interleave(rep, 0))
        x = x + f("o", a.reshape(1, -1))
        h = torch.nn.functional.rms_norm(x, (cfg.hidden,))
        return x + f("down", torch.nn.functional.silu(f("gate", h)) * f("up", h))

    with torch.no_grad():
        layer(x0)
        n, t0 = 0, time.perf_counter()
        while True:
            layer(x0)
            n += 1
            if time.perf_counter() - t0 >= seconds:
                break
        t_layer = (time.perf_counter() - t0) / n
        t1 = time.perf_counter()
        for _ in range(3):
            torch.nn.functional.rms_norm(x0, (cfg.hidden,)) @ lm.t()
        t_head = (time.perf_counter() - t1) / 3
    return cfg.layers * t_layer + t_head, threads, n


def config_block(cfg, args, world, dec=None):
    """The line's config; with the decoder, the tensor-parallel sum it actually runs (the fused
    exchange falls back to NCCL where a shard's exchanging GEMV launch cannot run one CTA per SM)."""
    exchange = not getattr(args, "no_exchange", False) if dec is None else dec.tpx is not None
    return {"workload": f"{cfg.name} 0.55bpw batch-{args.batch} greedy decode after a {args.prompt}-token "
                        f"random-id prompt",
            "model": cfg.name, "global_batch": args.batch, "seq_len": args.prompt,
            "parallelism": f"tp{world}", "ranks": dict(cfg.ranks),
            "decode_path": "grouped GEMV launches with fused RMSNorm / SwiGLU prologues",
            "tp_allreduce": ("peer memory (nq_allreduce)" if getattr(args, "peer_allreduce", False) else
                             "NCCL" if not exchange else
                             "inside the GEMVs (push from o / down, pull in the next RMSNorm prologue)")
                            if world > 1 else None,
            "l2": "working set > L2 (weights + KV cache read per token)"}


def _configs_module():
    """nanoquant_b200/configs.py loaded by path: importing it through the package would run the
    package __init__, which maps this repository's native libraries into the process."""
    import importlib.util
    name = "nq_b200_configs"
    if name in sys.modules:
        return sys.modules[name]
    spec = importlib.util.spec_from_file_location(name, os.path.join(ROOT, "nanoquant_b200", "configs.py"))
    mod = importlib.util.module_from_spec(spec)
    sys.modules[name] = mod  # dataclasses resolve their module through sys.modules
    spec.loader.exec_module(mod)
    return mod


def repo_libraries_mapped():
    """The product's native libraries (nanoquant_b200/*.so) mapped into this process."""
    pkg = os.path.join(ROOT, "nanoquant_b200") + os.sep
    try:
        with open("/proc/self/maps") as f:
            paths = {line.split()[-1] for line in f if ".so" in line}
    except OSError:
        return []
    return sorted(p for p in paths if p.startswith(pkg))


def run_reference(args, world, rank):
    cfg = _configs_module().CONFIGS[args.model]
    if rank != 0:
        return
    sample = max(1.0, args.cpu_seconds / max(1, args.steps + args.warmup))
    times = []
    for i in range(args.warmup + args.steps):
        t, cores, n = cpu_reference_token_time(cfg, args.prompt + i, sample)
        if i >= args.warmup:
            times.append(t)
    sec = sum(times) / len(times)
    val = args.batch / sec
    line = {"impl": "reference", "metric": METRIC, "value": round(val, 4), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(sec * 1e3, 3),
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "f32",
            "data": "synthetic (seeded random +-1 factors and token ids)", "config": config_block(cfg, args, world),
            "cpu_baseline": {"value": round(val, 4), "unit": "tokens/s", "cores": cores, "kind": "port",
                             "sample": f"per step: one decoder layer (7 dense-factor linears, attention, norms) "
                                       f"timed ~{sample:.1f}s, x{cfg.layers} layers + lm_head"},
            "e2e": {"value": round(val, 4), "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    mapped = repo_libraries_mapped()
    if mapped:  # the reference arm must run without this repository's kernels
        raise SystemExit(f"reference arm mapped repository libraries: {mapped}")
    emit(line)


def gemv_roofline(dec, reps: int = 5):
    """Average duration of a fused GEMV launch over one token's worth of launches exactly as
    the decode step issues them (for every layer of this rank: q/k/v with RMSNorm(x + residual)
    in the prologue, o, gate/up with RMSNorm and SiLU on the gate, down with gate * up in the
    prologue; replayed from a CUDA graph), and the algorithmic bytes per launch: sign planes,
    scales, the input vectors the launch reads and the vectors it writes."""
    from nanoquant_b200 import chain as nqchain
    units = []  # (callable, algorithmic bytes)
    B, ops, eps = dec.batch, torch.ops.nq_b200, dec.cfg.rms_eps
    fused = dec.fuse_neighbours and B <= 8
    for lay in dec.layers:
        for key in ("qkv", "o", "gate_up", "down"):
            unit = lay[key]
            members = unit.members if hasattr(unit, "members") else (unit,)
            n_in = members[0].in_features
            x = torch.randn(B, n_in, device=dec.device, dtype=dec.dtype)
            alg = sum(m.nbytes() + 2 * B * m.out_features for m in members) + 2 * B * n_in
            if fused and key in ("qkv", "gate_up"):
                x2, res = torch.randn_like(x), torch.empty_like(x)
                nw = lay["in_norm" if key == "qkv" else "post_norm"]
                act = 1 if key == "gate_up" else 0
                alg += 2 * B * n_in * 2 + 2 * n_in  # residual read, sum written, norm weight
                fn = (lambda u, xx, r, w, o, a: (lambda: ops.gemv_group_ex(xx, r, w, eps, nqchain.RMSNORM, o, a, u.s2, u.vb,
                                                                            u.smid, u.ub, u.s1)))(unit, x, x2, nw, res, act)
            elif fused and key == "down" and dec.fuse_down:
                x2 = torch.randn_like(x)
                alg += 2 * B * n_in  # the second factor (up)
                fn = (lambda u, xx, yy: (lambda: ops.gemv_group_ex(xx, yy, None, 0.0, nqchain.MUL, None, 0, [u.s2], [u.vb],
                                                                    [u.smid], [u.ub], [u.s1])))(unit, x, x2)
            elif hasattr(unit, "members"):
                fn = (lambda u, xx: (lambda: ops.gemv_group(xx, u.s2, u.vb, u.smid, u.ub, u.s1)))(unit, x)
            else:
                fn = (lambda u, xx: (lambda: u.gemv(xx)))(unit, x)
            units.append((fn, alg))
    s = torch.cuda.Stream(device=dec.device)
    s.wait_stream(torch.cuda.current_stream(dec.device))
    with torch.cuda.stream(s):
        for fn, _ in units:
            fn()
    torch.cuda.current_stream(dec.device).wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g, stream=s):
        for fn, _ in units:
            fn()
    for _ in range(2):
        g.replay()
    torch.cuda.synchronize(dec.device)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    cur = torch.cuda.current_stream(dec.device)
    e0.record(cur)
    for _ in range(reps):
        g.replay()
    e1.record(cur)
    torch.cuda.synchronize(dec.device)
    us_per_launch = e0.elapsed_time(e1) * 1e3 / (reps * len(units))
    alg = sum(a for _, a in units) / len(units)
    del g
    return alg, us_per_launch, len(units)


def run_nq(args, world, rank, local):
    from nanoquant_b200.decoder import CONFIGS, Decoder
    cfg = CONFIGS[args.model]
    dev = torch.device("cuda", local)
    group = torch.distributed.group.WORLD if world > 1 else None
    max_seq = args.prompt + args.warmup + 2 * args.steps + 16
    dec = Decoder(cfg, max_seq=max_seq, batch=args.batch, tp_rank=rank, tp=world, group=group, seed=1234,
                  dtype=torch.float16, device=dev, peer_allreduce=args.peer_allreduce,
                  tp_exchange=not args.no_exchange)
    g = torch.Generator().manual_seed(42)
    prompt = torch.randint(0, cfg.vocab, (args.batch, args.prompt), generator=g)  # one random-id prompt per row
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    first = dec.prefill(prompt.to(dev))
    e1.record()
    torch.cuda.synchronize(dev)
    prefill_ms = e0.elapsed_time(e1)
    # a second, warm prefill of the same prompt (first-call costs -- library loading, cuDNN and
    # cuBLAS heuristics, kernel attribute setup -- are paid by the first one)
    e0.record()
    dec.prefill(prompt.to(dev))
    e1.record()
    torch.cuda.synchronize(dev)
    prefill_warm_ms = e0.elapsed_time(e1)
    graphed = dec.capture(warmup=2)
    cur = torch.cuda.current_stream(dev)

    def barrier():
        if world > 1:
            torch.distributed.barrier(device_ids=[local])

    def max_over_ranks(v):
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        torch.distributed.all_reduce(t, op=torch.distributed.ReduceOp.MAX)
        return float(t.item())

    # ---------------- device-timed decode (inputs resident in HBM)
    for _ in range(args.warmup):
        graphed.replay()
    barrier()
    torch.cuda.synchronize(dev)
    with ClockSampler(local) as clocks:
        e0.record(cur)
        for _ in range(args.steps):
            graphed.replay()
        e1.record(cur)
        torch.cuda.synchronize(dev)
    barrier()
    ms = max_over_ranks(e0.elapsed_time(e1))
    ms_per_step = ms / args.steps
    value = args.batch * args.steps / (ms / 1e3)

    # ---------------- end to end through the public step API (host token ids in and out)
    host_in = torch.empty(args.batch, dtype=torch.long).pin_memory()
    host_out = torch.empty(args.batch, dtype=torch.long).pin_memory()
    host_in.copy_(dec.next_tokens.cpu())
    barrier()
    torch.cuda.synchronize(dev)
    e0.record(cur)
    for _ in range(args.steps):
        graphed.generate(host_in, host_out)
        host_in.copy_(host_out)
    e1.record(cur)
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = max_over_ranks(e0.elapsed_time(e1))
    e2e = args.batch * args.steps / (e2e_ms / 1e3)
    graphed.release()

    # ---------------- dominant kernel vs the HBM roofline
    alg_bytes, us_launch, n_lin = gemv_roofline(dec)
    peak, peak_kind = peaks()
    achieved = alg_bytes / (us_launch * 1e-6) / 1e9
    launches_per_step = dec.own_launches_per_step()

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        t, cores, n = cpu_reference_token_time(cfg, args.prompt, args.cpu_seconds)
        cpu = {"value": round(args.batch / t, 4), "unit": "tokens/s", "cores": cores, "kind": "port",
               "sample": f"one decoder layer (reference _compute_forward on dense +-1 fp32 factors x7, attention "
                         f"over {args.prompt} positions, norms) repeated {n}x in ~{args.cpu_seconds:.0f}s, "
                         f"scaled x{cfg.layers} layers + fp32 lm_head"}

    if world > 1:
        torch.distributed.barrier(device_ids=[local])
    if rank == 0:
        line = {"metric": METRIC, "value": round(value, 3), "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": round(ms_per_step, 4), "higher_is_better": True,
                "scaling": "strong", "vs_baseline": None, "dtype": "f16",
                "data": "synthetic (seeded random +-1 factors, fp16 scales, random token ids)",
                "config": config_block(cfg, args, world, dec),
                "e2e": {"value": round(e2e, 3), "unit": "tokens/s", "h2d_bytes_per_step": 8 * args.batch,
                        "d2h_bytes_per_step": 8 * args.batch},
                "roofline": {"bound": "hbm", "kernel": "gemv_kernel (fused decode GEMV)",
                             "achieved": round(achieved, 2), "peak": peak, "unit": "GB/s",
                             "frac": round(achieved / peak, 5), "peak_source": peak_kind,
                             "traffic": profile_traffic(alg_bytes), "bytes_per_launch": round(alg_bytes, 1),
                             "us_per_launch": round(us_launch, 3), "launches_measured": n_lin},
                "cpu_baseline": cpu,
                "clocks": clocks.summary(),
                "gpu_launches": launches_per_step * args.steps,
                "prefill_ms": round(prefill_ms, 2), "prefill_warm_ms": round(prefill_warm_ms, 2),
                "first_token": int(first[0])}
        emit(line)
    if world > 1:
        torch.distributed.barrier(device_ids=[local])
        torch.distributed.destroy_process_group()


GEMV_PHASES = ["start", "copies issued", "pdl wait", "x landed", "x transformed", "x folded", "stage-1 MMA",
               "stage-1 reduce", "grid barrier", "U landed", "stage-2 MMA", "end"]


def run_gemv_trace(args, world, rank, local):
    """One decode step's fused GEMV launches, phase by phase, from the debug build's globaltimer
    stamps (nq_debug_gemv_trace).  Prints a table of microseconds from each launch's first CTA."""
    import ctypes
    import numpy as np
    from nanoquant_b200 import _lib
    from nanoquant_b200.decoder import CONFIGS, Decoder
    lib = _lib.cuda_lib()
    if not hasattr(lib, "nq_debug_gemv_trace"):
        raise SystemExit("--gemv-trace needs the library built with NQ_NVCC_EXTRA=-DNQ_GEMV_TRACE")
    fn = lib.nq_debug_gemv_trace
    fn.restype = ctypes.c_int
    fn.argtypes = [ctypes.c_void_p, ctypes.c_int, ctypes.c_int]
    cfg = CONFIGS[args.model]
    dev = torch.device("cuda", local)
    group = torch.distributed.group.WORLD if world > 1 else None
    dec = Decoder(cfg, max_seq=args.prompt + 64, batch=args.batch, tp_rank=rank, tp=world, group=group, seed=1234,
                  dtype=torch.float16, device=dev, tp_exchange=not args.no_exchange)
    prompt = torch.randint(0, cfg.vocab, (args.batch, args.prompt), generator=torch.Generator().manual_seed(42))
    dec.prefill(prompt.to(dev))
    g = dec.capture(warmup=2)
    for _ in range(3):
        g.replay()
    torch.cuda.synchronize(dev)
    buf = np.zeros((512, 160, 12), dtype=np.uint64)
    fn(buf.ctypes.data, 512, 1)
    if world > 1:
        torch.distributed.barrier(device_ids=[local])
    g.replay()
    torch.cuda.synchronize(dev)
    n = fn(buf.ctypes.data, 512, 1)
    if world > 1:
        torch.distributed.barrier(device_ids=[local])
    g.release()
    if rank != 0:
        return
    G = torch.cuda.get_device_properties(dev).multi_processor_count
    kinds = ["q/k/v", "o", "gate/up", "down"]
    lines = [f"{cfg.name} tp{world} batch {args.batch}: {n} fused GEMV launches in one decode step; microseconds "
             f"from the launch's first CTA start, median CTA / slowest CTA (median over the step's launches)",
             "| phase | " + " | ".join(kinds) + " |", "|---" * (len(kinds) + 1) + "|"]
    per = {k: [] for k in kinds}
    for li in range(n):
        st = buf[li, :G, :].astype(np.int64)
        active = st[:, 11] > 0
        rel = (st[active] - st[active, 0].min()) / 1000.0
        rel[rel < 0] = np.nan  # a phase this CTA skips (no stage-1 tiles) has no stamp
        per[kinds[li % 4]].append(rel)
    cols = {}
    for k in kinds:
        arr = per[k]
        med = np.median(np.stack([np.nanmedian(a, axis=0) for a in arr]), axis=0)
        mx = np.median(np.stack([np.nanmax(a, axis=0) for a in arr]), axis=0)
        cols[k] = (med, mx)
    for i, ph in enumerate(GEMV_PHASES):
        lines.append(f"| {ph} | " + " | ".join(f"{cols[k][0][i]:.2f} / {cols[k][1][i]:.2f}" for k in kinds) + " |")
    starts = [buf[li, :G, 0].astype(np.int64).min() for li in range(n)]
    ends = [buf[li, :G, 11].astype(np.int64).max() for li in range(n)]
    gaps = [(starts[i + 1] - ends[i]) / 1000 for i in range(n - 1)]
    for j, k in enumerate(kinds):
        sel = [gaps[i] for i in range(len(gaps)) if i % 4 == j]
        lines.append(f"gap from the end of a {k} launch to the next GEMV launch: median {np.median(sel):.2f} us")
    lines.append(f"first GEMV start to last GEMV end: {(ends[-1] - starts[0]) / 1000:.1f} us")
    print("\n".join(lines), flush=True)


def run_layer(args):
    """One NanoQuant layer's fused decode GEMV (the per-layer measurement): --copies distinct
    seeded weight sets, more bytes than L2 holds, cycled so every launch reads its weights
    from HBM; algorithmic bytes per launch / device time per launch."""
    from nanoquant_b200.decoder import QuantLinearShard, _random_planes
    out_f, in_f, r = (int(v) for v in args.layer.split(","))
    dev = torch.device("cuda", 0)
    layers = []
    for c in range(args.copies):
        gen = torch.Generator(device=dev)
        gen.manual_seed(1000 + c)
        vb, ub = _random_planes(gen, r, in_f, dev), _random_planes(gen, out_f, r, dev)
        s2 = (torch.rand(in_f, generator=gen, device=dev) + 0.5).half()
        s1 = (torch.rand(out_f, generator=gen, device=dev) * 0.02).half()
        layers.append(QuantLinearShard(vb, ub, s2, None, s1))
    x = torch.randn(args.batch, in_f, device=dev).half()
    alg = layers[0].nbytes() + 2 * args.batch * (in_f + out_f)
    for i in range(max(args.warmup, 3)):
        layers[i % args.copies].gemv(x)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = args.steps * args.copies
    e0.record()
    for i in range(n):
        layers[i % args.copies].gemv(x)
    e1.record()
    torch.cuda.synchronize(dev)
    us = e0.elapsed_time(e1) * 1e3 / n
    peak, kind = peaks()
    gbs = alg / (us * 1e-6) / 1e9
    print(json.dumps({"metric": "decode GEMV GB/s (algorithmic bytes)", "value": round(gbs, 2), "unit": "GB/s",
                      "layer": {"out": out_f, "in": in_f, "rank": r, "batch": args.batch}, "us_per_launch": round(us, 3),
                      "bytes_per_launch": alg, "copies": args.copies, "launches": n,
                      "roofline": {"bound": "hbm", "peak": peak, "frac": round(gbs / peak, 5), "peak_source": kind},
                      "dtype": "f16", "data": "synthetic"}), flush=True)


def run_gemm(args):
    """One NanoQuant layer's prefill GEMM (tcgen05): --copies distinct seeded weight sets cycled,
    bf16 activations N(0,1) [M, in], bf16 output; TFLOP/s counts the algorithmic flops of the two
    rank-r contractions, 2*M*r*(in+out), per device time per launch (CUDA events)."""
    from nanoquant_b200.decoder import QuantLinearShard, _random_planes
    m, out_f, in_f, r = (int(v) for v in args.gemm.split(","))
    dev = torch.device("cuda", 0)
    copies = max(2, min(args.copies, 8))
    layers = []
    for c in range(copies):
        gen = torch.Generator(device=dev)
        gen.manual_seed(2000 + c)
        vb, ub = _random_planes(gen, r, in_f, dev), _random_planes(gen, out_f, r, dev)
        s2 = (torch.rand(in_f, generator=gen, device=dev) + 0.5).bfloat16()
        s1 = (torch.rand(out_f, generator=gen, device=dev) * 0.02).bfloat16()
        layers.append(QuantLinearShard(vb, ub, s2, None, s1))
    x = torch.randn(m, in_f, device=dev).bfloat16()
    precise = not args.fast_gemm
    ops = torch.ops.nq_b200

    def call(i):
        q = layers[i % copies]
        return ops.gemm(x, q.s2, q.vb, q.smid, q.ub, q.s1, precise)

    for i in range(max(args.warmup, 3)):
        call(i)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = max(args.steps, 1) * copies
    with ClockSampler(0) as clocks:
        e0.record()
        for i in range(n):
            call(i)
        e1.record()
        torch.cuda.synchronize(dev)
    us = e0.elapsed_time(e1) * 1e3 / n
    flops = 2.0 * m * r * (in_f + out_f)
    tflops = flops / (us * 1e-6) / 1e12
    pk = _peak_tflops()
    print(json.dumps({"metric": "prefill GEMM TFLOP/s (two rank-r contractions)", "value": round(tflops, 2),
                      "unit": "TFLOP/s", "layer": {"m": m, "out": out_f, "in": in_f, "rank": r,
                                                   "mode": "precise" if precise else "fast"},
                      "us_per_launch": round(us, 3), "flops_per_launch": flops, "copies": copies, "launches": n,
                      "roofline": {"bound": "tensor", "peak": pk[0], "frac": round(tflops / pk[0], 5),
                                   "peak_source": pk[1], "unit": "TFLOP/s"},
                      "clocks": clocks.summary(), "dtype": "bf16", "data": "synthetic"}), flush=True)


def _ref_ops(what: str):
    """The reference's own CUDA kernels (oracle/_ref, built from its sources), or None after
    printing the reference arm's `unavailable` line."""
    from oracle import ref_kernels as rk
    if not rk.available():
        emit({"impl": "reference", "unavailable": f"{what}: the reference kernels are not built "
                                                  "(python oracle/build_ref.py needs the reference sources)"})
        return None, rk
    return rk.load(), rk


def run_reference_layer(args):
    """--impl reference --layer OUT,IN,RANK: the reference's own decode GEMV
    (binary_kernels::nanoquant_dyn_forward, gemv_kernel.cu:308-429, with the reference module's
    launch configuration) on this GPU, timed exactly like run_layer: --copies distinct random
    weight sets cycled past L2, CUDA events, algorithmic bytes per launch."""
    out_f, in_f, r = (int(v) for v in args.layer.split(","))
    if not torch.cuda.is_available():
        emit({"impl": "reference", "unavailable": "--layer times the reference's CUDA GEMV and needs a GPU"})
        return
    ops, rk = _ref_ops("--layer")
    if ops is None:
        return
    if not rk.gemv_shape_ok(out_f, in_f, r):
        emit({"impl": "reference", "unavailable": f"the reference GEMV reads and writes out of bounds at rank {r} / "
                                                  f"in {in_f} / out {out_f} (needs multiples of 32 and 8)"})
        return
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev)
    gen.manual_seed(1000)
    # uniformly random words are uniformly random +-1 planes (no padding bits at these shapes)
    words = lambda rows, cols: torch.randint(-2**31, 2**31 - 1, (rows, cols // 32), generator=gen,  # noqa: E731
                                             device=dev, dtype=torch.int32)
    layers = [(words(r, in_f), words(out_f, r), (torch.rand(in_f, generator=gen, device=dev) + 0.5).half(),
               (torch.rand(out_f, generator=gen, device=dev) * 0.02).half()) for _ in range(args.copies)]
    x = torch.randn(args.batch, in_f, device=dev).half()
    alg = 4 * r * (in_f // 32) + 4 * out_f * (r // 32) + 2 * (in_f + out_f) + 2 * args.batch * (in_f + out_f)

    def call(i):
        vb, ub, s2, s1 = layers[i % args.copies]
        return rk.gemv(ops, x, s2, vb, None, ub, s1)

    for i in range(max(args.warmup, 3)):
        call(i)
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    n = args.steps * args.copies
    with ClockSampler(0) as clocks:
        e0.record()
        for i in range(n):
            call(i)
        e1.record()
        torch.cuda.synchronize(dev)
    us = e0.elapsed_time(e1) * 1e3 / n
    peak, kind = peaks()
    gbs = alg / (us * 1e-6) / 1e9
    emit({"impl": "reference", "metric": "decode GEMV GB/s (algorithmic bytes)", "value": round(gbs, 2),
          "unit": "GB/s", "kernel": "reference nanoquant_dyn_forward (two launches, fp16 accumulation)",
          "layer": {"out": out_f, "in": in_f, "rank": r, "batch": args.batch}, "us_per_launch": round(us, 3),
          "bytes_per_launch": alg, "copies": args.copies, "launches": n,
          "roofline": {"bound": "hbm", "peak": peak, "frac": round(gbs / peak, 5), "peak_source": kind},
          "clocks": clocks.summary(), "dtype": "f16", "data": "synthetic"})


def run_reference_gemm(args):
    """--impl reference --gemm: the reference's own prefill GEMM (marlin_nanoquant_forward,
    gemm.cpp:112-122) is not run on this GPU.  Built for sm_100a from its sources it stopped with
    "an illegal instruction was encountered" on a B200, on shapes its host checks accept
    (M = 128 / 2048 at 4096x4096 r1088 and 4096x11008 r1600, bf16), so this arm reports it as
    unavailable instead of running it again."""
    emit({"impl": "reference", "unavailable": "the reference Marlin GEMM (marlin_nanoquant_forward) built for "
                                              "sm_100a faults on B200 with an illegal instruction; not run"})


def _peak_tflops():
    """Dense bf16 burst TFLOP/s of MEASURED_PEAKS.json, else the recipe's fallback (1590)."""
    try:
        with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["bf16_tflops"]), "measured"
    except (OSError, KeyError, ValueError):
        return 1590.0, "fallback"


def run_attention(args):
    """The decode attention of one layer of --model (one new token per batch row at position
    L - 1, every head): 8 distinct KV caches (more bytes than L2 holds) cycled so every launch
    reads its cache from HBM; KV bytes read per launch / device time per launch."""
    from nanoquant_b200.decoder import CONFIGS
    _lib_load()
    cfg = CONFIGS[args.model]
    L, B, D = args.attention, args.batch, cfg.head_dim
    tp = max(1, args.attention_tp)
    hq, hkv = cfg.heads // tp, cfg.kv_heads // tp
    dev = torch.device("cuda", 0)
    max_seq = args.max_seq if args.max_seq else (L + 64 + 63) // 64 * 64
    caches = [(torch.randn(B, hkv, max_seq, D, device=dev).half(),
               torch.randn(B, hkv, max_seq, D, device=dev).half()) for _ in range(8)]
    q = torch.randn(B, hq, D, device=dev).half()
    k = torch.randn(B, hkv, D, device=dev).half()
    v = torch.randn(B, hkv, D, device=dev).half()
    pos = torch.full((B,), L - 1, dtype=torch.int32, device=dev)
    ops = torch.ops.nq_b200
    for i in range(max(args.warmup, 3)):
        kc, vc = caches[i % 8]
        ops.decode_attention_rope(q, k, v, pos, kc, vc, cfg.rope_theta)
    torch.cuda.synchronize(dev)
    n = args.steps * 8
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record()
    for i in range(n):
        kc, vc = caches[i % 8]
        ops.decode_attention_rope(q, k, v, pos, kc, vc, cfg.rope_theta)
    e1.record()
    torch.cuda.synchronize(dev)
    us = e0.elapsed_time(e1) * 1e3 / n
    kv = 2 * B * hkv * L * D * 2
    peak, kind = peaks()
    gbs = kv / (us * 1e-6) / 1e9
    print(json.dumps({"metric": "decode attention GB/s (KV-cache bytes)", "value": round(gbs, 2), "unit": "GB/s",
                      "attention": {"model": cfg.name, "seq_len": L, "max_seq": max_seq, "batch": B,
                                    "heads": hq, "kv_heads": hkv, "tp": tp}, "us_per_launch": round(us, 3), "bytes_per_launch": kv,
                      "launches": n, "roofline": {"bound": "hbm", "peak": peak, "frac": round(gbs / peak, 5),
                                                  "peak_source": kind},
                      "dtype": "f16", "data": "synthetic"}), flush=True)


def _lib_load():
    from nanoquant_b200 import _lib
    _lib.load_torch_ops()


def main():
    global _JSON_FD
    args = parse()
    if args.impl == "reference" and (args.layer or args.gemm):
        if int(os.environ.get("RANK", "0")) == 0:
            run_reference_layer(args) if args.layer else run_reference_gemm(args)
        return
    if args.layer:
        run_layer(args)
        return
    if args.attention:
        run_attention(args)
        return
    if args.gemm:
        _lib_load()
        run_gemm(args)
        return
    if int(os.environ.get("WORLD_SIZE", "1")) > 1:
        sys.stdout.flush()
        _JSON_FD = os.dup(1)
        os.dup2(2, 1)
    world, rank, local = dist_setup(args)
    if args.gemv_trace:
        _lib_load()
        run_gemv_trace(args, world, rank, local)
        if world > 1 and torch.distributed.is_initialized():
            torch.distributed.destroy_process_group()
        return
    if args.impl == "reference":
        run_reference(args, world, rank)
    else:
        run_nq(args, world, rank, local)
    if world > 1 and torch.distributed.is_initialized():
        torch.distributed.destroy_process_group()


if __name__ == "__main__":
    main()
