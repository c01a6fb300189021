"""Llama-architecture decoder whose linear layers are NanoQuant layers on the B200 kernels,
tensor-parallel over one process per GPU.

This is the harness the reference benchmarks decode with (src/nanoquant/kernel/test_decode.py:
HF LlamaForCausalLM with every nn.Linear swapped for NanoQuantLinear, StaticCache, greedy
decode with the step captured as a CUDA graph), rebuilt around the kernels of this package:

* every projection is a NanoQuant layer (half2 sign planes + fp16 scales) run by
  ``torch.ops.nq_b200.linear`` (fused GEMV for decode, tcgen05 GEMM for prefill);
* RMSNorm (+ residual add), RoPE + KV-cache write, split-KV decode attention and SwiGLU are
  this package's kernels (decode runs RoPE, the cache write and attention as one launch);
  prefill attention uses PyTorch's fused SDPA (causal, GQA);
* the decode step reads token ids / positions from device buffers and advances them itself,
  so a captured graph replays one autoregressive step with no host work.

Tensor parallelism (one sum over the ranks per attention block and per MLP block):
* q/k/v and gate/up are column-parallel: each rank holds the U rows of its heads / FFN
  columns (U split by output rows) and the full V;
* o and down receive their input sharded by heads / FFN columns, so each rank holds the V
  columns of its shard (V split by input columns) and the full U; by linearity the ranks'
  outputs s1 * U(smid * V_shard (s2 * x_shard)) sum to the full layer;
* in decode the sum runs inside the GEMVs (TPExchange: o / down push their rows to every rank
  over NVLink, the next RMSNorm prologue pulls and sums them) where every exchanging GEMV
  launch runs one CTA per SM, otherwise through torch.distributed (NCCL), as in prefill.
Weights are random (seeded) with the per-layer ranks of the benchmark configs; every rank
draws the same global planes and keeps its slice, so any TP degree computes the same model.
"""
from __future__ import annotations

import math
from typing import Optional

import torch
import torch.nn.functional as F

from . import _lib
from . import chain as nqchain
from .configs import (CONFIGS, LLAMA2_7B, LLAMA3_70B, PROJ, TINY, DecoderConfig,  # noqa: F401  (re-exported)
                      uniform_rank)


class QuantLinearShard:
    """This rank's part of one NanoQuant layer, in the kernel layout (half2 planes)."""

    def __init__(self, vb, ub, s2, smid, s1):
        self.vb, self.ub, self.s2, self.smid, self.s1 = vb, ub, s2, smid, s1
        self.rank = vb.shape[0]
        self.in_features = s2.numel()
        self.out_features = s1.numel()

    def __call__(self, x: torch.Tensor) -> torch.Tensor:
        return torch.ops.nq_b200.linear(x, self.s2, self.vb, self.smid, self.ub, self.s1)

    def gemv(self, x):
        return torch.ops.nq_b200.gemv(x, self.s2, self.vb, self.smid, self.ub, self.s1)

    def nbytes(self) -> int:
        t = 4 * (self.vb.numel() + self.ub.numel()) + 2 * (self.s2.numel() + self.s1.numel())
        return t + (2 * self.smid.numel() if self.smid is not None else 0)


class QuantGroup:
    """Layers that read the same input (q/k/v, gate/up), run as one grouped launch."""

    def __init__(self, *members: QuantLinearShard):
        self.members = members
        self.s2 = [m.s2 for m in members]
        self.vb = [m.vb for m in members]
        self.smid = [m.smid for m in members]
        self.ub = [m.ub for m in members]
        self.s1 = [m.s1 for m in members]

    def __call__(self, x: torch.Tensor):
        return torch.ops.nq_b200.linear_group(x, self.s2, self.vb, self.smid, self.ub, self.s1)


def _random_planes(gen, rows: int, cols: int, device) -> torch.Tensor:
    """i.i.d. +-1 signs as half2 planes [rows, ceil(cols/32)], padding bits cleared (+1)."""
    w = (cols + 31) // 32
    p = torch.randint(-2 ** 31, 2 ** 31 - 1, (rows, w), generator=gen, dtype=torch.int32, device=device)
    tail = cols - 32 * (w - 1)
    if tail < 32:
        # half2 order: column j of the last word sits at bit 15 - j//2 + 16*(j%2)
        mask = 0
        for j in range(tail):
            mask |= 1 << (15 - j // 2 + 16 * (j % 2))
        if mask >= 2 ** 31:
            mask -= 2 ** 32
        p[:, -1] &= mask
    return p


def _make_layer(cfg: DecoderConfig, proj: str, layer: int, seed: int, tp_rank: int, tp: int, dtype, device,
                with_mid: bool = False) -> QuantLinearShard:
    out_f, in_f = cfg.io(proj)
    r = cfg.ranks[proj]
    gen = torch.Generator(device=device)
    gen.manual_seed(seed * 1000003 + layer * 17 + PROJ.index(proj))
    vb = _random_planes(gen, r, in_f, device)
    ub = _random_planes(gen, out_f, r, device)
    # variance-preserving scale magnitudes: |N(0,1)|/sqrt(in) for s2 and |N(0,1)|/sqrt(r) for s1,
    # so activations stay O(1) through a random-init network (values do not affect timing)
    s2 = (torch.randn(in_f, generator=gen, device=device).abs() / math.sqrt(in_f)).to(dtype)
    s1 = (torch.randn(out_f, generator=gen, device=device).abs() / math.sqrt(r)).to(dtype)
    smid = (torch.randn(r, generator=gen, device=device).abs() + 0.5).to(dtype) if with_mid else None
    return shard_layer(proj, vb, ub, s2, smid, s1, tp_rank, tp)


def shard_layer(proj: str, vb, ub, s2, smid, s1, tp_rank: int, tp: int) -> QuantLinearShard:
    """This rank's shard of a whole layer given as half2 planes and 1-D scales: column-parallel
    projections (q/k/v/gate/up) keep the U rows of their outputs, row-parallel ones (o/down) the V
    columns of their input slice (a multiple of 32 columns, whole words)."""
    if tp == 1:
        return QuantLinearShard(vb, ub, s2, smid, s1)
    out_f, in_f = s1.numel(), s2.numel()
    if proj in ("q", "k", "v", "gate", "up"):  # column-parallel: U rows of this rank's outputs
        n = out_f // tp
        sl = slice(tp_rank * n, (tp_rank + 1) * n)
        return QuantLinearShard(vb, ub[sl].contiguous(), s2, smid, s1[sl].contiguous())
    # row-parallel: V columns of this rank's input shard (shards are multiples of 32 columns)
    n = in_f // tp
    c0, c1 = tp_rank * n, (tp_rank + 1) * n
    assert c0 % 32 == 0 and c1 % 32 == 0, "input shards must be word aligned"
    return QuantLinearShard(vb[:, c0 // 32:c1 // 32].contiguous(), ub, s2[c0:c1].contiguous(), smid, s1)


def _map_peer_regions(lib, region: int, group, rank: int, world: int):
    """Exchange CUDA IPC handles of every rank's region (all_gather over `group`) and map the
    others' here: returns (every rank's region as mapped in this process, the ones opened)."""
    import ctypes
    handle = (ctypes.c_char * 64)()
    _lib.check(lib.nq_ipc_handle(region, handle))
    handles = [None] * world
    torch.distributed.all_gather_object(handles, bytes(handle), group=group)
    ptrs, opened = [], []
    for r in range(world):
        if r == rank:
            ptrs.append(region)
            continue
        peer = ctypes.c_void_p()
        _lib.check(lib.nq_ipc_open(ctypes.create_string_buffer(handles[r], 64), ctypes.byref(peer)))
        ptrs.append(peer.value)
        opened.append(peer.value)
    return ptrs, opened


class TPExchange:
    """The tensor-parallel sum fused into the decode GEMVs (nq_gemv_group_tp, include/nq_b200.h):
    the row-parallel o / down GEMVs PUSH their rounded output rows into every rank's receive buffer
    over NVLink, and the next GEMV's RMSNorm prologue PULLs (waits for every rank, sums in rank
    order).  One region per rank, mapped by every other rank over CUDA IPC here, once."""

    PULL, PUSH = 1, 2

    def __init__(self, group, rank: int, world: int, max_elems: int, device):
        import ctypes
        self.lib, self.rank, self.world = _lib.cuda_lib(), rank, world
        self.max_elems = (max_elems + 7) // 8 * 8
        with torch.cuda.device(device):
            region = ctypes.c_void_p()
            _lib.check(self.lib.nq_tp_region_alloc(world, self.max_elems, ctypes.byref(region)))
            self.region = region.value
            self.regions, self.opened = _map_peer_regions(self.lib, self.region, group, rank, world)
            torch.distributed.barrier(group=group)  # every region zeroed and mapped before any call

    def args(self, mode: int):
        return self.regions, self.rank, self.max_elems, mode

    def status(self) -> int:
        """The region's status word (NQ_OK, or NQ_ERR_DEVICE_TIMEOUT if a wait for another rank gave
        up); synchronises the current stream."""
        import ctypes
        st = ctypes.c_int(-1)
        n = self.lib.nq_tp_region_bytes(self.world, self.max_elems)
        _lib.check(self.lib.nq_workspace_status(self.region, n, torch.cuda.current_stream().cuda_stream,
                                                ctypes.byref(st)))
        return st.value


class PeerAllReduce:
    """Sum of a small tensor over the tensor-parallel ranks of one node through peer memory
    (nq_allreduce): every rank maps every other rank's region over CUDA IPC once, here; a call
    is one kernel launch, capturable in the decode graph.  Tensors above `max_elems` elements
    (prefill) go through torch.distributed instead; the choice depends only on the size, so
    every rank makes the same sequence of peer calls."""

    def __init__(self, group, rank: int, world: int, max_elems: int, device):
        import ctypes
        self.lib, self.rank, self.world, self.group = _lib.cuda_lib(), rank, world, group
        self.max_elems = max_elems
        with torch.cuda.device(device):
            region = ctypes.c_void_p()
            _lib.check(self.lib.nq_allreduce_region_alloc(world, max_elems, ctypes.byref(region)))
            self.region = region.value
            ptrs, self.opened = _map_peer_regions(self.lib, self.region, group, rank, world)
            self.ptrs = (ctypes.c_void_p * world)(*ptrs)
            torch.distributed.barrier(group=group)  # every region zeroed and mapped before any call

    def __call__(self, t: torch.Tensor) -> torch.Tensor:
        if t.numel() > self.max_elems or t.numel() % 8 or not t.is_contiguous():
            torch.distributed.all_reduce(t, group=self.group)
            return t
        dt = _lib.NQ_DTYPE_F16 if t.dtype == torch.float16 else _lib.NQ_DTYPE_BF16
        _lib.check(self.lib.nq_allreduce(dt, t.data_ptr(), t.data_ptr(), t.numel(), self.rank, self.world, self.ptrs,
                                         self.max_elems, torch.cuda.current_stream(t.device).cuda_stream))
        return t

    def status(self) -> int:
        """The region's device-side status word (NQ_OK, or NQ_ERR_DEVICE_TIMEOUT if a call gave up
        waiting for another rank); synchronises the current stream."""
        import ctypes
        st = ctypes.c_int(-1)
        n = self.lib.nq_allreduce_region_bytes(self.world, self.max_elems)
        _lib.check(self.lib.nq_workspace_status(self.region, n, torch.cuda.current_stream().cuda_stream,
                                                ctypes.byref(st)))
        return st.value


class Decoder:
    """One TP shard of the decoder plus its KV cache and a graph-capturable decode step."""

    def __init__(self, cfg: DecoderConfig, max_seq: int, batch: int = 1, tp_rank: int = 0, tp: int = 1,
                 group=None, seed: int = 0, dtype=torch.float16, device=None, with_mid: bool = False,
                 peer_allreduce: bool = False, tp_exchange: bool = True,
                 weights: Optional[dict] = None):
        """``weights`` (from nanoquant_b200.loader) replaces the seeded random weights: "embed",
        "lm_head", "final_norm" tensors and "layers", one dict per layer with "in_norm",
        "post_norm" and, per projection, (V planes, U planes, scale_pre, scale_mid, scale_post) --
        planes in half2 order, scales 1-D -- all on this rank's device, unsharded."""
        _lib.load_torch_ops()
        assert cfg.heads % tp == 0 and cfg.kv_heads % tp == 0 and cfg.ffn % tp == 0
        self.cfg, self.max_seq, self.batch, self.tp, self.tp_rank, self.group = cfg, max_seq, batch, tp, tp_rank, group
        self.dtype = dtype
        self.device = torch.device(device) if device is not None else torch.device("cuda", torch.cuda.current_device())
        dev = self.device
        self.hq, self.hkv = cfg.heads // tp, cfg.kv_heads // tp
        self.layers = []
        if weights is not None:
            cast = lambda t: None if t is None else t.to(device=dev, dtype=dtype).reshape(-1).contiguous()  # noqa: E731
            self.embed = weights["embed"].to(device=dev, dtype=dtype).contiguous()
            self.lm_head = weights["lm_head"].to(device=dev, dtype=dtype).contiguous()
            self.final_norm = cast(weights["final_norm"])
            for w in weights["layers"]:
                lay = {}
                for p in PROJ:
                    vb, ub, s2, smid, s1 = w[p]
                    lay[p] = shard_layer(p, vb.to(dev), ub.to(dev), cast(s2), cast(smid), cast(s1), tp_rank, tp)
                lay["in_norm"] = cast(w["in_norm"])
                lay["post_norm"] = cast(w["post_norm"])
                self.layers.append(lay)
        else:
            gen = torch.Generator(device=dev)
            gen.manual_seed(seed * 7919 + 1)
            self.embed = (torch.randn(cfg.vocab, cfg.hidden, generator=gen, device=dev) * 0.02).to(dtype)
            self.lm_head = (torch.randn(cfg.vocab, cfg.hidden, generator=gen, device=dev) * 0.02).to(dtype)
            self.final_norm = torch.ones(cfg.hidden, device=dev, dtype=dtype)
            for li in range(cfg.layers):
                lay = {p: _make_layer(cfg, p, li, seed, tp_rank, tp, dtype, dev, with_mid) for p in PROJ}
                lay["in_norm"] = torch.ones(cfg.hidden, device=dev, dtype=dtype)
                lay["post_norm"] = torch.ones(cfg.hidden, device=dev, dtype=dtype)
                self.layers.append(lay)
        for lay in self.layers:
            lay["qkv"] = QuantGroup(lay["q"], lay["k"], lay["v"])
            lay["gate_up"] = QuantGroup(lay["gate"], lay["up"])
        # cache capacity rounded up to whole 64-position blocks: each block of a head is then one
        # 16 KB-aligned range, which the decode attention streams far faster than unaligned ones
        cap = (max_seq + 63) // 64 * 64
        self.k_cache = torch.zeros(cfg.layers, batch, self.hkv, cap, cfg.head_dim, device=dev, dtype=dtype)
        self.v_cache = torch.zeros_like(self.k_cache)
        # decode-step state, all on the device
        self.tokens = torch.zeros(batch, dtype=torch.long, device=dev)
        self.pos = torch.zeros(batch, dtype=torch.int32, device=dev)
        self.seq_len = torch.ones(batch, dtype=torch.int32, device=dev)
        self.next_tokens = torch.zeros(batch, dtype=torch.long, device=dev)
        # RMSNorm / SiLU*up folded into the GEMV prologues and the gate's SiLU into its epilogue
        # (nq_gemv_group_ex); batches above 8 use the separate kernels.
        self.fuse_neighbours = True
        # the fused prologues stage their inputs in shared memory: where the RMSNorm one has no plan
        # (wide hidden sizes at large batches: Llama-3-70B at batch 8), the step uses separate
        # RMSNorm / SiLU*up kernels and plain GEMVs (and NCCL for tensor-parallel sums)
        if batch > 8 or not self._norm_prologue_fits():
            self.fuse_neighbours = False
        # gate * up in the down GEMV's prologue needs both FFN vectors staged in shared memory;
        # for wide FFN shards (Llama-3-70B on one GPU) no plan fits, and the block uses the
        # SiLU*up kernel and a plain down GEMV instead
        self.fuse_down = self.fuse_neighbours and self._down_prologue_fits()
        # tensor parallel: `peer_allreduce` sums the blocks' partial outputs through peer memory
        # (nq_allreduce) at decode sizes instead of torch.distributed / NCCL
        self.peer_ar = None
        if tp > 1 and peer_allreduce:
            self.peer_ar = PeerAllReduce(group, tp_rank, tp, 8 * cfg.hidden, dev)
        # `tp_exchange` (the default for tp > 1): the decode step's per-block sums run inside the
        # GEMVs (push from o / down, pull in the next RMSNorm prologue); NCCL stays for prefill
        # (every rank holds shards of the same shapes, so every rank makes the same choice)
        self.tpx = None
        if (tp > 1 and tp_exchange and not peer_allreduce and batch <= 8 and self.fuse_neighbours
                and self._exchange_fits()):
            self.tpx = TPExchange(group, tp_rank, tp, batch * cfg.hidden, dev)

    # ------------------------------------------------------------------ pieces
    def _norm_prologue_fits(self) -> bool:
        """Whether the q/k/v launch with RMSNorm(x + residual) in its prologue has a plan."""
        g = self.layers[0]["qkv"]
        x = torch.zeros(self.batch, self.cfg.hidden, device=self.device, dtype=self.dtype)
        try:
            torch.ops.nq_b200.gemv_group_ex(x, x, self.layers[0]["in_norm"], 1e-5, nqchain.RMSNORM, None, 0, g.s2, g.vb,
                                            g.smid, g.ub, g.s1)
        except RuntimeError as e:
            if "shared-memory budget" in str(e):
                return False
            raise
        torch.cuda.synchronize(self.device)
        return True

    def _down_prologue_fits(self) -> bool:
        dn = self.layers[0]["down"]
        g = torch.zeros(self.batch, dn.in_features, device=self.device, dtype=self.dtype)
        try:
            torch.ops.nq_b200.gemv_group_ex(g, g, None, 0.0, nqchain.MUL, None, 0, [dn.s2], [dn.vb], [dn.smid], [dn.ub],
                                            [dn.s1])
        except RuntimeError as e:
            if "shared-memory budget" in str(e):
                return False
            raise
        torch.cuda.synchronize(self.device)
        return True

    def _exchange_fits(self) -> bool:
        """Whether the four exchange GEMVs of a decoder block (q/k/v and gate/up pulling, o and
        down pushing) have a plan whose exchanging launch runs one CTA per SM at this shard's
        shapes: planned with NQ_TP_CHECK, nothing launched.  The two-launch GEMV of a wide shard
        (Llama-3-70B gate/up at TP2) qualifies when its pulling (stage-1) or pushing (stage-2)
        launch does; where it does not (70B at TP2 batch 8) the step keeps the NCCL sums."""
        ops, lay, B, dev, dt = torch.ops.nq_b200, self.layers[0], self.batch, self.device, self.dtype
        check, mx = 4, (B * self.cfg.hidden + 7) // 8 * 8
        ex = ([0] * self.tp, self.tp_rank, mx)
        h = torch.zeros(B, self.cfg.hidden, device=dev, dtype=dt)
        a = torch.zeros(B, self.hq * self.cfg.head_dim, device=dev, dtype=dt)
        f = torch.zeros(B, lay["down"].in_features, device=dev, dtype=dt)
        g, gu, ol, dn = lay["qkv"], lay["gate_up"], lay["o"], lay["down"]
        try:
            ops.gemv_group_tp(h, h, lay["in_norm"], 1e-5, nqchain.RMSNORM, torch.empty_like(h), 0, g.s2, g.vb, g.smid,
                              g.ub, g.s1, *ex, TPExchange.PULL | check)
            ops.gemv_group_tp(a, None, None, 0.0, nqchain.PLAIN, None, 0, [ol.s2], [ol.vb], [ol.smid], [ol.ub],
                              [ol.s1], *ex, TPExchange.PUSH | check)
            ops.gemv_group_tp(h, h, lay["post_norm"], 1e-5, nqchain.RMSNORM, torch.empty_like(h),
                              1 if self.fuse_down else 0, gu.s2, gu.vb, gu.smid, gu.ub, gu.s1, *ex,
                              TPExchange.PULL | check)
            if self.fuse_down:
                ops.gemv_group_tp(f, f, None, 0.0, nqchain.MUL, None, 0, [dn.s2], [dn.vb], [dn.smid], [dn.ub],
                                  [dn.s1], *ex, TPExchange.PUSH | check)
            else:
                ops.gemv_group_tp(f, None, None, 0.0, nqchain.PLAIN, None, 0, [dn.s2], [dn.vb], [dn.smid], [dn.ub],
                                  [dn.s1], *ex, TPExchange.PUSH | check)
        except RuntimeError as e:
            if "unsupported" in str(e) or "shared-memory budget" in str(e):
                return False
            raise
        return True

    def _all_reduce(self, t: torch.Tensor):
        if self.tp > 1:
            if self.peer_ar is not None:
                return self.peer_ar(t)
            torch.distributed.all_reduce(t, group=self.group)
        return t

    def quant_linears(self):
        for lay in self.layers:
            for p in PROJ:
                yield lay[p]

    def weight_bytes(self) -> int:
        """Bytes one decode token reads on this rank: quantized linears + lm_head (+ norms)."""
        return sum(q.nbytes() for q in self.quant_linears()) + self.lm_head.numel() * 2

    # ------------------------------------------------------------------ prefill
    @torch.no_grad()
    def prefill(self, prompt: torch.Tensor) -> torch.Tensor:
        """Run the prompt through the model, fill the caches and return the first generated token
        of every batch row (greedy).  ``prompt``: token ids [T] (batch 1) or [batch, T] (every row
        the same length).  All rows go through each projection as one GEMM of batch * T rows;
        attention is causal per row.  Sets the decode state."""
        if prompt.dim() == 1:
            prompt = prompt[None]
        B, T = prompt.shape
        assert B == self.batch, f"prompt has {B} rows, the decoder was built for batch {self.batch}"
        assert T < self.max_seq
        cfg, D = self.cfg, self.cfg.head_dim
        pos = torch.arange(T, dtype=torch.int32, device=self.device).repeat(B)
        bidx = torch.arange(B, dtype=torch.int32, device=self.device).repeat_interleave(T)
        h = F.embedding(prompt.reshape(-1).to(self.device), self.embed)
        residual = None
        for li, lay in enumerate(self.layers):
            x, residual = torch.ops.nq_b200.rmsnorm(h, residual, lay["in_norm"], cfg.rms_eps)
            q, k, v = lay["qkv"](x)
            q, k, v = q.view(B * T, self.hq, D), k.view(B * T, self.hkv, D), v.view(B * T, self.hkv, D)
            torch.ops.nq_b200.rope_cache(q, k, v, pos, bidx, self.k_cache[li], self.v_cache[li], cfg.rope_theta)
            a = F.scaled_dot_product_attention(q.view(B, T, self.hq, D).transpose(1, 2),
                                               k.view(B, T, self.hkv, D).transpose(1, 2),
                                               v.view(B, T, self.hkv, D).transpose(1, 2), is_causal=True,
                                               enable_gqa=self.hq != self.hkv)
            a = a.transpose(1, 2).reshape(B * T, self.hq * D).contiguous()
            o = self._all_reduce(lay["o"](a))
            x, residual = torch.ops.nq_b200.rmsnorm(o, residual, lay["post_norm"], cfg.rms_eps)
            act = torch.ops.nq_b200.silu_mul(*lay["gate_up"](x))
            h = self._all_reduce(lay["down"](act))
        last = torch.arange(B, device=self.device) * T + (T - 1)
        x, _ = torch.ops.nq_b200.rmsnorm(h[last].contiguous(), residual[last].contiguous(), self.final_norm,
                                         cfg.rms_eps)
        nxt = torch.argmax(x @ self.lm_head.t(), dim=-1)
        self.tokens.copy_(nxt)
        self.pos.fill_(T)
        self.seq_len.fill_(T + 1)
        return nxt

    # ------------------------------------------------------------------ decode
    @torch.no_grad()
    def _step_logits_fused(self) -> torch.Tensor:
        """Five launches per block: q/k/v with RMSNorm(x + residual) in its prologue, attention
        (RoPE + cache write fused), o, gate/up with RMSNorm(o + residual) in its prologue and
        SiLU on the gate in its epilogue, down with gate * up in its prologue."""
        cfg, B, D = self.cfg, self.batch, self.cfg.head_dim
        ops, eps = torch.ops.nq_b200, cfg.rms_eps
        if self.tpx is not None:
            return self._step_logits_exchange()
        d = F.embedding(self.tokens, self.embed)  # the first block's input; no residual yet
        residual = None
        for li, lay in enumerate(self.layers):
            g = lay["qkv"]
            res = torch.empty_like(d)
            q, k, v = ops.gemv_group_ex(d, residual, lay["in_norm"], eps, nqchain.RMSNORM, res, 0, g.s2, g.vb, g.smid,
                                        g.ub, g.s1)
            residual = res
            a = ops.decode_attention_rope(q.view(B, self.hq, D), k.view(B, self.hkv, D), v.view(B, self.hkv, D),
                                          self.pos, self.k_cache[li], self.v_cache[li], cfg.rope_theta)
            o = self._all_reduce(lay["o"](a.view(B, self.hq * D)))
            g = lay["gate_up"]
            res = torch.empty_like(o)
            gate, up = ops.gemv_group_ex(o, residual, lay["post_norm"], eps, nqchain.RMSNORM, res,
                                         1 if self.fuse_down else 0, g.s2, g.vb, g.smid, g.ub, g.s1)
            residual = res
            dn = lay["down"]
            if self.fuse_down:
                d = self._all_reduce(ops.gemv_group_ex(gate, up, None, 0.0, nqchain.MUL, None, 0, [dn.s2], [dn.vb],
                                                       [dn.smid], [dn.ub], [dn.s1])[0])
            else:
                d = self._all_reduce(dn.gemv(ops.silu_mul(gate, up)))
        x, _ = ops.rmsnorm(d, residual, self.final_norm, eps)
        return x @ self.lm_head.t()

    @torch.no_grad()
    def _step_logits_exchange(self) -> torch.Tensor:
        """The fused step with the tensor-parallel sums inside the GEMVs: o and down PUSH their
        partial rows to every rank; the next q/k/v or gate/up launch PULLs (its RMSNorm prologue
        sums the ranks' rows and adds the residual); a standalone pull feeds the final norm."""
        cfg, B, D = self.cfg, self.batch, self.cfg.head_dim
        ops, eps, ex = torch.ops.nq_b200, cfg.rms_eps, self.tpx
        d = F.embedding(self.tokens, self.embed)  # replicated on every rank: the first block does not pull
        residual = None
        for li, lay in enumerate(self.layers):
            g = lay["qkv"]
            res = torch.empty_like(d)
            if li == 0:
                q, k, v = ops.gemv_group_ex(d, residual, lay["in_norm"], eps, nqchain.RMSNORM, res, 0, g.s2, g.vb,
                                            g.smid, g.ub, g.s1)
            else:
                q, k, v = ops.gemv_group_tp(d, residual, lay["in_norm"], eps, nqchain.RMSNORM, res, 0, g.s2, g.vb,
                                            g.smid, g.ub, g.s1, *ex.args(ex.PULL))
            residual = res
            a = ops.decode_attention_rope(q.view(B, self.hq, D), k.view(B, self.hkv, D), v.view(B, self.hkv, D),
                                          self.pos, self.k_cache[li], self.v_cache[li], cfg.rope_theta)
            ol = lay["o"]
            o = ops.gemv_group_tp(a.view(B, self.hq * D), None, None, 0.0, nqchain.PLAIN, None, 0, [ol.s2], [ol.vb],
                                  [ol.smid], [ol.ub], [ol.s1], *ex.args(ex.PUSH))[0]
            g = lay["gate_up"]
            res = torch.empty_like(o)
            gate, up = ops.gemv_group_tp(o, residual, lay["post_norm"], eps, nqchain.RMSNORM, res,
                                         1 if self.fuse_down else 0, g.s2, g.vb, g.smid, g.ub, g.s1,
                                         *ex.args(ex.PULL))
            residual = res
            dn = lay["down"]
            if self.fuse_down:
                d = ops.gemv_group_tp(gate, up, None, 0.0, nqchain.MUL, None, 0, [dn.s2], [dn.vb], [dn.smid],
                                      [dn.ub], [dn.s1], *ex.args(ex.PUSH))[0]
            else:
                d = ops.gemv_group_tp(ops.silu_mul(gate, up), None, None, 0.0, nqchain.PLAIN, None, 0, [dn.s2],
                                      [dn.vb], [dn.smid], [dn.ub], [dn.s1], *ex.args(ex.PUSH))[0]
        d = ops.tp_pull(d, *ex.args(ex.PULL)[:3])
        x, _ = ops.rmsnorm(d, residual, self.final_norm, eps)
        return x @ self.lm_head.t()

    @torch.no_grad()
    def own_launches_per_step(self) -> int:
        """Kernels of this package that one decode step launches (library kernels such as the
        lm_head GEMM, argmax and the embedding gather are not counted)."""
        n = self.cfg.layers
        ar = 2 * n if self.peer_ar is not None else 0  # peer all-reduces (o and down of every block)
        if self.tpx is not None:  # sums inside the GEMVs; one standalone pull before the final norm
            return n * (5 if self.fuse_down else 6) + 1 + 1
        if self.fuse_neighbours and self.batch <= 8:
            return n * (5 if self.fuse_down else 6) + 1 + ar  # q/k/v, attention, o, gate/up, (SiLU*up,) down; final norm
        return n * (4 + 2 + 1 + 1) + 1 + ar  # four GEMVs, two norms, attention, SiLU·up; final norm

    def step_logits(self) -> torch.Tensor:
        """Logits for the current tokens at the current positions (writes the caches)."""
        if self.fuse_neighbours and self.batch <= 8:
            return self._step_logits_fused()
        cfg, B, D = self.cfg, self.batch, self.cfg.head_dim
        h = F.embedding(self.tokens, self.embed)
        residual = None
        for li, lay in enumerate(self.layers):
            x, residual = torch.ops.nq_b200.rmsnorm(h, residual, lay["in_norm"], cfg.rms_eps)
            q, k, v = lay["qkv"](x)
            q, k, v = q.view(B, self.hq, D), k.view(B, self.hkv, D), v.view(B, self.hkv, D)
            a = torch.ops.nq_b200.decode_attention_rope(q, k, v, self.pos, self.k_cache[li], self.v_cache[li],
                                                        cfg.rope_theta)
            o = self._all_reduce(lay["o"](a.view(B, self.hq * D)))
            x, residual = torch.ops.nq_b200.rmsnorm(o, residual, lay["post_norm"], cfg.rms_eps)
            act = torch.ops.nq_b200.silu_mul(*lay["gate_up"](x))
            h = self._all_reduce(lay["down"](act))
        x, _ = torch.ops.nq_b200.rmsnorm(h, residual, self.final_norm, cfg.rms_eps)
        return x @ self.lm_head.t()

    @torch.no_grad()
    def step(self) -> torch.Tensor:
        """One greedy decode step: next token from the current one, then advance the state."""
        logits = self.step_logits()
        self.next_tokens.copy_(torch.argmax(logits, dim=-1))
        self.tokens.copy_(self.next_tokens)
        self.pos.add_(1)
        self.seq_len.add_(1)
        return self.next_tokens

    def capture(self, warmup: int = 2) -> "GraphedStep":
        return GraphedStep(self, warmup)


class GraphedStep:
    """The decode step captured once as a CUDA graph; replay() = one autoregressive token.

    The graph advances the device-side state (tokens, positions) itself; warm-up steps run
    eagerly before capture and are rolled back so the caller's position is unchanged."""

    def __init__(self, dec: Decoder, warmup: int = 2):
        self.dec = dec
        saved = (dec.tokens.clone(), dec.pos.clone(), dec.seq_len.clone())
        s = torch.cuda.Stream(device=dec.device)
        s.wait_stream(torch.cuda.current_stream(dec.device))
        with torch.cuda.stream(s):
            for _ in range(warmup):
                dec.step()
        torch.cuda.current_stream(dec.device).wait_stream(s)
        self.graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(self.graph, stream=s):
            dec.step()
        dec.tokens.copy_(saved[0])
        dec.pos.copy_(saved[1])
        dec.seq_len.copy_(saved[2])
        torch.cuda.synchronize(dec.device)

    def replay(self) -> torch.Tensor:
        self.graph.replay()
        return self.dec.next_tokens

    def generate(self, host_tokens: torch.Tensor, host_out: torch.Tensor) -> torch.Tensor:
        """The user-facing step: host token ids (pinned int64 [batch]) in, next token ids out
        (written into the pinned ``host_out``), synchronised on the current stream."""
        self.dec.tokens.copy_(host_tokens, non_blocking=True)
        self.graph.replay()
        host_out.copy_(self.dec.next_tokens, non_blocking=True)
        torch.cuda.current_stream(self.dec.device).synchronize()
        return host_out

    def release(self):
        self.graph = None
