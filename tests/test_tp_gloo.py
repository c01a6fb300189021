"""Tensor-parallel sharding of the decoder's NanoQuant layers, checked on CPU with two gloo
ranks: column-parallel shards (U split by output rows) concatenate to the full layer and
row-parallel shards (V split by input columns) all-reduce to it.  The per-shard math is the
reference dense path evaluated by the oracle, so no GPU is involved."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from nanoquant_b200.decoder import LLAMA2_7B, PROJ, TINY, DecoderConfig, _make_layer
from oracle import decoder_ref as ref
from oracle import oracle as orc

SMALL = DecoderConfig("small-tp", 512, 512, 1, 4, 2, 128, 1024,
                      {"q": 100, "k": 40, "v": 40, "o": 100, "gate": 150, "up": 150, "down": 150})


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        errs = []
        g = torch.Generator().manual_seed(11)
        for proj in PROJ:
            out_f, in_f = SMALL.io(proj)
            full = _make_layer(SMALL, proj, 0, 5, 0, 1, torch.float16, "cpu", with_mid=True)
            shard = _make_layer(SMALL, proj, 0, 5, rank, world, torch.float16, "cpu", with_mid=True)
            x = torch.randn(3, in_f, generator=g)
            want = ref.linear(x, ref.dense_factors(full))
            if proj in ("q", "k", "v", "gate", "up"):
                part = ref.linear(x, ref.dense_factors(shard))
                parts = [torch.empty_like(part) for _ in range(world)]
                dist.all_gather(parts, part)
                got = torch.cat(parts, dim=1)
            else:
                n = in_f // world
                part = ref.linear(x[:, rank * n:(rank + 1) * n].contiguous(), ref.dense_factors(shard))
                dist.all_reduce(part)
                got = part
            errs.append((proj, orc.rel_l2(got.numpy(), want.numpy())))
        q.put((rank, errs))
    finally:
        dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_tp2_shards_reassemble_full_layers():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, 2, port, q)) for r in range(2)]
    for p in procs:
        p.start()
    results = [q.get(timeout=240) for _ in procs]
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    for rank, errs in results:
        for proj, e in errs:
            assert e < 1e-5, (rank, proj, e)


def test_tp_shapes_divide_for_benchmark_configs():
    for cfg in (LLAMA2_7B, TINY):
        for tp in (1, 2, 4, 8):
            if cfg.heads % tp or cfg.kv_heads % tp:
                continue
            for proj in ("o", "down"):
                assert (cfg.io(proj)[1] // tp) % 32 == 0


def test_packed_bytes_per_token_7b():
    # section 8(d) per-call bytes at batch 1, minus the activation terms, times 32 layers
    per_layer = 4 * (1199104 - 4 * 4096) + 2 * (3974144 - 2 * (11008 + 4096)) + (3951680 - 2 * (11008 + 4096))
    assert LLAMA2_7B.packed_bytes_per_token() == per_layer * 32
