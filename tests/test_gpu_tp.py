"""Tensor-parallel decode on 2 GPUs: the sharded model must produce the same greedy tokens and
nearly the same logits as the unsharded one, with the per-block sums fused into the GEMVs (the
default exchange), through NCCL, or through the standalone peer all-reduce.  A one-block model of
Llama-3-70B width runs the exchange through the two-launch GEMV (its gate/up shard pulls in the
stage-1 launch; at batch 2 its down shard pushes from the stage-2 launch).  Skipped with fewer
than 2 GPUs."""
import os
import tempfile

import pytest
import torch
import torch.multiprocessing as mp

from nanoquant_b200.configs import LLAMA3_70B
from nanoquant_b200.decoder import Decoder, DecoderConfig

pytestmark = pytest.mark.gpu

CFG = DecoderConfig("tp-small", 1024, 512, 2, 4, 2, 128, 1024,
                    {"q": 160, "k": 96, "v": 96, "o": 160, "gate": 200, "up": 200, "down": 200})
W70B = DecoderConfig("llama3-70b-1l", 4096, 8192, 1, 64, 8, 128, 28672, dict(LLAMA3_70B.ranks),
                     rope_theta=LLAMA3_70B.rope_theta)


def _rendezvous():
    """A fresh file for torch.distributed's file rendezvous (no TCP port that another process
    could hold)."""
    fd, path = tempfile.mkstemp(prefix="nq_tp_rdzv_")
    os.close(fd)
    os.unlink(path)
    return "file://" + path


def _run(rank, world, rdzv, prompt, steps, q, mode="exchange", cfg=CFG):
    import datetime
    os.environ.update(NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group("nccl", init_method=rdzv, rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        dec = Decoder(cfg, max_seq=128, batch=prompt.shape[0], tp_rank=rank, tp=world,
                      group=torch.distributed.group.WORLD, seed=3, peer_allreduce=mode == "peer_allreduce",
                      tp_exchange=mode == "exchange", device=f"cuda:{rank}")
        assert (dec.tpx is not None) == (mode == "exchange")
        first = dec.prefill(prompt.cuda()).tolist()
        logits = dec.step_logits().float().cpu()
        dec.tokens.copy_(torch.argmax(logits, dim=-1))
        dec.pos.add_(1)
        dec.seq_len.add_(1)
        g = dec.capture(warmup=2)
        toks = [g.replay().tolist() for _ in range(steps)]
        g.release()
        status = dec.tpx.status() if dec.tpx is not None else 0
        torch.distributed.barrier(device_ids=[rank])
        q.put((rank, first, logits, toks, status))
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.timeout(300)
@pytest.mark.parametrize("mode,cfg,batch", [("exchange", CFG, 1), ("nccl", CFG, 1), ("peer_allreduce", CFG, 1),
                                            ("exchange", W70B, 1), ("exchange", W70B, 2)],
                         ids=["exchange", "nccl", "peer_allreduce", "exchange-70b-width", "exchange-70b-width-b2"])
def test_tp2_matches_tp1(mode, cfg, batch):
    prompt = torch.randint(0, cfg.vocab, (batch, 37), generator=torch.Generator().manual_seed(9))
    ref = Decoder(cfg, max_seq=128, batch=batch, seed=3, device="cuda:0")
    first = ref.prefill(prompt.cuda()).tolist()
    logits = ref.step_logits().float().cpu()
    ref.tokens.copy_(torch.argmax(logits, dim=-1))
    ref.pos.add_(1)
    ref.seq_len.add_(1)
    toks = [ref.step().tolist() for _ in range(6)]
    del ref
    torch.cuda.empty_cache()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    rdzv = _rendezvous()
    procs = [ctx.Process(target=_run, args=(r, 2, rdzv, prompt, 6, q, mode, cfg)) for r in range(2)]
    for p in procs:
        p.start()
    outs = sorted([q.get(timeout=240) for _ in range(2)], key=lambda t: t[0])
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    for rank, got_first, got_logits, got_toks, status in outs:
        assert got_first == first
        rel = float((got_logits - logits).norm() / logits.norm())
        assert rel < 2e-2, rel
        assert got_toks == toks
        assert status == 0, f"rank {rank}: device-side timeout in the exchange"
    # the ranks' residual streams are bit-identical, so are their logits
    assert torch.equal(outs[0][2], outs[1][2])


def _ar_run(rank, world, rdzv, q):
    import datetime
    os.environ.update(NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group("nccl", init_method=rdzv, rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        from nanoquant_b200.decoder import PeerAllReduce
        dev = torch.device("cuda", rank)
        ar = PeerAllReduce(torch.distributed.group.WORLD, rank, world, 8192, dev)
        eager = []
        for it in range(5):  # consecutive calls alternate the receive buffers
            x = _ar_input(it, rank).to(dev)
            ar(x)
            eager.append(x.cpu())
        buf = torch.empty(4096, dtype=torch.float16, device=dev)
        s = torch.cuda.Stream(device=dev)
        s.wait_stream(torch.cuda.current_stream(dev))
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=s):
            ar(buf)
        graphed = []
        for it in range(5, 8):  # the same launch replayed: device-side epochs keep the ranks in step
            buf.copy_(_ar_input(it, rank).to(dev))
            g.replay()
            graphed.append(buf.cpu())
        torch.cuda.synchronize(dev)
        status = ar.status()
        del g
        torch.distributed.barrier(device_ids=[rank])
        q.put((rank, eager, graphed, status))
    finally:
        torch.distributed.destroy_process_group()


def _ar_input(it: int, rank: int) -> torch.Tensor:
    g = torch.Generator().manual_seed(1000 * it + rank)
    return torch.randn(4096, generator=g).half()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.timeout(300)
def test_peer_allreduce_two_gpus():
    """nq_allreduce over 2 GPUs: exactly the float32 rank-order sum rounded once, the same bits on
    both ranks, for eager calls and for replays of a captured launch, and no device timeout."""
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    rdzv = _rendezvous()
    procs = [ctx.Process(target=_ar_run, args=(r, world, rdzv, q)) for r in range(world)]
    for p in procs:
        p.start()
    out = [q.get(timeout=240) for _ in range(world)]
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    out.sort(key=lambda t: t[0])
    for it in range(8):
        want = sum(_ar_input(it, r).float() for r in range(world)).half()
        for rank, eager, graphed, status in out:
            got = eager[it] if it < 5 else graphed[it - 5]
            assert torch.equal(got, want), f"rank {rank} call {it}"
    assert all(st == 0 for _, _, _, st in out)
