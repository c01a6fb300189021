"""Tensor-parallel decode on 2 GPUs (NCCL): the sharded model must produce the same greedy
tokens and nearly the same logits as the unsharded one.  Skipped with fewer than 2 GPUs."""
import os
import socket

import pytest
import torch
import torch.multiprocessing as mp

from nanoquant_b200.decoder import Decoder, DecoderConfig

pytestmark = pytest.mark.gpu

CFG = DecoderConfig("tp-small", 1024, 512, 2, 4, 2, 128, 1024,
                    {"q": 160, "k": 96, "v": 96, "o": 160, "gate": 200, "up": 200, "down": 200})


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _run(rank, world, port, prompt, steps, q):
    import datetime
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    torch.cuda.set_device(rank)
    torch.distributed.init_process_group("nccl", rank=rank, world_size=world,
                                         timeout=datetime.timedelta(seconds=60), device_id=torch.device("cuda", rank))
    try:
        dec = Decoder(CFG, max_seq=128, tp_rank=rank, tp=world, group=torch.distributed.group.WORLD, seed=3,
                      device=f"cuda:{rank}")
        first = int(dec.prefill(prompt.cuda())[0])
        logits = dec.step_logits().float().cpu()
        dec.tokens.fill_(int(torch.argmax(logits[0])))
        dec.pos.add_(1)
        dec.seq_len.add_(1)
        g = dec.capture(warmup=2)
        toks = [int(g.replay()[0]) for _ in range(steps)]
        g.release()
        torch.distributed.barrier(device_ids=[rank])
        if rank == 0:
            q.put((first, logits, toks))
    finally:
        torch.distributed.destroy_process_group()


@pytest.mark.skipif(torch.cuda.device_count() < 2, reason="needs 2 GPUs")
@pytest.mark.timeout(600)
def test_tp2_matches_tp1():
    prompt = torch.randint(0, CFG.vocab, (37,), generator=torch.Generator().manual_seed(9))
    ref = Decoder(CFG, max_seq=128, seed=3, device="cuda:0")
    first = int(ref.prefill(prompt.cuda())[0])
    logits = ref.step_logits().float().cpu()
    ref.tokens.fill_(int(torch.argmax(logits[0])))
    ref.pos.add_(1)
    ref.seq_len.add_(1)
    toks = [int(ref.step()[0]) for _ in range(6)]
    del ref
    torch.cuda.empty_cache()
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    procs = [ctx.Process(target=_run, args=(r, 2, port, prompt, 6, q)) for r in range(2)]
    for p in procs:
        p.start()
    got_first, got_logits, got_toks = q.get(timeout=500)
    for p in procs:
        p.join(timeout=120)
        assert p.exitcode == 0
    assert got_first == first
    rel = float((got_logits - logits).norm() / logits.norm())
    assert rel < 2e-2, rel
    assert got_toks == toks
