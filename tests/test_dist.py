"""Multi-rank host logic on CPU (gloo, world size 2-3): batch sharding, the
logits gather, and failure detection of a rank that never joins.

Each rank runs a small ViT with the SC operators on the noise surrogate (the
engine itself needs a GPU) on its shard; the gathered logits must equal the
single-process forward over the whole batch, row for row.
"""
import os
import socket
import time

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from scmp_vit_b200.dist import gather_logits, shard_range


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_shard_range_covers_batch_once():
    for gb in (1, 7, 256, 2048):
        for world in (1, 2, 3, 8):
            spans = [shard_range(gb, r, world) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == gb
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(b - a for a, b in spans) - min(b - a for a, b in spans) <= 1


def _model():
    from scmp_vit_b200 import sc_linear, vit
    sc_linear.set_noise_model(True)
    m = vit.vit_l14(seed=0, dim=64, depth=2, heads=2, hidden=128, img=28)
    vit.patch_vit(m, 7, ("qk", "av", "proj"))
    return m


def _images(gb):
    return torch.randn(gb, 3, 28, 28, generator=torch.Generator().manual_seed(5))


def _forward(m, x):
    torch.manual_seed(123)  # the noise surrogate draws from torch's RNG
    outs = []
    with torch.no_grad():
        for i in range(x.shape[0]):  # one image at a time: per-image RNG draws
            torch.manual_seed(1000 + i)
            outs.append(m(x[i:i + 1]))
    return torch.cat(outs)


def _worker(rank, world, port, gb, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world,
                            timeout=__import__("datetime").timedelta(seconds=30))
    try:
        m = _model()
        x = _images(gb)
        a, b = shard_range(gb, rank, world)
        outs = []
        with torch.no_grad():
            for i in range(a, b):
                torch.manual_seed(1000 + i)
                outs.append(m(x[i:i + 1]))
        local = torch.cat(outs) if outs else torch.zeros(0, 1000)
        full = gather_logits(local, gb, world)
        if rank == 0:
            q.put(full.numpy().copy())  # by value: the child may exit before the read
    finally:
        dist.destroy_process_group()


@pytest.mark.parametrize("world,gb", [(2, 6), (3, 7)])
def test_gathered_logits_match_single_process(world, gb):
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, gb, q)) for r in range(world)]
    for p in procs:
        p.start()
    full = torch.from_numpy(q.get(timeout=120))
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    from scmp_vit_b200 import sc_linear
    try:
        ref = _forward(_model(), _images(gb))
    finally:
        sc_linear.set_noise_model(False)  # the switch is process-wide
    assert full.shape == (gb, 1000)
    torch.testing.assert_close(full, ref, rtol=0, atol=0)


def _lonely(port, q):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    t0 = time.time()
    try:
        dist.init_process_group("gloo", rank=0, world_size=2,
                                timeout=__import__("datetime").timedelta(seconds=3))
        q.put(("joined", time.time() - t0))
    except Exception as e:  # the peer never arrives: rendezvous times out
        q.put(("error", type(e).__name__))


def test_missing_rank_is_detected_not_hung():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    p = ctx.Process(target=_lonely, args=(_free_port(), q))
    p.start()
    kind, info = q.get(timeout=90)
    p.join(timeout=30)
    if p.is_alive():
        p.kill()
    assert kind == "error", info
