"""Host-side sharding logic of the multi-GPU bench, run as world-size-2 gloo ranks on CPU:
each rank builds its own length-bucketed shard, the shards are disjoint and cover the
corpus, and the all-gather of per-rank results reassembles the global order."""
import os
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _rank_main(rank, world, port, q):
    sys.path.insert(0, os.path.join(ROOT, "bert-by-hand_b200"))
    import synthetic as sy

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    n, batch = 3000, 256
    lengths = sy.lengths_uniform(n, 8, 128, seed=3 + 7919 * rank)
    corpus = sy.bucketed_corpus(lengths, batch, seed=3 + 104729 * rank)
    # per-sentence "embedding" stand-in: (rank, original index, length) rows
    emb = np.zeros((n, 3), np.float32)
    for b in corpus.batches:
        for k in range(b.count):
            src = corpus.order[b.first + k]
            emb[b.first + k] = (rank, src, lengths[src])
        assert b.tokens == int(b.cu[-1]) and b.max_len == int(np.diff(b.cu).max())
        assert np.all(np.diff(b.cu) >= 8)
    t = torch.from_numpy(emb)
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    if rank == 0:
        g = torch.cat(out).numpy()
        q.put(g)
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_rank_shards_gather():
    world = 2
    port = 29500 + os.getpid() % 1000
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    g = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    assert g.shape == (6000, 3)
    for r in range(world):
        part = g[r * 3000:(r + 1) * 3000]
        assert np.all(part[:, 0] == r)
        # every original sentence index appears exactly once per rank, in length order
        assert sorted(part[:, 1].astype(int).tolist()) == list(range(3000))
        assert np.all(np.diff(part[:, 2]) >= 0)


def _failing_rank(rank, world, port):
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    import datetime

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=10))
    if rank == 1:
        raise SystemExit(3)  # a rank leaves between steps
    try:
        dist.all_reduce(torch.ones(1))
        code = 0
    except Exception:
        code = 7  # the survivor learns of it on the host, from its collective
    os._exit(code)


@pytest.mark.timeout(300)
def test_rank_failure_surfaces_on_host():
    world = 2
    port = 30500 + os.getpid() % 1000
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_failing_rank, args=(r, world, port)) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(timeout=120)
    assert procs[1].exitcode == 3
    assert procs[0].exitcode == 7
