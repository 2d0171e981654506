"""Host-side sharding logic of the multi-GPU bench (bert-by-hand_b200/sharding.py), run as
world-size-2 gloo ranks on CPU: every rank plans the SAME corpus with bbh_plan_batches(...,
world=2), packs its own batches, and Rank0Gather reassembles every sentence's row on rank 0
in corpus order. Stand-in "embeddings" encode (sentence index, length, rank, token checksum)
so a misplaced or duplicated row, a wrong token gather, or a missing sentence is caught."""
import os
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _corpus(n):
    sys.path.insert(0, os.path.join(ROOT, "bert-by-hand_b200"))
    import synthetic as sy

    lengths = sy.lengths_uniform(n, 8, 128, seed=3)
    ids = sy.sentence_tokens(lengths, 3)
    offsets = np.zeros(n + 1, np.int64)
    offsets[1:] = np.cumsum(lengths)
    return lengths, ids, offsets


def _rank_main(rank, world, port, q):
    sys.path.insert(0, os.path.join(ROOT, "bert-by-hand_b200"))
    import bbh
    import sharding

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    n, batch = 3000, 256
    lengths, ids, offsets = _corpus(n)
    types = (ids % 2).astype(np.int32)
    plan = bbh.plan_batches(lengths, batch, batch * 128, world)
    sh = sharding.shard(plan, rank, ids, types, offsets)
    # rows of this rank in plan order: (sentence, length, rank, sum of its ids, sum of types)
    rows = np.zeros((sh.order.size, 5), np.float64)
    for b in sh.batches:
        assert b.tokens == int(b.cu[-1]) and b.max_len == int(np.diff(b.cu).max())
        for k in range(b.count):
            s, e = b.tok + int(b.cu[k]), b.tok + int(b.cu[k + 1])
            rows[b.row + k] = (sh.order[b.row + k], e - s, rank, sh.ids[s:e].sum(), sh.types[s:e].sum())
    gat = sharding.Rank0Gather(plan, world, rank, n, "cpu", dtype=torch.float64, width=5)
    out = gat(torch.from_numpy(rows))
    if rank == 0:
        q.put((out.numpy().copy(), gat.counts))
    dist.barrier()
    dist.destroy_process_group()


@pytest.mark.timeout(300)
def test_two_rank_plan_shards_and_rank0_gather():
    world = 2
    port = 29500 + os.getpid() % 1000
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    procs = [ctx.Process(target=_rank_main, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    g, counts = q.get(timeout=240)
    for p in procs:
        p.join(timeout=60)
        assert p.exitcode == 0
    lengths, ids, offsets = _corpus(3000)
    assert g.shape == (3000, 5) and sum(counts) == 3000 and min(counts) > 0
    # row i is sentence i, with its own length and tokens, computed by exactly one rank
    assert np.array_equal(g[:, 0], np.arange(3000))
    assert np.array_equal(g[:, 1], lengths)
    want = np.array([ids[offsets[i]:offsets[i + 1]].sum() for i in range(3000)], np.float64)
    assert np.array_equal(g[:, 3], want)
    want_t = np.array([(ids[offsets[i]:offsets[i + 1]] % 2).sum() for i in range(3000)], np.float64)
    assert np.array_equal(g[:, 4], want_t)
    assert set(np.unique(g[:, 2]).tolist()) == {0.0, 1.0}
    # both ranks carry a similar share of the work (LPT on FLOPs)
    work = np.zeros(2)
    for r in (0, 1):
        L = lengths[g[:, 2] == r].astype(np.float64)
        work[r] = (3538944.0 * L + 1536.0 * L * L).sum()
    assert abs(work[0] - work[1]) / work.sum() < 0.05


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
