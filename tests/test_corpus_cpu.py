"""Host corpus planning (bbh_plan_batches), no GPU: the C++ planner against a plain-Python
restatement of the same rules, its invariants, its edge cases, and a world-size-2 gloo run
in which each rank plans the same corpus and keeps its own batches.

Rules (the reference's bench/corpus.cu:87-124 sorts by length and cuts batches of a fixed
size; here batches are also bounded by tokens and assigned to ranks):
  * order = stable sort of the sentence indices by length;
  * batches = consecutive runs of order with <= max_batch sentences and <= max_tokens tokens;
  * each batch's work = sum over its sentences of 3,538,944 L + 1,536 L^2 FLOPs;
  * batches in decreasing work (ties: lower index) go to the least-loaded rank (ties: lower rank).
"""
import os
import sys

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def plan_py(lengths, max_batch, max_tokens, world):
    n = len(lengths)
    order = sorted(range(n), key=lambda i: (lengths[i], i))
    first, work = [], []
    tokens = count = 0
    for pos, i in enumerate(order):
        L = int(lengths[i])
        if count == 0 or count == max_batch or tokens + L > max_tokens:
            first.append(pos)
            work.append(0.0)
            tokens = count = 0
        tokens += L
        count += 1
        work[-1] += 3538944.0 * L + 1536.0 * L * L
    by_work = sorted(range(len(first)), key=lambda b: (-work[b], b))
    load = [0.0] * world
    rank = [0] * len(first)
    for b in by_work:
        r = min(range(world), key=lambda k: (load[k], k))
        rank[b] = r
        load[r] += work[b]
    return order, first + [n], rank, work


@pytest.mark.parametrize("seed,n,max_batch,max_tokens,world", [
    (0, 1, 4, 64, 1), (1, 37, 4, 100, 3), (2, 500, 64, 2048, 8), (3, 1000, 1024, 4096, 2),
    (4, 257, 16, 512, 5), (5, 64, 64, 100000, 1),
])
def test_plan_matches_restatement(seed, n, max_batch, max_tokens, world):
    import bbh

    rng = np.random.default_rng(seed)
    lengths = np.clip(np.round(rng.lognormal(np.log(12), 0.555, n)), 5, 64).astype(np.int32)
    lengths[rng.integers(0, n, size=max(1, n // 10))] = 9  # many ties
    p = bbh.plan_batches(lengths, max_batch, max_tokens, world)
    order, first, rank, work = plan_py(lengths.tolist(), max_batch, max_tokens, world)
    assert p.order.tolist() == order
    assert p.batch_first.tolist() == first
    assert p.batch_rank.tolist() == rank
    # invariants
    assert sorted(p.order.tolist()) == list(range(n))
    assert np.all(np.diff(lengths[p.order]) >= 0)
    for b, idx in p.batches():
        assert 1 <= len(idx) <= max_batch and lengths[idx].sum() <= max_tokens
    loads = np.zeros(world)
    for b in range(p.n_batches):
        loads[p.batch_rank[b]] += work[b]
    # LPT: no rank ends more than one batch's work above the least-loaded one
    assert loads.max() - loads.min() <= max(work) + 1e-6


def test_plan_edge_cases():
    import bbh

    p = bbh.plan_batches(np.zeros(0, np.int32), 8, 100, 4)
    assert p.n_batches == 0 and p.batch_first.tolist() == [0]
    p = bbh.plan_batches(np.array([3, 0, 2], np.int32), 8, 100, 4)  # zero-length sentence, world > batches
    assert p.order.tolist() == [1, 2, 0] and p.n_batches == 1 and p.batch_rank.tolist() == [0]
    with pytest.raises(bbh.BBHError) as e:
        bbh.plan_batches(np.array([10, 200], np.int32), 8, 100, 1)  # one sentence above max_tokens
    assert e.value.code == -2
    with pytest.raises(bbh.BBHError) as e:
        bbh.plan_batches(np.array([10, 600], np.int32), 8, 4096, 1)  # above the 512 positions
    assert e.value.code == -2
    with pytest.raises(bbh.BBHError) as e:
        bbh.plan_batches(np.array([10, -1], np.int32), 8, 100, 1)
    assert e.value.code == -1
    with pytest.raises(bbh.BBHError):
        bbh.plan_batches(np.array([10], np.int32), 8, 100, 0)


def _rank_main(rank, world, port, q):
    sys.path.insert(0, os.path.join(ROOT, "bert-by-hand_b200"))
    import bbh

    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    rng = np.random.default_rng(11)
    lengths = rng.integers(8, 129, size=5000).astype(np.int32)
    p = bbh.plan_batches(lengths, 1024, 1024 * 128, world)
    mine = np.full(5000, -1, np.int64)
    work = 0.0
    for b, idx in p.batches(rank):
        mine[idx] = rank
        work += float((3538944.0 * lengths[idx] + 1536.0 * lengths[idx].astype(np.float64) ** 2).sum())
    t = torch.from_numpy(mine)
    out = [torch.zeros_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    w = torch.tensor([work], dtype=torch.float64)
    ws = [torch.zeros_like(w) for _ in range(world)]
    dist.all_gather(ws, w)
    if rank == 0:
        q.put((torch.stack(out).numpy(), torch.cat(ws).numpy()))
    dist.barrier()
    dist.destroy_process_group()


def test_two_ranks_partition_the_corpus():
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = 29600 + os.getpid() % 300
    procs = [ctx.Process(target=_rank_main, args=(r, 2, port, q)) for r in range(2)]
    for pr in procs:
        pr.start()
    owners, works = q.get(timeout=240)
    for pr in procs:
        pr.join(timeout=120)
        assert pr.exitcode == 0
    # every sentence is owned by exactly one rank
    assert np.all((owners >= 0).sum(0) == 1)
    assert set(np.unique(owners[owners >= 0]).tolist()) == {0, 1}
    # LPT keeps the two ranks' FLOPs within a few percent
    assert abs(works[0] - works[1]) / works.sum() < 0.05


def test_cpp_dropin_plan_matches(tmp_path):
    """bert_by_hand.hpp's plan_batches (C++ caller, linked against libbbh.so) gives the
    same plan as the Python binding."""
    import shutil
    import subprocess

    import bbh

    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    if not os.path.exists(nvcc):
        pytest.skip("no nvcc")
    src = tmp_path / "plan.cpp"
    src.write_text(
        '#include <cstdio>\n#include "bert_by_hand.hpp"\n'
        "int main() {\n"
        "  std::vector<int32_t> L;\n"
        "  for (int i = 0; i < 300; ++i) L.push_back(5 + (i * 37) % 60);\n"
        "  CorpusPlan p = plan_batches(L, 16, 400, 3);\n"
        "  std::printf(\"%d\\n\", p.n_batches);\n"
        "  for (int v : p.order) std::printf(\"%d \", v);\n  std::printf(\"\\n\");\n"
        "  for (int v : p.batch_first) std::printf(\"%d \", v);\n  std::printf(\"\\n\");\n"
        "  for (int v : p.batch_rank) std::printf(\"%d \", v);\n  std::printf(\"\\n\");\n"
        "  return 0;\n}\n")
    exe = tmp_path / "plan"
    libdir = os.path.join(ROOT, "bert-by-hand_b200")
    r = subprocess.run([nvcc, "-std=c++17", "-I" + os.path.join(ROOT, "include"), str(src), "-o", str(exe),
                        "-L" + libdir, "-lbbh", "-Xlinker", "-rpath=" + libdir], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    out = subprocess.run([str(exe)], capture_output=True, text=True, check=True).stdout.split("\n")
    lengths = np.array([5 + (i * 37) % 60 for i in range(300)], np.int32)
    p = bbh.plan_batches(lengths, 16, 400, 3)
    assert int(out[0]) == p.n_batches
    assert [int(v) for v in out[1].split()] == p.order.tolist()
    assert [int(v) for v in out[2].split()] == p.batch_first.tolist()
    assert [int(v) for v in out[3].split()] == p.batch_rank.tolist()
