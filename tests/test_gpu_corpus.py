"""Host corpus driver on the GPU (bbh_embed_corpus): the pipelined host->device->host loop
gives exactly the embeddings of one bbh_embed_varlen per planned batch, in corpus order,
matching the CPU oracle; two ranks' halves of a plan reassemble the whole corpus; plans
that do not fit the workspace are rejected before any work is queued."""
import numpy as np
import pytest
import torch

from oracle import model as om

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


@pytest.fixture(scope="module")
def setup():
    import bbh
    import synthetic as sy

    w = om.make_weights(0)
    gw = bbh.ModelWeights.from_numpy(w, 6, 0)
    rng = np.random.default_rng(5)
    n = 700
    lengths = np.clip(np.round(rng.lognormal(np.log(12), 0.555, n)), 5, 64).astype(np.int32)
    lengths[:40] = rng.integers(65, 129, size=40)  # some long sentences too
    ids = sy.sentence_tokens(lengths, 5)
    types = (rng.random(ids.size) < 0.2).astype(np.int32)
    offsets = np.zeros(n + 1, np.int64)
    offsets[1:] = np.cumsum(lengths)
    return bbh, w, gw, lengths, ids, types, offsets


def test_corpus_matches_per_batch_forward(setup):
    bbh, w, gw, lengths, ids, types, offsets = setup
    plan = bbh.plan_batches(lengths, 96, 4096, 1)
    ws = bbh.Workspace(gw, 4096, 96, 128)
    got = ws.embed_corpus(ids, types, offsets, plan)
    # the same batches, one bbh_embed_varlen each, device inputs
    ref = np.zeros_like(got)
    for b, idx in plan.batches():
        seg_ids = np.concatenate([ids[offsets[i]:offsets[i + 1]] for i in idx])
        seg_types = np.concatenate([types[offsets[i]:offsets[i + 1]] for i in idx])
        cu = np.zeros(len(idx) + 1, np.int32)
        cu[1:] = np.cumsum(lengths[idx])
        d = lambda a: torch.as_tensor(a, dtype=torch.int32, device="cuda")
        out = ws.embed_varlen(d(seg_ids), d(seg_types), d(cu), int(lengths[idx].max()))
        ref[idx] = out.cpu().numpy()
    assert ws.device_error() == 0
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))
    # against the CPU oracle on a sample of sentences (cosine gate of the north star)
    orc = om.Oracle(w)
    sample = np.r_[0:24, 300:324]
    cu = np.zeros(sample.size + 1, np.int64)
    cu[1:] = np.cumsum(lengths[sample])
    seg_ids = np.concatenate([ids[offsets[i]:offsets[i + 1]] for i in sample])
    seg_types = np.concatenate([types[offsets[i]:offsets[i + 1]] for i in sample])
    e = orc.embed_varlen(seg_ids, seg_types, cu).numpy()
    g = got[sample].astype(np.float64)
    cos = (g * e).sum(1) / (np.linalg.norm(g, axis=1) * np.linalg.norm(e, axis=1))
    assert cos.min() >= 0.9999


def test_two_ranks_reassemble(setup):
    bbh, w, gw, lengths, ids, types, offsets = setup
    one = bbh.plan_batches(lengths, 128, 8192, 1)
    two = bbh.plan_batches(lengths, 128, 8192, 2)
    ws = bbh.Workspace(gw, 8192, 128, 128)
    full = ws.embed_corpus(ids, types, offsets, one)
    half = np.zeros_like(full)
    for r in (0, 1):
        ws.embed_corpus(ids, types, offsets, two, rank=r, out=half)
        mine = np.concatenate([idx for _, idx in two.batches(r)])
        assert np.abs(half[mine].astype(np.float32)).sum() > 0
    # same batches at both world sizes (assignment differs), so identical results
    assert np.array_equal(full.view(np.uint16), half.view(np.uint16))
    norms = np.linalg.norm(full.astype(np.float32), axis=1)
    assert np.all(np.abs(norms - 1) < 2e-3)


def test_rank_workspace_sized_for_its_own_batches(setup):
    """A rank's workspace needs only its own batches' capacity: another rank's larger batches
    are not this rank's to run (the multi-GPU bench sizes each rank's workspace this way);
    host and device outputs agree with the one-rank run."""
    bbh, w, gw, lengths, ids, types, offsets = setup
    one = bbh.plan_batches(lengths, 128, 8192, 1)
    two = bbh.plan_batches(lengths, 128, 8192, 2)
    full = bbh.Workspace(gw, 8192, 128, 128).embed_corpus(ids, types, offsets, one)
    for r in (0, 1):
        mine = two.rank_order(r)
        own_tokens = max(int(lengths[idx].sum()) for _, idx in two.batches(r))
        own_len = max(int(lengths[idx].max()) for _, idx in two.batches(r))
        ws = bbh.Workspace(gw, own_tokens, 128, own_len)
        host = ws.embed_corpus(ids, types, offsets, two, rank=r)
        dev = ws.embed_corpus_device(ids, types, offsets, two, rank=r)
        assert np.array_equal(host[mine].view(np.uint16), full[mine].view(np.uint16))
        assert np.array_equal(dev[:mine.size].cpu().numpy().view(np.uint16), full[mine].view(np.uint16))


def test_capacity_checked_before_work(setup):
    bbh, w, gw, lengths, ids, types, offsets = setup
    ws = bbh.Workspace(gw, 1024, 32, 128)
    plan = bbh.plan_batches(lengths, 64, 4096, 1)  # batches larger than the workspace
    with pytest.raises(bbh.BBHError) as e:
        ws.embed_corpus(ids, types, offsets, plan)
    assert e.value.code == -2
    short = bbh.Workspace(gw, 4096, 96, 64)  # max_len below the longest sentence
    with pytest.raises(bbh.BBHError) as e:
        short.embed_corpus(ids, types, offsets, bbh.plan_batches(lengths, 96, 4096, 1))
    assert e.value.code == -2
    assert ws.device_error() == 0


def test_two_lanes_bit_identical(setup):
    """Two compute lanes (a second workspace and stream, alternate batches) give exactly the
    one-lane results."""
    bbh, w, gw, lengths, ids, types, offsets = setup
    plan = bbh.plan_batches(lengths, 64, 4096, 1)
    one = bbh.Workspace(gw, 4096, 64, 128).embed_corpus(ids, types, offsets, plan)
    ws = bbh.Workspace(gw, 4096, 64, 128)
    ws.set_corpus_lanes(2)
    two = ws.embed_corpus(ids, types, offsets, plan)
    assert plan.n_batches > 4
    assert np.array_equal(one.view(np.uint16), two.view(np.uint16))
    with pytest.raises(bbh.BBHError):
        ws.set_corpus_lanes(3)


@pytest.mark.parametrize("lanes", [1, 2])
def test_padded_corpus_matches_per_batch_embed(setup, lanes):
    """bbh_embed_padded (the reference's padded bench loop as one call, host arrays in and
    out) gives exactly one bbh_embed per batch of consecutive sentences, last batch short."""
    bbh, w, gw, *_ = setup
    rng = np.random.default_rng(11)
    n, seq, batch = 150, 48, 32
    lens = rng.integers(3, seq + 1, size=n)
    ids = rng.integers(1000, 30522, size=(n, seq)).astype(np.int32)
    ids[:, 0] = 101
    mask = (np.arange(seq)[None, :] < lens[:, None]).astype(np.int32)
    ids[np.arange(n), lens - 1] = 102
    ids *= mask
    types = ((rng.random((n, seq)) < 0.3) * mask).astype(np.int32)
    ws = bbh.Workspace(gw, batch * seq, batch, seq)
    ws.set_corpus_lanes(lanes)
    got = ws.embed_padded(ids, types, mask, batch)
    ref = np.zeros_like(got)
    d = lambda a: torch.as_tensor(a, dtype=torch.int32, device="cuda")
    for f in range(0, n, batch):
        sl = slice(f, min(n, f + batch))
        ref[sl] = ws.embed(d(ids[sl]), d(types[sl]), d(mask[sl])).cpu().numpy()
    assert ws.device_error() == 0
    assert np.array_equal(got.view(np.uint16), ref.view(np.uint16))
    norms = np.linalg.norm(got.astype(np.float32), axis=1)
    assert np.all(np.abs(norms - 1) < 2e-3)
    with pytest.raises(bbh.BBHError) as e:
        ws.embed_padded(ids, types, mask, batch + 1)
    assert e.value.code == -2
