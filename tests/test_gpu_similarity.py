"""The similarity step after the path, device half: bbh_pair_similarity against numpy on the
same fp16 embeddings, out-of-range pairs, and the whole evaluation (model embeddings ->
pair cosines -> Spearman) against the CPU oracle's embeddings and scipy."""
import numpy as np
import pytest
import torch
from scipy.stats import spearmanr

from oracle import model as om

pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module", autouse=True)
def _need_gpu():
    if not torch.cuda.is_available():
        pytest.skip("no GPU")


def test_pair_similarity_matches_numpy():
    import bbh

    rng = np.random.default_rng(0)
    n, m = 3000, 20000
    e = rng.standard_normal((n, 384)).astype(np.float32)
    e /= np.linalg.norm(e, axis=1, keepdims=True)
    e16 = e.astype(np.float16)
    pairs = rng.integers(0, n, size=(m, 2)).astype(np.int32)
    pairs[:5] = [[0, 0], [1, 2], [n - 1, n - 1], [n - 1, 0], [7, 7]]
    sims = bbh.pair_similarity(torch.from_numpy(e16).cuda(), torch.from_numpy(pairs).cuda()).cpu().numpy()
    ref = np.einsum("ij,ij->i", e16[pairs[:, 0]].astype(np.float64), e16[pairs[:, 1]].astype(np.float64))
    assert np.abs(sims - ref).max() < 1e-5
    bad = torch.tensor([[0, n], [-1, 3], [2, 3]], dtype=torch.int32).cuda()
    s = bbh.pair_similarity(torch.from_numpy(e16).cuda(), bad).cpu().numpy()
    assert np.isnan(s[0]) and np.isnan(s[1]) and not np.isnan(s[2])


def test_evaluation_end_to_end():
    """benchmark.py's correlate(): pair cosines of the model's embeddings vs gold scores."""
    import bbh
    import synthetic as sy

    w = om.make_weights(0)
    gw = bbh.ModelWeights.from_numpy(w, 6, 0)
    rng = np.random.default_rng(9)
    n = 200
    lengths = np.clip(np.round(rng.lognormal(np.log(12), 0.555, n)), 5, 64).astype(np.int32)
    ids = sy.sentence_tokens(lengths, 9)
    offsets = np.zeros(n + 1, np.int64)
    offsets[1:] = np.cumsum(lengths)
    ws = bbh.Workspace(gw, 8192, 256, 64)
    emb = ws.embed_corpus(ids, None, offsets, bbh.plan_batches(lengths, 256, 8192, 1))
    pairs = rng.integers(0, n, size=(500, 2)).astype(np.int32)
    gold = np.round(rng.uniform(0, 5, 500) * 5) / 5
    sims = bbh.pair_similarity(torch.from_numpy(emb).cuda(), torch.from_numpy(pairs).cuda()).cpu().numpy()
    rho = bbh.spearman(sims, gold)
    # oracle: CPU fp32 embeddings of the same sentences, numpy cosines, scipy Spearman
    cu = offsets.astype(np.int64)
    ref_emb = om.Oracle(w).embed_varlen(ids, np.zeros_like(ids), cu).numpy()
    ref_sims = np.einsum("ij,ij->i", ref_emb[pairs[:, 0]], ref_emb[pairs[:, 1]])
    assert np.abs(sims - ref_sims).max() < 2e-3
    assert abs(rho - spearmanr(ref_sims, gold).statistic) < 1e-2
    assert abs(rho - spearmanr(sims, gold).statistic) < 1e-12
