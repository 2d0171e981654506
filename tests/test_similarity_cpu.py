"""The similarity step after the path, host half: bbh_spearman against scipy.stats.spearmanr
(the reference's scripts/benchmark.py:54-61 correlates pair cosines with gold scores that
way), including ties, constant inputs and argument errors."""
import numpy as np
import pytest
from scipy.stats import spearmanr


@pytest.mark.parametrize("seed,n,ties", [(0, 2, False), (1, 10, False), (2, 1379, False), (3, 1379, True),
                                         (4, 5000, True)])
def test_spearman_matches_scipy(seed, n, ties):
    import bbh

    rng = np.random.default_rng(seed)
    x = rng.standard_normal(n).astype(np.float32)
    y = (0.6 * x + rng.standard_normal(n)).astype(np.float32)
    if ties:  # gold scores come in steps (STS scores are multiples of 0.2)
        y = np.round(y * 5) / 5
        x[: n // 4] = x[n // 4: 2 * (n // 4)]
    got = bbh.spearman(x, y)
    ref = spearmanr(x.astype(np.float64), y.astype(np.float64)).statistic
    assert abs(got - ref) < 1e-12


def test_spearman_edges():
    import bbh

    assert np.isnan(bbh.spearman(np.ones(5), np.arange(5)))  # a constant input has no ranking
    assert bbh.spearman([1, 2, 3], [3, 2, 1]) == pytest.approx(-1.0)
    with pytest.raises(bbh.BBHError):
        bbh.spearman([1.0], [2.0])
    with pytest.raises(bbh.BBHError):
        bbh.spearman([1.0, np.nan, 2.0], [1.0, 2.0, 3.0])
