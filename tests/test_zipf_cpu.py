"""The skewed-routing workload (128-token speculative verify, Zipf(1.1)
expert popularity): the stored bias strength is what the bisection finds, and
at that strength the top-8 selection of seeded tokens fits Zipf(1.1)."""

import numpy as np

from mlxlr8_b200 import synthetic


def test_stored_gamma_is_the_calibrated_one():
    gamma = synthetic.calibrate_zipf_gamma()
    assert abs(gamma - synthetic.ZIPF_GAMMA) < 2e-5, gamma


def test_selection_fits_zipf_at_the_stored_gamma():
    logits = synthetic._zipf_logits(synthetic.ZIPF_SEED + 7, 50_000)
    rank = np.random.default_rng(3).permutation(256).astype(np.float64)
    bias = -synthetic.ZIPF_GAMMA * synthetic.ZIPF_S * np.log(rank + 1.0)
    slope, freq = synthetic.zipf_selection_slope(logits, bias, rank)
    assert abs(slope + synthetic.ZIPF_S) < 0.03, slope
    assert abs(freq.sum() - 8.0) < 1e-9
    by_rank = freq[np.argsort(rank)]
    assert by_rank[0] > 5 * by_rank[-1]  # the head is far more popular than the tail
