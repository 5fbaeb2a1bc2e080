"""Distribution tests of the stochastic sampler (host fp64 path, which the
device sampler is replay-tested against): over many counter-addressed draws
the empirical token frequencies match the intended distribution
(temperature softmax restricted by top-k and top-p, renormalised), by a
chi-square goodness-of-fit test; tokens outside the support never appear."""
import math

import numpy as np
import pytest
from scipy import stats

from lunaflux_b200.sampling.host import counter_unit, stochastic_sample


def intended(logits, temperature, top_k, top_p):
    order = sorted(range(len(logits)), key=lambda i: (-logits[i], i))
    if top_k:
        order = order[:top_k]
    z = np.array([logits[i] / temperature for i in order], dtype=np.float64)
    p = np.exp(z - z.max())
    p /= p.sum()
    if top_p is not None and top_p < 1.0:
        keep, run = [], 0.0
        for i, q in zip(order, p):
            keep.append((i, q))
            run += q
            if run >= top_p:
                break
        tot = sum(q for _, q in keep)
        return {i: q / tot for i, q in keep}
    return {i: q for i, q in zip(order, p)}


@pytest.mark.parametrize("temperature,top_k,top_p", [(1.0, None, None), (0.7, None, 0.9), (1.3, 5, None),
                                                     (0.5, 8, 0.8)])
def test_sampler_matches_intended_distribution(temperature, top_k, top_p):
    rng = np.random.default_rng(11)
    logits = list(rng.normal(0, 1.5, 24))
    want = intended(logits, temperature, top_k, top_p)
    n = 20000
    counts = {}
    for k in range(n):
        t = stochastic_sample(logits, temperature, top_k, top_p, counter_unit(1234, k))
        counts[t] = counts.get(t, 0) + 1
    assert set(counts) <= set(want)                       # nothing outside top-k / top-p support
    ids = sorted(want)
    obs = np.array([counts.get(i, 0) for i in ids], dtype=np.float64)
    exp = np.array([want[i] * n for i in ids])
    # pool cells with small expectations (chi-square needs >= 5 per cell)
    small = exp < 5
    if small.any():
        obs = np.append(obs[~small], obs[small].sum())
        exp = np.append(exp[~small], exp[small].sum())
    chi2, p = stats.chisquare(obs, exp)
    assert p > 1e-3, (chi2, p)


def test_counter_units_are_uniform():
    u = np.array([counter_unit(7, k) for k in range(50000)])
    assert 0.0 <= u.min() and u.max() < 1.0
    hist, _ = np.histogram(u, bins=20, range=(0, 1))
    assert stats.chisquare(hist).pvalue > 1e-3
    assert abs(np.corrcoef(u[:-1], u[1:])[0, 1]) < 0.02     # successive draws uncorrelated
