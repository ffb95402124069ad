"""The oracle's sampler (test infrastructure): the restatement of the
reference's llm_sample used to check the device sampler."""
import numpy as np


def test_oracle_sampler_recipe(oracle):
    """llm_sample restated (llm.c:1143-1246): the greedy limit is llm_argmax,
    draws follow the top-40 / nucleus-0.9 distribution, ties keep the lower
    index, fewer than 40 candidates work"""
    rng = np.random.default_rng(2)
    x = rng.normal(0, 2, 1000).astype(np.float32)
    assert oracle.sample(x, 0.001, 123) == oracle.argmax(x)
    # the distribution: top-40 by value, softmax with llm_expf, cut at 0.9
    order = sorted(range(len(x)), key=lambda i: (-x[i], i))[:40]
    e = np.array([oracle.expf(np.float32(x[i] - x[order[0]]) / np.float32(0.8)) for i in order], np.float64)
    p = e / e.sum()
    cut = int(np.searchsorted(np.cumsum(p), 0.9) + 1)
    p = p[:cut] / p[:cut].sum()
    draws = [oracle.sample(x, 0.8, int(w)) for w in rng.integers(0, 2**32, 20000)]
    assert set(draws) <= set(order[:cut])
    freq = np.array([draws.count(i) for i in order[:cut]]) / len(draws)
    assert np.max(np.abs(freq - p)) < 0.02
    y = np.full(50, 1.0, np.float32)
    assert oracle.sample(y, 0.001, 7) == 0
    assert oracle.sample(rng.normal(0, 1, 5).astype(np.float32), 1.0, 99) in range(5)
