"""The sampling restatement (oracle/sampling.py) on the CPU: its noise is
standard Gumbel and its draws follow softmax(logits / T)."""

import numpy as np

from oracle.sampling import gumbel, sample, uniform24


def test_uniform_in_open_interval_and_uniform():
    u = uniform24(1234, 77, np.arange(200_000))
    assert u.dtype == np.float32
    assert u.min() > 0.0 and u.max() < 1.0
    hist, _ = np.histogram(u, bins=20, range=(0.0, 1.0))
    assert np.abs(hist / len(u) - 0.05).max() < 0.003


def test_gumbel_moments():
    g = gumbel(7, 1023, np.arange(400_000))
    assert abs(g.mean() - 0.5772156649) < 0.01  # Euler-Mascheroni constant
    assert abs(g.var() - np.pi**2 / 6) < 0.03


def test_noise_depends_on_seed_position_index():
    a = gumbel(1, 5, np.arange(1000))
    assert not np.allclose(a, gumbel(2, 5, np.arange(1000)))
    assert not np.allclose(a, gumbel(1, 6, np.arange(1000)))
    assert np.array_equal(a, gumbel(1, 5, np.arange(1000)))


def test_draws_follow_softmax():
    """Gumbel-max over many positions reproduces softmax(logits / T)."""
    logits = np.array([1.0, 0.5, 0.0, -1.0, 2.0], dtype=np.float32)
    T = 0.7
    p = np.exp(logits / T) / np.exp(logits / T).sum()
    n = 40_000
    counts = np.zeros(len(logits))
    for pos in range(n):
        counts[sample(logits, T, seed=99, position=pos)[0]] += 1
    assert np.abs(counts / n - p).max() < 0.01


def test_top_k_draws_follow_renormalized_softmax():
    logits = np.array([1.0, 0.5, 0.0, -1.0, 2.0, 1.5], dtype=np.float32)
    T, k = 0.9, 3
    top = np.argsort(-logits)[:k]
    p = np.zeros(len(logits))
    p[top] = np.exp(logits[top] / T) / np.exp(logits[top] / T).sum()
    n = 30_000
    counts = np.zeros(len(logits))
    for pos in range(n):
        counts[sample(logits, T, seed=7, position=pos, top_k=k)[0]] += 1
    assert counts[np.setdiff1d(np.arange(len(logits)), top)].sum() == 0
    assert np.abs(counts / n - p).max() < 0.012


def test_top_1_is_greedy():
    logits = np.random.default_rng(3).standard_normal(5000).astype(np.float32)
    for pos in range(50):
        assert sample(logits, 1.3, seed=11, position=pos, top_k=1)[0] == int(np.argmax(logits))
