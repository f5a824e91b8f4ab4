"""The oracle's sampler against the reference's own sample.zig tests, and the
random stream's structure (test infrastructure for the device sampler)."""
from __future__ import annotations

import numpy as np
import pytest


def test_greedy_returns_argmax(oracle):  # sample.zig "greedy: returns argmax"
    assert oracle.greedy([0.1, 5.0, 2.0, 3.0]) == 1


def test_temperature_zero_is_greedy(oracle):  # "sample: temperature=0 behaves like greedy"
    assert oracle.sample([1.0, 3.0, 2.0], 0.0, 0, 1.0, oracle.Rng(42)) == 1


def test_stays_within_vocab(oracle):  # "sample: stays within vocab range"
    logits = np.arange(100, dtype=np.float32)
    assert 0 <= oracle.sample(logits, 1.0, 10, 1.0, oracle.Rng(0)) < 100


def test_top_p_zero_picks_top(oracle):  # "sample: top_p=0.0 always picks highest-prob token"
    assert oracle.sample([0.5, 2.0, 0.1], 1.0, 0, 0.0, oracle.Rng(7)) == 1


def test_fast_top_k_matches_full_filtering(oracle):
    """sample.zig "fast top-k path matches full filtering semantics": the
    fast path against softmax + top-k + top-p + renormalise + draw written
    out here, with the same seed."""
    base = np.array([0.2, 2.0, -1.0, 1.5, 0.7, 3.0, 2.5, -0.3], np.float32)
    temp, k, tp = 0.7, 4, 0.8
    fast = oracle.sample(base, temp, k, tp, oracle.Rng(99))
    ref = (base * np.float32(np.float32(1.0) / np.float32(temp))).astype(np.float32)
    ref = np.exp(ref - ref.max()).astype(np.float32)
    ref = (ref / ref.sum(dtype=np.float32)).astype(np.float32)
    thr = np.sort(ref)[::-1][k - 1]
    ref[ref < thr] = 0
    order = np.argsort(-ref, kind="stable")
    cum, cut = np.float32(0), False
    for i in order:
        if cut:
            ref[i] = 0
        else:
            cum = np.float32(cum + ref[i])
            cut = cum >= tp
    ref = (ref * (np.float32(1) / ref.sum(dtype=np.float32))).astype(np.float32)
    r = oracle.Rng(99).float()
    c, tok = np.float32(0), len(ref) - 1
    for i, p in enumerate(ref):
        c = np.float32(c + p)
        if r <= c:
            tok = i
            break
    assert fast == tok


def test_rng_float_range_and_stream(oracle, pkg):
    """Random.float(f32) lies in [0, 1) and is a function of the seed; the
    C ABI's seeding equals the oracle's."""
    a, b = oracle.Rng(5), oracle.Rng(5)
    xs = [a.float() for _ in range(1000)]
    assert all(0.0 <= x < 1.0 for x in xs)
    assert xs == [b.float() for _ in range(1000)]
    assert abs(np.mean(xs) - 0.5) < 0.05
    assert pkg.rng_seed(12345) == oracle.Rng(12345).words()


@pytest.mark.parametrize("k,tp", [(40, 0.9), (0, 1.0), (0, 0.5), (300, 1.0)])
def test_sample_distribution(oracle, k, tp):
    """Draws follow the filtered distribution (chi-square-free sanity: the
    most likely token is drawn most often; excluded tokens never)."""
    rng = np.random.default_rng(1)
    logits = rng.normal(0, 2, 500).astype(np.float32)
    r = oracle.Rng(3)
    draws = [oracle.sample(logits, 1.0, k, tp, r) for _ in range(400)]
    if k:
        allowed = set(np.argsort(-logits, kind="stable")[:k].tolist())
        assert set(draws) <= allowed
    assert max(set(draws), key=draws.count) in np.argsort(-logits)[:5]
