"""The CPU sampler restatement (oracle/sampling.py) on its own.

The kernel (``mk_sample``) is checked against it on the GPU
(tests/test_gpu_sampling.py); here the restatement is pinned to the
definitions it states: greedy cases are the lowest-index argmax, the uniform
is a fixed function of (seed, step, sequence), a top_p that the first token
alone reaches is greedy, and over many draws the frequencies follow the
tempered softmax restricted to the top_k.
"""
from __future__ import annotations

import numpy as np

from oracle import sampling as S


def test_uniform_is_a_fixed_hash():
    u = [S.uniform(7, s, q) for s in range(50) for q in range(4)]
    assert all(0.0 <= x < 1.0 for x in u)
    assert u == [S.uniform(7, s, q) for s in range(50) for q in range(4)]
    assert len(set(u)) == len(u)
    assert all((x * 2**24).is_integer() for x in u)  # 24-bit values


def test_greedy_cases_are_the_lowest_index_argmax():
    v = np.array([0.5, 2.0, -1.0, 2.0, 1.9], dtype=np.float32)
    for k, t in ((1, 1.0), (50, 0.0), (1, 0.0)):
        assert S.sample(v, k, 1.0, t, 3, 0, 0) == 1
    # a top_p the largest probability alone reaches
    assert S.sample(np.array([10.0, 0.0, 0.0], dtype=np.float32), 3, 0.5, 1.0, 1, 2, 0) == 0


def test_frequencies_follow_the_truncated_softmax():
    rng = np.random.default_rng(1)
    v = rng.standard_normal(64).astype(np.float32)
    k, t = 8, 0.7
    top = np.argsort(-v, kind="stable")[:k]
    p = np.exp((v[top] - v[top[0]]) / t)
    p /= p.sum()
    n = 20000
    draws = [S.sample(v, k, 1.0, t, 11, s, 0) for s in range(n)]
    counts = np.array([draws.count(int(i)) for i in top]) / n
    assert set(draws) <= set(int(i) for i in top)
    assert np.abs(counts - p).max() < 0.015


def test_top_p_keeps_the_smallest_prefix():
    v = np.log(np.array([0.5, 0.3, 0.15, 0.05], dtype=np.float32))
    draws = {S.sample(v, 4, 0.79, 1.0, 5, s, 0) for s in range(2000)}
    assert draws == {0, 1}  # 0.5 + 0.3 reaches 0.79, 0.5 alone does not
