"""CPU restatement of the token sampler (test infrastructure only).

Checks ``mk_sample`` (csrc/mk_sample.cuh). The knobs are the reference's
per-sequence generation parameters (top_k, top_p, temperature; main.py:57-61,
prepare_sampling_params main.py:197-205); the reference samples through
NxDI's on-device sampler (main.py:129-130), which is not in the reference
sources, so this follows the published order of those operations: logits /
temperature, top_k largest (ties: lowest index), softmax, the smallest prefix
reaching top_p, one draw. The uniform is the same 24-bit splitmix64 hash the
kernel uses, so draws agree except when the uniform falls within rounding of a
prefix boundary (the kernel sums fp32, this sums fp64).
"""
from __future__ import annotations

import numpy as np

M64 = (1 << 64) - 1
MAX_K = 1024


def splitmix64(x: int) -> int:
    x = (x + 0x9E3779B97F4A7C15) & M64
    x = ((x ^ (x >> 30)) * 0xBF58476D1CE4E5B9) & M64
    x = ((x ^ (x >> 27)) * 0x94D049BB133111EB) & M64
    return x ^ (x >> 31)


def uniform(seed: int, step: int, seq: int) -> float:
    h = splitmix64((seed ^ splitmix64((step * 0xD1B54A32D192ED03 + seq) & M64)) & M64)
    return float(np.float32(h >> 40) * np.float32(1.0 / 16777216.0))


def sample(logits: np.ndarray, top_k: int, top_p: float, temperature: float, seed: int, step: int,
           seq: int) -> int:
    v = np.asarray(logits, dtype=np.float32)
    V = v.shape[0]
    order = np.lexsort((np.arange(V), -v.astype(np.float64)))  # logit desc, index asc
    if top_k == 1 or not temperature > 0:
        return int(order[0])
    k = MAX_K if top_k <= 0 or top_k > MAX_K else top_k
    k = min(k, V)
    idx = order[:k]
    x = (v[idx].astype(np.float64) - float(v[idx[0]])) / float(np.float32(temperature))
    cum = np.cumsum(np.exp(x))
    m = k
    if top_p < 1.0:
        cut = float(np.float32(top_p)) * cum[-1]
        m = int(np.searchsorted(cum, cut, side="left")) + 1
        m = min(max(m, 1), k)
    r = uniform(seed, step, seq) * cum[m - 1]
    j = int(np.searchsorted(cum[:m], r, side="right"))
    return int(idx[min(j, m - 1)])
