"""The sampler's rule (src/sampler.rs:28-73) in float64, for the sampler tests.

The device sampler holds each probability as an exact 64-bit fixed-point
mass (2^-50 resolution) and sums them as integers, so its pick is the pick
of this float64 restatement except where the draw lies within ~1e-9 of a
cumulative boundary. The oracle follows the reference's f32 arithmetic
(sequential sums, normalise, cumulative `>= top_p`, renormalise,
WeightedIndex), whose rounding can move a boundary by up to a few ulps of
the running sum per element; `ref_eps(n)` bounds that drift in normalised
mass. `candidates(..., eps)` is the set of tokens the rule can pick when
every cumulative boundary may move by eps: with eps = DEVICE_EPS it must
contain the device's pick, with eps = ref_eps(n) the oracle's. A device /
oracle disagreement is therefore confined to draws near a boundary, and the
tests count those draws instead of allowing a blanket number of misses.
"""
from __future__ import annotations

import numpy as np

DEVICE_EPS = 1e-9


def ref_eps(n: int) -> float:
    """Drift of an f32 running sum of n positive terms that total 1: each
    addition rounds by at most half an ulp of a partial sum <= 1 (2^-25);
    eight standard deviations of that random walk."""
    return 8.0 * np.sqrt(n) * 2.0 ** -25 + 1e-7


def probabilities(logits, temperature):
    """p_i = exp(z_i / T) with the division in f32 and the exponential rounded
    once to f32 (sampler.rs:34-38: no max subtraction)."""
    z = np.asarray(logits, np.float32)
    q = (z / np.float32(temperature)).astype(np.float32)
    return np.exp(q.astype(np.float64)).astype(np.float32)


def candidates(logits, temperature, top_k, top_p, u, eps):
    n = len(logits)
    if temperature == 0.0:
        z = np.asarray(logits, np.float32)
        return {int(n - 1 - np.argmax(z[::-1]))}  # last index on ties
    p32 = probabilities(logits, temperature)
    p = p32.astype(np.float64)
    w = p / p.sum()
    filt = top_k > 0 or top_p < 1.0
    order = np.argsort(-p32, kind="stable") if filt else np.arange(n)
    if top_k > 0:
        order = order[:top_k]
    L = len(order)
    cuts = [L]
    if top_p < 1.0:
        c = np.cumsum(w[order])
        lo = min(int(np.searchsorted(c, top_p - eps, side="left")) + 1, L)
        hi = min(int(np.searchsorted(c, top_p + eps, side="left")) + 1, L)
        cuts = list(range(max(lo, 1), hi + 1))
        if len(cuts) > 256:  # a flat tail: the ends and a sample between them
            cuts = sorted(set(cuts[:: len(cuts) // 128]) | {cuts[0], cuts[-1]})
    out = set()
    for cut in cuts:
        kept = order[:cut]
        cw = np.cumsum(w[kept])
        cw = cw / cw[-1]
        # WeightedIndex: the first candidate whose cumulative weight exceeds u
        a = min(int(np.searchsorted(cw, u - eps, side="right")), cut - 1)
        b = min(int(np.searchsorted(cw, u + eps, side="right")), cut - 1)
        out.update(int(t) for t in kept[a:b + 1])
    return out
