"""CPU restatement of the reference's sampling -- TEST INFRASTRUCTURE ONLY.

hetero/backends.py:106-120 (NumpyBackend.sample): temperature 0 is numpy's
argmax; otherwise z = logits / T, z -= max, p = exp(z), p /= sum, an
optional top-p mask over the probabilities sorted in descending order (an
element is kept when the mass before it is below top_p), renormalised, and
one draw of rng.choice(len(p), p=p).  The draw is restated with the uniform
variate taken outside: choice's cumulative distribution (float32 cumsum,
divided by its last entry) searched for u = rng.random() (side "right").
tests/test_sample.py pins this against the reference's own sample() on the
same seeded generators; the device sampler (hq4_sample) is checked against
it with the same u.
"""
from __future__ import annotations

import numpy as np


def probabilities(logits, temperature: float, top_p: float) -> np.ndarray:
    """The distribution the reference draws from (backends.py:113-119)."""
    z = np.asarray(logits, dtype=np.float32).reshape(-1)
    z = z / temperature
    z -= z.max()
    p = np.exp(z)
    p /= p.sum()
    if top_p < 1.0:
        order = np.argsort(-p)
        keep = np.cumsum(p[order]) - p[order] < top_p
        masked = np.zeros_like(p)
        masked[order[keep]] = p[order[keep]]
        p = masked / masked.sum()
    return p


def draw(p: np.ndarray, u: float) -> int:
    """rng.choice(len(p), p=p) for the uniform variate u."""
    cdf = p.cumsum()
    cdf /= cdf[-1]
    return int(cdf.searchsorted(u, side="right"))


def sample_with_u(logits, temperature: float, top_p: float, u: float) -> int:
    if temperature <= 0:
        return int(np.asarray(logits, dtype=np.float32).reshape(-1).argmax())
    return draw(probabilities(logits, temperature, top_p), u)
