"""PARITY ORACLE -- test infrastructure, not product code.

The reference's host sampler restated: ``sample_token``
(examples/generate_tinyllama.py:124-143), plus the decomposition of NumPy's
``Generator.choice(V, p=p)`` that the device sampler relies on: one
``u = rng.random()`` draw, then ``cdf.searchsorted(u, side="right")`` with
``cdf = cumsum(p) / cumsum(p)[-1]`` (NumPy's published algorithm for
``choice`` with probabilities; ``tests/test_sampling.py`` checks that the two
agree and leave the generator in the same state).

Only ``tests/`` may import this module; ``cuda_b200`` never does.
"""

from __future__ import annotations

import numpy as np


def sample_token(logits: np.ndarray, *, temperature: float, top_k: int, rng: np.random.Generator) -> int:
    """generate_tinyllama.py:124-143: temperature, top-k filter, softmax, ``rng.choice``."""
    values = np.asarray(logits[0], dtype=np.float64)
    if temperature == 0:
        return int(values.argmax())
    values /= temperature
    if top_k > 0 and top_k < values.size:
        indexes = np.argpartition(values, -top_k)[-top_k:]
        filtered = np.full_like(values, -np.inf)
        filtered[indexes] = values[indexes]
        values = filtered
    values -= np.max(values)
    probabilities = np.exp(values)
    probabilities /= probabilities.sum()
    return int(rng.choice(values.size, p=probabilities))


def probabilities(row: np.ndarray, *, temperature: float, top_k: int) -> np.ndarray:
    """The float64 p of ``sample_token`` for one row, with ties at the k-th value kept lowest-index first."""
    values = np.asarray(row, dtype=np.float64) / temperature
    if top_k > 0 and top_k < values.size:
        order = np.lexsort((np.arange(values.size), -values))  # descending value, then ascending index
        keep = np.zeros(values.size, bool)
        keep[order[:top_k]] = True
        values = np.where(keep, values, -np.inf)
    values = values - np.max(values)
    p = np.exp(values)
    return p / p.sum()


def sample_with_draw(row: np.ndarray, u: float, *, temperature: float, top_k: int) -> int:
    """The token ``sample_token`` returns when ``rng.random()`` yields ``u`` (ties lowest-index first)."""
    p = probabilities(row, temperature=temperature, top_k=top_k)
    cdf = np.cumsum(p)
    cdf /= cdf[-1]
    return int(cdf.searchsorted(u, side="right"))
