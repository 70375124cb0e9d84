"""Temperature / top-k sampling on the host side (no GPU).

The reference samples with ``sample_token`` (examples/generate_tinyllama.py
:124-143).  ``tests/golden/sampling.npz`` holds the tokens the reference's own
function returned for seeded logit rows, settings and seeds, and
``tiny_fp32_sampled.npz`` a whole sampled generation through the reference's
loop (``sample_native_token`` with ``default_rng(seed)``, :146-157, :712).
These pin the oracle's restatement, the one-draw decomposition of
``Generator.choice`` that the device sampler (cb_sample_rows) is built on,
and the runtime's use of the generator.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden
from oracle import sampling


def test_oracle_sampler_matches_the_reference_tokens():
    g = golden("sampling")
    for r, row in enumerate(g["rows"]):
        for s, (temperature, top_k) in enumerate(g["settings"]):
            for j, seed in enumerate(g["seeds"]):
                got = sampling.sample_token(row[None], temperature=float(temperature), top_k=int(top_k),
                                            rng=np.random.default_rng(int(seed)))
                assert got == g["tokens"][r, s, j], (r, s, j)


def test_one_draw_decomposition_matches_the_reference_tokens():
    """token == searchsorted(cdf, u) for the single u = rng.random() Generator.choice takes."""
    g = golden("sampling")
    for r, row in enumerate(g["rows"]):
        for s, (temperature, top_k) in enumerate(g["settings"]):
            for j, seed in enumerate(g["seeds"]):
                u = np.random.default_rng(int(seed)).random()
                got = sampling.sample_with_draw(row, u, temperature=float(temperature), top_k=int(top_k))
                assert got == g["tokens"][r, s, j], (r, s, j)


def test_choice_consumes_exactly_one_draw():
    rng = np.random.default_rng(5)
    for _ in range(300):
        width = int(rng.integers(1, 400))
        row = rng.normal(0, 2, width).astype(np.float32)
        seed = int(rng.integers(0, 1 << 31))
        ref_rng, dev_rng = np.random.default_rng(seed), np.random.default_rng(seed)
        k = int(rng.integers(0, width + 2))
        want = sampling.sample_token(row[None], temperature=0.9, top_k=k, rng=ref_rng)
        got = sampling.sample_with_draw(row, dev_rng.random(), temperature=0.9, top_k=k)
        assert got == want
        assert ref_rng.random() == dev_rng.random()  # both generators advanced alike


def test_runtime_sampling_on_the_oracle_matches_the_reference_loop(oracle):
    """LlamaRuntime.generate(temperature, top_k, seed) drives the generator like the reference loop."""
    from cuda_b200.models import WORKLOADS, synthetic_weights
    from cuda_b200.runtime import LlamaRuntime

    g = golden("tiny_fp32_sampled")
    wl = WORKLOADS["tiny-fp32"]
    rt = LlamaRuntime(wl.config, synthetic_weights(wl.config, dtype=wl.np_dtype), compiler="cpu")
    result = rt.generate(list(g["prompt"]), len(g["tokens"]), temperature=0.8, top_k=40, seed=3)
    assert result.tokens == [int(t) for t in g["tokens"]]
    with pytest.raises(ValueError):
        rt.generate(list(g["prompt"]), 2, temperature=-1.0)
