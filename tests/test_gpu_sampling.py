"""cb_sample_rows (device temperature / top-k sampling) against the reference's sampler.

Bars: the token equals the reference's for the same generator state -- the
golden tokens of the reference's own ``sample_token`` and sampled generation
loop, and the oracle's one-draw form (``oracle.sampling.sample_with_draw``,
ties at the k-th value lowest-index first) on wide rows.  The float64 sums
run in another order than NumPy's, so a token could differ only when the
draw falls within a few ulps of a cdf boundary; none of these cases does.
"""

from __future__ import annotations

import ml_dtypes
import numpy as np
import pytest

from conftest import golden
from oracle import sampling

pytestmark = pytest.mark.gpu


def test_device_sampler_matches_the_reference_tokens(gpu):
    g = golden("sampling")
    dev = gpu.device
    for r, row in enumerate(g["rows"]):
        native = dev.array(row[None].copy())
        for s, (temperature, top_k) in enumerate(g["settings"]):
            for j, seed in enumerate(g["seeds"]):
                rng = np.random.default_rng(int(seed))
                got = dev.sample(native, temperature=float(temperature), top_k=int(top_k), rng=rng)
                assert got == g["tokens"][r, s, j], (r, s, j)


@pytest.mark.parametrize("width", [1, 7, 1000, 32000, 128256])
@pytest.mark.parametrize("dtype", [np.float32, ml_dtypes.bfloat16, np.float16])
def test_device_sampler_matches_the_one_draw_oracle(gpu, width, dtype):
    """Wide rows (TinyLlama's and Llama-3's vocabularies), low-precision logits, every top-k regime."""
    dev = gpu.device
    rng = np.random.default_rng(width)
    row = (rng.normal(0, 2.5, width)).astype(dtype)
    exact = row.astype(np.float32)
    native = dev.array(row[None].copy())
    for temperature, top_k in ((1.0, 0), (0.7, 50), (1.3, 1), (0.9, width - 1), (1.0, width), (2.0, width + 5)):
        for seed in range(12):
            draws = np.random.default_rng(seed)
            got = dev.sample(native, temperature=temperature, top_k=top_k, rng=draws)
            want = sampling.sample_with_draw(exact, np.random.default_rng(seed).random(),
                                             temperature=temperature, top_k=top_k)
            assert got == want, (temperature, top_k, seed)


def test_ties_and_masked_logits(gpu):
    """Many equal values at the k-th largest (lowest indices kept) and -inf entries (probability 0)."""
    dev = gpu.device
    rng = np.random.default_rng(3)
    row = rng.integers(-3, 4, 5000).astype(np.float32)  # 7 distinct values, ~700 copies each
    row[rng.permutation(5000)[:1500]] = -np.inf
    native = dev.array(row[None].copy())
    for top_k in (1, 10, 700, 1000, 3499, 3500, 4000):
        for seed in range(16):
            got = dev.sample(native, temperature=0.8, top_k=top_k, rng=np.random.default_rng(seed))
            want = sampling.sample_with_draw(row, np.random.default_rng(seed).random(), temperature=0.8,
                                             top_k=top_k)
            assert got == want, (top_k, seed)
            assert np.isfinite(row[got])


def test_rows_draw_in_row_order(gpu):
    """sample_rows: row i takes the i-th draw, like calling the reference's sampler row by row."""
    dev = gpu.device
    rng = np.random.default_rng(8)
    rows = rng.normal(0, 2, (5, 32000)).astype(np.float32)
    got = dev.sample_rows(dev.array(rows), temperature=1.0, top_k=50, rng=np.random.default_rng(4))
    ref_rng = np.random.default_rng(4)
    want = [sampling.sample_token(rows[i:i + 1], temperature=1.0, top_k=50, rng=ref_rng) for i in range(5)]
    assert list(got) == want


def test_nan_probabilities_raise_like_numpy(gpu):
    dev = gpu.device
    row = np.zeros((1, 64), np.float32)
    row[0, 9] = np.nan
    with pytest.raises(ValueError):
        dev.sample(dev.array(row), temperature=1.0, top_k=0, rng=np.random.default_rng(0))
    with pytest.raises(ValueError):
        dev.sample(dev.array(np.full((1, 64), -np.inf, np.float32)), temperature=1.0, top_k=0,
                   rng=np.random.default_rng(0))
    with pytest.raises(ValueError):
        dev.sample(dev.array(np.zeros((1, 4), np.float32)), temperature=-1.0, top_k=0, rng=np.random.default_rng(0))
    # the device is fine afterwards
    ok = np.zeros((1, 64), np.float32)
    ok[0, 5] = 50.0
    assert dev.sample(dev.array(ok), temperature=1.0, top_k=0, rng=np.random.default_rng(0)) == 5


def test_sampled_generation_matches_the_reference_loop(gpu):
    """The reference's loop sampling with default_rng(3), temperature 0.8, top-k 40 (golden)."""
    from cuda_b200.models import WORKLOADS, synthetic_weights
    from cuda_b200.runtime import LlamaRuntime

    g = golden("tiny_fp32_sampled")
    wl = WORKLOADS["tiny-fp32"]
    rt = LlamaRuntime(wl.config, synthetic_weights(wl.config, dtype=wl.np_dtype), compiler="cuda-b200")
    result = rt.generate(list(g["prompt"]), len(g["tokens"]), temperature=0.8, top_k=40, seed=3)
    assert result.tokens == [int(t) for t in g["tokens"]]


def test_batched_top1_sampling_is_greedy(gpu):
    from cuda_b200.batched import BatchedRuntime
    from cuda_b200.models import WORKLOADS, synthetic_prompt, synthetic_weights

    wl = WORKLOADS["tiny-bf16"]
    rt = BatchedRuntime(wl.config, synthetic_weights(wl.config, dtype=wl.np_dtype), batch=3)
    prompts = [list(synthetic_prompt(wl.config, 12, seed=s)[0]) for s in range(3)]
    greedy = rt.generate_batch(prompts, 10)
    assert rt.generate_batch(prompts, 10, temperature=0.5, top_k=1, seed=9) == greedy
