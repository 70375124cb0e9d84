"""The mirror front-end builds the reference's graphs node for node.

When the reference checkout is available, its own builders and the mirror's
are run side by side and their ``GraphPlan.signature``s compared with and
without the lowerings the plugin uses; elsewhere these tests are skipped and
the host-logic tests still run.
"""

from __future__ import annotations

import sys

import numpy as np
import pytest

from conftest import REFERENCE
from cuda_b200.frontend import lazy as ML
from cuda_b200.frontend import llama as L
from cuda_b200.frontend.tensor import Tensor, compile_graph
from cuda_b200.generation import verify_greedy_candidates
from cuda_b200.models import WORKLOADS, synthetic_prompt, synthetic_weights


@pytest.fixture(scope="module")
def ref():
    if not (REFERENCE / "chomikgrad" / "lazy.py").exists():
        pytest.skip("reference checkout not present on this machine")
    sys.dont_write_bytecode = True
    sys.path.insert(0, str(REFERENCE))
    import chomikgrad

    return chomikgrad


LOWERINGS = [(), ("rms_norm", "rope", "sdpa", "softmax")]


def _graphs(module, T, lib, cfg, dt, weights):
    S, ctx = 7, 12
    ids = synthetic_prompt(cfg, S)
    pre = lib.LlamaForCausalLM(cfg, weights, sequence_length=S, dtype=dt, cache_length=ctx).prefill(
        T(ids, copy=False), T(lib.position_selector(S - 1, S, dtype=dt)))
    caches = [T.from_native(np.zeros((1, cfg.num_key_value_heads, ctx, cfg.head_size), np.float32),
                            backend="cpu", shape=(1, cfg.num_key_value_heads, ctx, cfg.head_size), dtype=dt)
              for _ in range(2 * cfg.num_hidden_layers)]
    am, wm = L.decode_masks(5, ctx, dt)
    step = lib.LlamaDecoderStep(cfg, weights, cache_length=ctx, dtype=dt)
    dec = step(T(np.array([[3]], np.int32), copy=False),
               T(L.rope_rotations(1, cfg.head_size, cfg.rope_theta, dt, offset=5), copy=False),
               T(am, copy=False), T(wm, copy=False), list(zip(caches[::2], caches[1::2])),
               position=T(np.asarray(5, np.int32), copy=False))
    return pre, dec


@pytest.mark.parametrize("name", ["tiny-fp32", "tiny-bf16"])
def test_llama_graphs_equal_reference_signatures(ref, name):
    wl = WORKLOADS[name]
    raw = synthetic_weights(wl.config, dtype=wl.np_dtype)
    rcfg = ref.llama.LlamaConfig(**{k: getattr(wl.config, k) for k in (
        "vocab_size", "hidden_size", "intermediate_size", "num_hidden_layers", "num_attention_heads",
        "num_key_value_heads", "max_position_embeddings")})
    theirs = _graphs(ref, ref.Tensor, ref.llama, rcfg, wl.np_dtype,
                     {n: ref.Tensor(v) for n, v in raw.items()})
    mine = _graphs(ML, Tensor, L, wl.config, wl.np_dtype, {n: Tensor(v) for n, v in raw.items()})
    for a, b in zip(theirs, mine):
        for lowerings in LOWERINGS:
            assert (ref.lazy.GraphPlan([t._node for t in a], lowerings).signature()
                    == ML.GraphPlan([t._node for t in b], lowerings).signature())


def test_plugin_installs_into_reference_registry(ref):
    import cuda_b200

    cuda_b200.install(ref)
    assert "cuda-b200" in ref.lazy._COMPILERS


def test_registry_contract():
    with pytest.raises(ValueError):
        ML.register_compiler("", lambda: None)
    with pytest.raises(KeyError):
        ML.get_compiler("no-such-compiler")
    with pytest.raises(ValueError):
        compile_graph()


def test_rope_rotation_matches_rotate_half():
    """Known answer of test_llama.py:38-55."""
    value = np.arange(8, dtype=np.float32).reshape(1, 1, 1, 8)
    rotation = L.rope_rotations(2, 8, 10_000.0, np.dtype(np.float32))
    angle = 1 / (10_000.0 ** (np.arange(0, 8, 2) / 8))
    c, s = np.cos(angle), np.sin(angle)
    v = value.reshape(8)
    expected = np.concatenate([v[:4] * c - v[4:] * s, v[4:] * c + v[:4] * s])
    actual = value.reshape(1, 1, 1, 1, 8) @ rotation[:, :, 1:2]
    np.testing.assert_allclose(actual.reshape(8), expected, rtol=1e-6, atol=1e-6)


def test_config_validation():
    with pytest.raises(ValueError, match="divisible by KV heads"):
        L.LlamaConfig(vocab_size=10, hidden_size=24, intermediate_size=48, num_hidden_layers=1,
                      num_attention_heads=6, num_key_value_heads=4, max_position_embeddings=16).validate()
    with pytest.raises(ValueError, match="missing Llama config"):
        L.LlamaConfig.from_dict({"vocab_size": 1})


def test_greedy_verification():
    assert verify_greedy_candidates([3, 4, 5], [3, 4, 5]).accepted_draft_tokens == 3
    r = verify_greedy_candidates([3, 9, 5], [3, 4, 7])
    assert r.emitted_tokens == (3, 4) and r.accepted_draft_tokens == 1
    with pytest.raises(ValueError):
        verify_greedy_candidates([], [])
