"""cb_sdpa_tc (tcgen05 flash attention) against a float64 reference and cb_sdpa.

out = softmax(q k^T / divisor + mask) v over grouped-query heads
(chomikgrad/llama.py:332-369).  q, k, v enter as float32 and are split into
bf16 hi/lo planes: every product keeps about 2^-16 of its magnitude, so the
bound below is 2e-4 of max|v| (float32 softmax and accumulation included).
"""

from __future__ import annotations

import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _args(torch, q, k, v, mask, out, divisor):
    from cuda_b200 import _lib

    a = _lib.SdpaArgs()
    for name, t in (("q", q), ("k", k), ("v", v), ("mask", mask)):
        setattr(a, name, t.data_ptr())
        setattr(a, f"{name}_dtype", _lib.F32 if t.dtype == torch.float32 else _lib.BF16)
        strides = getattr(a, f"{name}_strides")
        for d in range(4):
            strides[d] = 0 if t.shape[d] == 1 else t.stride(d)
    a.out = out.data_ptr()
    a.batch, a.heads, a.tq, a.head_size = q.shape
    a.kv_heads, a.tk = k.shape[1], k.shape[2]
    a.divisor = divisor
    return a


def _reference(q, k, v, mask, divisor):
    groups = q.shape[1] // k.shape[1]
    k = k.double().repeat_interleave(groups, dim=1)
    v = v.double().repeat_interleave(groups, dim=1)
    s = (q.double() @ k.transpose(-1, -2)) / divisor + mask.double()
    return s.softmax(dim=-1) @ v


def _causal(torch, tq, tk):
    i = torch.arange(tq)[:, None]
    j = torch.arange(tk)[None, :]
    return torch.where(j > i + (tk - tq), -1e4, 0.0).to(torch.bfloat16).reshape(1, 1, tq, tk)


SKIP, ZERO = 1, 2  # CB_CAUSAL_SKIP, CB_CAUSAL_ZERO_BELOW
CASES = [  # batch, heads, kv_heads, tq, tk, head_size, causal flags
    (1, 8, 2, 300, 300, 64, SKIP | ZERO),
    (1, 8, 2, 300, 300, 64, 0),
    (1, 8, 2, 300, 300, 64, SKIP),
    (2, 4, 4, 200, 200, 128, SKIP | ZERO),
    (1, 4, 1, 64, 192, 64, SKIP | ZERO),  # verify-block shape: queries at the end of the keys
    (1, 32, 4, 1024, 1024, 64, SKIP | ZERO),
    (1, 2, 2, 129, 129, 128, 0),
]


@pytest.mark.parametrize("batch,heads,kv,tq,tk,hd,causal", CASES)
def test_sdpa_tc_matches_float64(batch, heads, kv, tq, tk, hd, causal):
    torch = pytest.importorskip("torch")
    from cuda_b200 import _lib

    gen = torch.Generator().manual_seed(tq * 31 + hd + heads)
    q = torch.randn(batch, heads, tq, hd, generator=gen)
    k = torch.randn(batch, kv, tk, hd, generator=gen)
    v = torch.randn(batch, tk, kv, hd, generator=gen).permute(0, 2, 1, 3)  # strided, like the model's v
    mask = _causal(torch, tq, tk)
    divisor = float(np.sqrt(hd))
    qd, kd, vd, md = q.cuda(), k.cuda(), v.cuda(), mask.cuda()
    out = torch.full((batch, heads, tq, hd), float("nan"), device="cuda")
    a = _args(torch, qd, kd, vd, md, out, divisor)
    lib = _lib.load()
    scratch = torch.empty(lib.cb_sdpa_tc_scratch(ctypes.byref(a)), dtype=torch.uint8, device="cuda")
    flag = torch.zeros(1, dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    _lib.call("cb_sdpa_tc", ctypes.byref(a), int(causal), scratch.data_ptr(), flag.data_ptr(), stream)
    torch.cuda.synchronize()
    assert int(flag.item()) == 0
    ref = _reference(q, k, v, mask.float(), divisor)
    got = out.cpu().double()
    assert torch.isfinite(got).all()
    err = float((got - ref).abs().max())
    assert err <= 2e-4 * float(v.abs().max()), err
    # and the generic float32 kernel agrees to the same bound
    generic = torch.zeros_like(out)
    a.out = generic.data_ptr()
    _lib.call("cb_sdpa", ctypes.byref(a), stream)
    torch.cuda.synchronize()
    assert float((generic.cpu().double() - got).abs().max()) <= 2e-4 * float(v.abs().max())


def test_sdpa_tc_rejects_unsupported_head_size():
    torch = pytest.importorskip("torch")
    from cuda_b200 import _lib

    q = torch.zeros(1, 2, 8, 32, device="cuda")
    mask = torch.zeros(1, 1, 8, 8, device="cuda")
    out = torch.zeros_like(q)
    a = _args(torch, q, q, q, mask, out, 1.0)
    with pytest.raises(_lib.KernelError, match="head_size"):
        _lib.call("cb_sdpa_tc", ctypes.byref(a), 0, out.data_ptr(), None, None)


def test_prefill_with_tensor_core_attention_matches_cpu_graph(gpu, oracle):
    """A 1-layer, head_size-64 bf16 model over 130 tokens: GEMMs + cb_sdpa_tc vs the cpu compiler."""
    import ml_dtypes

    from chomikgrad.llama import LlamaConfig, LlamaForCausalLM, position_selector, required_weight_shapes
    from chomikgrad.tensor import Tensor, compile_graph

    dt = np.dtype(ml_dtypes.bfloat16)
    config = LlamaConfig(vocab_size=512, hidden_size=256, intermediate_size=512, num_hidden_layers=1,
                         num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=256)
    rng = np.random.default_rng(5)
    weights = {name: Tensor(np.ones(shape, np.float32).astype(dt) if "norm.weight" in name
                            else rng.normal(0, 0.02, shape).astype(np.float32).astype(dt))
               for name, shape in required_weight_shapes(config).items()}
    seq = 130
    model = LlamaForCausalLM(config, weights, sequence_length=seq, dtype=dt, cache_length=seq + 4)
    ids = Tensor(rng.integers(0, config.vocab_size, (1, seq)).astype(np.int32), copy=False)
    outputs = model.prefill(ids, Tensor(position_selector(seq - 1, seq, dtype=dt), copy=False))
    program = compile_graph(*outputs, compiler="cuda-b200")
    assert "causal=3" in program.source and "place(" in program.source
    got = program()
    want = [o.numpy(compiler="cpu") for o in outputs]
    np.testing.assert_allclose(got[0], want[0], rtol=0, atol=2e-3)  # logits
    for g, w in zip(got[1:], want[1:]):  # the KV caches
        np.testing.assert_allclose(np.asarray(g, np.float32), np.asarray(w, np.float32), rtol=0, atol=1e-3)


QUERY_CASES = [  # batch, heads, kv_heads, tk, head_size
    (3, 8, 2, 100, 64),   # ragged last split
    (32, 32, 4, 768, 64),  # the batched TinyLlama step
    (2, 4, 4, 33, 128),
    (1, 2, 1, 5, 32),
    (2, 8, 8, 64, 256),
    (4, 32, 8, 1024, 128),  # Llama-3-8B shape
]


@pytest.mark.parametrize("batch,heads,kv,tk,hd", QUERY_CASES)
def test_sdpa_query_matches_float64(batch, heads, kv, tk, hd):
    """cb_sdpa_query (one query row, split over keys) vs float64 and the generic cb_sdpa."""
    torch = pytest.importorskip("torch")
    from cuda_b200 import _lib

    gen = torch.Generator().manual_seed(tk * 7 + hd + batch)
    q = torch.randn(batch, 1, heads, hd, generator=gen).permute(0, 2, 1, 3)  # strided q, like a view
    k = torch.randn(batch, kv, tk, hd, generator=gen)
    v = torch.randn(batch, kv, tk, hd, generator=gen)
    # decode mask: -1e4 past the current position, shared by every head
    mask = torch.where(torch.arange(tk) > tk - 3, -1e4, 0.0).to(torch.bfloat16).reshape(1, 1, 1, tk)
    divisor = float(np.sqrt(hd))
    qd, kd, vd, md = q.cuda(), k.cuda(), v.cuda(), mask.cuda()
    out = torch.full((batch, heads, 1, hd), float("nan"), device="cuda")
    a = _args(torch, qd, kd, vd, md, out, divisor)
    lib = _lib.load()
    scratch = torch.empty(lib.cb_sdpa_query_scratch(ctypes.byref(a)), dtype=torch.uint8, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    for _ in range(2):  # the scratch is reused: a second call gives the same result
        _lib.call("cb_sdpa_query", ctypes.byref(a), scratch.data_ptr(), stream)
    torch.cuda.synchronize()
    ref = _reference(q, k, v, mask.float(), divisor)
    got = out.cpu().double()
    assert torch.isfinite(got).all()
    assert float((got - ref).abs().max()) <= 2e-5 * float(v.abs().max())
    generic = torch.zeros_like(out)
    a.out = generic.data_ptr()
    _lib.call("cb_sdpa", ctypes.byref(a), stream)
    torch.cuda.synchronize()
    assert float((generic.cpu().double() - got).abs().max()) <= 2e-5 * float(v.abs().max())


def test_sdpa_query_rejects_unaligned_cache_rows():
    torch = pytest.importorskip("torch")
    from cuda_b200 import _lib

    q = torch.zeros(1, 2, 1, 64, device="cuda")
    kv = torch.zeros(1, 2, 8, 66, device="cuda")[..., :64]  # row stride 66 floats
    mask = torch.zeros(1, 1, 1, 8, device="cuda")
    out = torch.zeros_like(q)
    a = _args(torch, q, kv, kv, mask, out, 8.0)
    with pytest.raises(_lib.KernelError, match="16-byte aligned"):
        _lib.call("cb_sdpa_query", ctypes.byref(a), out.data_ptr(), None)
