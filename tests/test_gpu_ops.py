"""GPU parity of the generic six-op lowering and the rms_norm/rope/sdpa kernels.

Patterns follow the reference's backend tests (tests/test_cuda.py:32-138,
tests/test_lazy.py:49-63): every result is compared with the reference
``cpu`` compiler's output -- the golden fixtures for the known answers, the
restated oracle for random cases.
"""

from __future__ import annotations

import numpy as np
import pytest

from conftest import golden
from chomikgrad.tensor import Tensor, compile_graph

pytestmark = pytest.mark.gpu


def bf16():
    import ml_dtypes

    return np.dtype(ml_dtypes.bfloat16)


def test_six_ir_operations_and_gather_match_golden(gpu, oracle):
    g = golden("six_ops")
    left, right = Tensor(g["chain_left"]), Tensor(g["chain_right"])
    result = ((left @ right).relu() + 0.25).permute(1, 0).reshape(1, 4).sum(axis=1)
    program = compile_graph(result, compiler="cuda-b200")
    np.testing.assert_allclose(program()[0], g["chain_out"], rtol=1e-5, atol=1e-6)
    assert "matmul" in program.source and "elementwise" in program.source
    gathered = Tensor(g["gather_table"]).gather(Tensor(g["gather_idx"], copy=False))
    out = gathered.numpy(compiler="cuda-b200")
    assert np.array_equal(out, g["gather_out"])  # bit-exact


def test_batched_and_broadcast_matmul_match_golden(gpu, oracle):
    g = golden("six_ops")
    np.testing.assert_allclose((Tensor(g["bmm_a"]) @ Tensor(g["bmm_b"])).numpy(compiler="cuda-b200"),
                               g["bmm_out"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose((Tensor(g["proj_x"]) @ Tensor(g["proj_w"])).numpy(compiler="cuda-b200"),
                               g["proj_out"], rtol=1e-5, atol=1e-6)


def test_softmax_portable_path_matches_golden(gpu, oracle):
    g = golden("six_ops")
    np.testing.assert_allclose(Tensor(g["softmax_x"]).softmax(axis=-1).numpy(compiler="cuda-b200"),
                               g["softmax_out"], rtol=1e-5, atol=1e-6)
    np.testing.assert_allclose(Tensor(g["softmax_x"]).softmax(axis=1).numpy(compiler="cuda-b200"),
                               g["softmax1_out"], rtol=1e-5, atol=1e-6)


def test_bf16_sum_accumulates_sequentially_like_numpy(gpu, oracle):
    g = golden("six_ops")
    x = g["bf16_sumsq_x"].view(bf16())
    t = Tensor(x)
    out = (t * t).sum(axis=-1, keepdims=True).numpy(compiler="cuda-b200")
    assert np.array_equal(out.view(np.uint16), g["bf16_sumsq_out"])  # bit-exact


def test_dynamic_input_and_deferred_synchronization(gpu):
    source = Tensor([1.0, 2.0], dtype=np.float32)
    program = compile_graph(source * 2.0, compiler="cuda-b200", dynamic_inputs=(source,))
    replacement = program.device.array(np.array([3.0, 4.0], dtype=np.float32))
    native = program.run({source._node: replacement}, synchronize=False)[0]
    program.device.synchronize()
    np.testing.assert_allclose(program.device.to_numpy(native), [6.0, 8.0])
    assert program.inputs == (source._node,)
    assert program.device.argmax(native) == 1
    np.testing.assert_allclose(program()[0], [2.0, 4.0])


def test_copy_false_observes_host_mutation(gpu):
    source = np.array([1.0, 2.0], dtype=np.float32)
    tensor = Tensor(source, copy=False)
    np.testing.assert_allclose(tensor.numpy(compiler="cuda-b200"), [1.0, 2.0])
    source[0] = 9.0
    np.testing.assert_allclose(tensor.numpy(compiler="cuda-b200"), [9.0, 2.0])


def test_repeated_runs_replay_a_graph_and_stay_bit_identical(gpu, oracle):
    rng = np.random.default_rng(3)
    x = Tensor(rng.normal(size=(4, 33)).astype(np.float32))
    w = Tensor(rng.normal(size=(33, 17)).astype(np.float32))
    out = ((x @ w).exp() / 3.0 - 1.0).max(axis=0)
    program = compile_graph(out, compiler="cuda-b200")
    first = program()[0]
    for _ in range(3):
        assert np.array_equal(program()[0], first)
    assert program._graphs, "second and later runs should replay a CUDA graph"
    np.testing.assert_allclose(first, out.numpy(compiler="cpu"), rtol=1e-5, atol=1e-6)


def test_argmax_first_occurrence_and_nan(gpu):
    device = gpu.device
    values = np.array([[1.0, 5.0, 5.0, -2.0]], dtype=np.float32)
    assert device.argmax(device.array(values)) == 1
    with_nan = np.array([1.0, np.nan, 7.0, np.nan], dtype=np.float32)
    assert device.argmax(device.array(with_nan)) == int(np.argmax(with_nan))
    rows = np.random.default_rng(5).normal(size=(6, 100)).astype(np.float32)
    np.testing.assert_array_equal(device.argmax_last_axis(device.array(rows)), rows.argmax(axis=-1))


@pytest.mark.parametrize("ranks", [1, 2, 4, 8])
def test_sharded_argmax_records_and_pick(gpu, ranks):
    """cb_argmax_rows_partial over column slices (one per emulated rank) + cb_argmax_pick == np.argmax of the
    whole row: ties across slice boundaries (lower index), NaN (first NaN), inf, all-equal rows; bf16 too."""
    import ml_dtypes
    import torch

    from cuda_b200 import _lib

    rng = np.random.default_rng(ranks)
    vocab = 96 * ranks
    logits = rng.normal(0, 1, (10, vocab)).astype(np.float32)
    cols = vocab // ranks
    logits[1, [5, min(cols, vocab - 1)]] = 9.0
    logits[2, [vocab - 1, 0]] = 7.0
    logits[3, vocab // 2 + 1] = np.nan
    logits[4, [3, vocab - 2]] = np.nan
    logits[5] = 0.0
    logits[6, -1] = np.inf
    logits[7] = -np.inf
    for dtype, code in ((np.float32, _lib.F32), (ml_dtypes.bfloat16, _lib.BF16)):
        host = logits.astype(dtype)
        dev = torch.from_numpy(host.view(np.uint16) if dtype != np.float32 else host).cuda()
        records = torch.zeros(ranks * host.shape[0] * 4, dtype=torch.float32, device="cuda")
        out = torch.full((host.shape[0],), -7, dtype=torch.int64, device="cuda")
        stream = torch.cuda.current_stream().cuda_stream
        for r in range(ranks):
            piece = dev[:, r * cols:(r + 1) * cols].contiguous()
            _lib.call("cb_argmax_rows_partial", piece.data_ptr(), code, host.shape[0], cols, r * cols,
                      records.data_ptr() + r * host.shape[0] * 16, stream)
        _lib.call("cb_argmax_pick", records.data_ptr(), ranks, host.shape[0], out.data_ptr(), stream)
        np.testing.assert_array_equal(out.cpu().numpy(), np.argmax(host.astype(np.float32), axis=-1))
        # the whole path on one rank (no communicator): partial, copy, pick
        scratch = torch.zeros(2 * host.shape[0] * 4, dtype=torch.float32, device="cuda")
        out.fill_(-7)
        _lib.call("cb_argmax_rows_sharded", None, 1, dev.data_ptr(), code, host.shape[0], vocab, 0,
                  scratch.data_ptr(), out.data_ptr(), stream)
        np.testing.assert_array_equal(out.cpu().numpy(), np.argmax(host.astype(np.float32), axis=-1))


def test_gather_out_of_range_raises(gpu):
    table = Tensor(np.arange(6, dtype=np.float32).reshape(3, 2))
    bad = Tensor(np.array([[0, 3]], dtype=np.int32), copy=False)
    with pytest.raises(IndexError):
        table.gather(bad).numpy(compiler="cuda-b200")


def test_float64_is_rejected_without_fallback(gpu):
    with pytest.raises(TypeError):
        (Tensor([1.0, 2.0]) * 2.0).numpy(compiler="cuda-b200")


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_llama_lowerings_match_portable_cpu_graph(gpu, oracle, dtype):
    """rms_norm/rope/sdpa lowerings on a 1-layer model (pattern of test_mlx.py:120-158)."""
    from chomikgrad.llama import LlamaConfig, LlamaForCausalLM, position_selector, required_weight_shapes

    dt = np.dtype(np.float32) if dtype == "float32" else bf16()
    config = LlamaConfig(vocab_size=64, hidden_size=64, intermediate_size=96, num_hidden_layers=1,
                         num_attention_heads=4, num_key_value_heads=2, max_position_embeddings=16)
    rng = np.random.default_rng(23)
    weights = {name: Tensor(np.ones(shape, np.float32).astype(dt) if "norm.weight" in name
                            else rng.normal(0, 0.05, shape).astype(np.float32).astype(dt))
               for name, shape in required_weight_shapes(config).items()}
    model = LlamaForCausalLM(config, weights, sequence_length=5, dtype=dt)
    output = model(Tensor(np.array([[1, 3, 4, 9, 2]], dtype=np.int32), copy=False),
                   Tensor(position_selector(4, 5, dtype=dt), copy=False))
    program = compile_graph(output, compiler="cuda-b200")
    for name in ("rms_norm", "rope", "sdpa", "gather"):
        assert name in program.source
    np.testing.assert_allclose(program()[0], output.numpy(compiler="cpu"), rtol=2e-4, atol=2e-5)


@pytest.mark.parametrize("dtype", ["float32", "bfloat16"])
def test_placement_matmul_is_a_bit_exact_column_copy(gpu, oracle, dtype):
    """x @ P for a placement P (llama.py:411-418) runs cb_place_columns and equals the cpu matmul."""
    dt = bf16() if dtype == "bfloat16" else np.dtype(np.float32)
    rng = np.random.default_rng(7)
    x = rng.standard_normal((1, 3, 6, 5)).astype(dt)
    cache = np.zeros((6, 9), dt)
    cache[np.arange(6), np.arange(6)] = 1  # the prefill's cache_placement
    perm = np.zeros((6, 9), dt)
    perm[np.arange(6), [4, 0, 8, 2, 1, 6]] = 1
    for p in (cache, perm):
        expr = (Tensor(x).permute(0, 1, 3, 2) @ Tensor(p)).permute(0, 1, 3, 2)
        program = compile_graph(expr, compiler="cuda-b200")
        assert "place(" in program.source and "matmul(" not in program.source
        got = np.asarray(program()[0])
        want = expr.numpy(compiler="cpu")
        assert got.dtype == want.dtype
        assert np.array_equal(got.astype(np.float32), want.astype(np.float32))


def test_load_safetensors_round_trip(gpu, tmp_path):
    """DeviceAdapter.load_safetensors (chomikgrad/lazy.py:140-145) through the reference's own
    wrapper chomikgrad.llama.load_safetensors (:186-203): bf16 and float32 tensors come back
    bit-exact as device arrays, with an optional cast."""
    import ml_dtypes
    import torch
    from safetensors.torch import save_file
    from chomikgrad.llama import load_safetensors

    rng = np.random.default_rng(8)
    bf16 = np.dtype(ml_dtypes.bfloat16)
    tensors = {"a.weight": rng.normal(0, 0.02, (64, 32)).astype(np.float32).astype(bf16),
               "b.bias": rng.normal(0, 1, (17,)).astype(np.float32)}
    path = tmp_path / "tiny.safetensors"
    save_file({"a.weight": torch.from_numpy(tensors["a.weight"].view(np.int16)).view(torch.bfloat16),
               "b.bias": torch.from_numpy(tensors["b.bias"])}, str(path))
    loaded = load_safetensors(path, gpu.device)
    assert set(loaded) == set(tensors)
    for name, want in tensors.items():
        got = gpu.device.to_numpy(loaded[name]._node.native_values[gpu.device.name])
        assert got.dtype == want.dtype and got.shape == want.shape
        np.testing.assert_array_equal(got.view(np.uint8), np.ascontiguousarray(want).view(np.uint8))
    cast = gpu.device.load_safetensors(path, dtype=np.float32)
    np.testing.assert_array_equal(gpu.device.to_numpy(cast["a.weight"]), tensors["a.weight"].astype(np.float32))
