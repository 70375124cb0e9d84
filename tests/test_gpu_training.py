"""Training on the B200: the fused lowerings' kernels and the SGD update against the CPU.

Patterns of the reference's own CUDA tests (tests/test_cuda.py:140-379),
with ``compiler="cuda-b200"`` in place of its CuPy ``cuda`` compiler and the
parity oracle (the restated reference ``cpu`` compiler) as the CPU side:
layer_norm, softmax / log_softmax backward and layer_norm backward
(one launch for three gradients) through ``compile_graph``; SGD that keeps
parameters on the device (new storage, or in place); the grouped update over
several launches' worth of tensors; ``compile_train_step`` that reuses one
backward graph and matches eager steps.  Then a few steps of a small
transformer-style model trained on both sides.
"""

from __future__ import annotations

import numpy as np
import pytest

from chomikgrad import SGD, Parameter, Tensor, compile_graph, compile_train_step

pytestmark = pytest.mark.gpu

B = "cuda-b200"


def test_layer_norm_lowering(gpu, oracle):
    rng = np.random.default_rng(23)
    source = Tensor(rng.normal(size=(3, 4, 64)).astype(np.float32))
    weight = Tensor(rng.normal(size=64).astype(np.float32))
    bias = Tensor(rng.normal(size=64).astype(np.float32))
    result = source.layer_norm(weight, bias)
    expected = result.numpy(compiler="cpu")
    program = compile_graph(result, compiler=B)
    assert "layer_norm(" in program.source
    np.testing.assert_allclose(gpu.device.to_numpy(program()[0]), expected, rtol=1e-5, atol=1e-5)


def test_softmax_backward_lowerings(gpu, oracle):
    rng = np.random.default_rng(29)
    source = Tensor(rng.normal(size=(3, 5, 64)).astype(np.float32), requires_grad=True)
    upstream = Tensor(rng.normal(size=source.shape).astype(np.float32))
    (source.softmax(axis=-1) * upstream).sum().backward()
    program = compile_graph(source.grad, compiler=B)
    assert " = softmax(" in program.source and "softmax_backward(" in program.source
    np.testing.assert_allclose(gpu.device.to_numpy(program()[0]), source.grad.numpy(compiler="cpu"),
                               rtol=1e-5, atol=1e-6)
    log_source = Tensor(rng.normal(size=(4, 7)).astype(np.float32), requires_grad=True)
    log_up = Tensor(rng.normal(size=log_source.shape).astype(np.float32))
    (log_source.log_softmax(axis=-1) * log_up).sum().backward()
    program = compile_graph(log_source.grad, compiler=B)
    assert "log_softmax_backward(" in program.source
    np.testing.assert_allclose(gpu.device.to_numpy(program()[0]), log_source.grad.numpy(compiler="cpu"),
                               rtol=2e-5, atol=2e-6)
    other = Tensor(rng.normal(size=(2, 3, 4)).astype(np.float32), requires_grad=True)
    other_up = Tensor(rng.normal(size=other.shape).astype(np.float32))
    (other.softmax(axis=1) * other_up).sum().backward()
    np.testing.assert_allclose(other.grad.numpy(compiler=B), other.grad.numpy(compiler="cpu"), rtol=2e-5, atol=2e-6)
    empty = Tensor(np.empty((0, 4), dtype=np.float32)).softmax(axis=-1)
    assert empty.numpy(compiler=B).shape == (0, 4)
    wide = Tensor(rng.normal(0, 3, size=(5, 32000)).astype(np.float32), requires_grad=True)
    (wide.log_softmax(axis=-1) * Tensor(rng.normal(size=wide.shape).astype(np.float32))).sum().backward()
    np.testing.assert_allclose(wide.grad.numpy(compiler=B), wide.grad.numpy(compiler="cpu"), rtol=1e-4, atol=1e-5)


def test_layer_norm_backward_in_one_launch(gpu, oracle):
    rng = np.random.default_rng(31)
    source = Tensor(rng.normal(size=(3, 5, 64)).astype(np.float32), requires_grad=True)
    weight = Tensor(rng.normal(size=64).astype(np.float32), requires_grad=True)
    bias = Tensor(rng.normal(size=64).astype(np.float32), requires_grad=True)
    upstream = Tensor(rng.normal(size=source.shape).astype(np.float32))
    (source.layer_norm(weight, bias) * upstream).sum().backward()
    grads = (source.grad, weight.grad, bias.grad)
    expected = [g.numpy(compiler="cpu") for g in grads]
    program = compile_graph(*grads, compiler=B)
    assert program.source.count("layer_norm_backward(") == 1
    for actual, want in zip(program(), expected):
        np.testing.assert_allclose(gpu.device.to_numpy(actual), want, rtol=2e-5, atol=2e-5)


def test_sgd_keeps_parameters_on_the_device(gpu, oracle):
    parameter = Parameter(np.array([[1.0], [2.0]], dtype=np.float32))
    inputs = Tensor(np.array([[3.0, 4.0]], dtype=np.float32))
    old_graph = parameter * 2.0
    before = compile_graph(parameter, compiler=B).run(synchronize=True)[0]
    (inputs @ parameter).sum().backward()
    SGD([parameter], lr=0.1).step(compiler=B)
    assert parameter._node.value is None and B in parameter._node.native_values
    after = parameter._node.native_values[B]
    assert before.data_ptr() != after.data_ptr()
    np.testing.assert_allclose(parameter.numpy(compiler="cpu"), [[0.7], [1.6]], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(old_graph.numpy(compiler=B), [[2.0], [4.0]])


def test_inplace_sgd_reuses_the_parameter_storage(gpu, oracle):
    parameter = Parameter(np.array([[1.0], [2.0]], dtype=np.float32))
    inputs = Tensor(np.array([[3.0, 4.0]], dtype=np.float32))
    old_graph = parameter * 2.0
    before = compile_graph(parameter, compiler=B).run(synchronize=True)[0]
    (inputs @ parameter).sum().backward()
    SGD([parameter], lr=0.1, inplace=True).step(compiler=B)
    after = parameter._node.native_values[B]
    assert before.data_ptr() == after.data_ptr()
    np.testing.assert_allclose(parameter.numpy(compiler="cpu"), [[0.7], [1.6]], rtol=1e-6, atol=1e-6)
    np.testing.assert_allclose(old_graph.numpy(compiler=B), [[1.4], [3.2]])


def test_sgd_groups_many_parameters(gpu, oracle):
    parameters = [Parameter(np.array([float(i)], dtype=np.float32)) for i in range(18)]
    big = Parameter(np.random.default_rng(3).normal(size=(1003, 17)).astype(np.float32))  # ragged, > 1 block
    loss = parameters[0].sum()
    for p in parameters[1:]:
        loss = loss + p.sum()
    loss = loss + (big * big).sum()
    start = big.numpy(compiler="cpu").copy()
    loss.backward()
    SGD(parameters + [big], lr=0.25).step(compiler=B)
    for i, p in enumerate(parameters):
        np.testing.assert_allclose(p.numpy(compiler=B), [i - 0.25], rtol=1e-6, atol=1e-6)
    want = start - np.float32(0.25) * (np.float32(2) * start)
    np.testing.assert_array_equal(big.numpy(compiler=B), want)


def test_compiled_train_step_matches_eager_steps(gpu, oracle):
    initial = np.array([[0.2, -0.1, 0.4], [-0.3, 0.5, 0.1]], dtype=np.float32)
    reference, compiled = Parameter(initial.copy()), Parameter(initial.copy())
    ref_opt, comp_opt = SGD([reference], lr=0.05), SGD([compiled], lr=0.05)
    captures = 0

    def loss(parameter, inputs, targets):
        logits = inputs @ parameter
        return -(logits.log_softmax(axis=1) * targets).sum() / inputs.shape[0]

    def compiled_loss(inputs, targets):
        nonlocal captures
        captures += 1
        return loss(compiled, inputs, targets)

    step = compile_train_step(compiled_loss, comp_opt, Tensor.zeros((4, 2)), Tensor.zeros((4, 3)),
                              compiler=B, return_loss=True)
    batches = (
        (np.array([[1.0, 0.0], [0.0, 1.0], [1.0, 1.0], [-1.0, 0.5]], dtype=np.float32),
         np.eye(3, dtype=np.float32)[[0, 1, 2, 1]]),
        (np.array([[0.5, 1.0], [1.5, -0.5], [-0.5, 1.0], [2.0, 1.0]], dtype=np.float32),
         np.eye(3, dtype=np.float32)[[2, 0, 1, 2]]),
    )
    for inputs, targets in batches:
        ref_opt.zero_grad()
        ref_loss = loss(reference, Tensor(inputs, copy=False), Tensor(targets, copy=False))
        ref_loss.backward()
        ref_opt.step(compiler="cpu")
        got = step(inputs, targets)
        np.testing.assert_allclose(got.numpy(compiler=B), ref_loss.numpy(compiler="cpu"), rtol=2e-5, atol=2e-6)
    assert captures == 1
    np.testing.assert_allclose(compiled.numpy(compiler=B), reference.numpy(compiler="cpu"), rtol=2e-5, atol=2e-6)


def test_transformer_style_model_trains_like_the_cpu(gpu, oracle):
    """Eight compiled SGD steps of an embedding (one-hot rows @ table) / layer norm / attention /
    MLP / cross-entropy model on the B200, against the reference's eager SGD on its cpu compiler:
    losses and final parameters agree."""
    rng = np.random.default_rng(7)
    tokens, width, vocab, hidden = 8, 64, 29, 96
    shapes = {"table": (vocab, width), "ln_w": (width,), "ln_b": (width,), "wq": (width, width),
              "wk": (width, width), "wv": (width, width), "w1": (width, hidden), "w2": (hidden, vocab)}
    init = {k: (np.ones(s, np.float32) if k == "ln_w" else rng.normal(0, 0.1, s).astype(np.float32))
            for k, s in shapes.items()}
    # token ids enter as one-hot rows times the table: the reference's gather backward bakes the
    # trace-time indices into a constant (tensor.py:548-561), so a compiled step would keep the
    # example's ids for the table gradient
    eye = np.eye(vocab, dtype=np.float32)
    batch = (eye[rng.integers(0, vocab, tokens)], eye[rng.integers(0, vocab, tokens)])
    batches = [batch] * 8  # one batch, eight steps: the loss falls

    def train(compiler):
        p = {k: Parameter(v.copy()) for k, v in init.items()}
        opt = SGD(list(p.values()), lr=0.1)

        def loss(ids, targets):
            h = (ids @ p["table"]).layer_norm(p["ln_w"], p["ln_b"])
            scores = (h @ p["wq"]) @ (h @ p["wk"]).transpose(1, 0) / np.float32(8.0)
            mixed = scores.softmax(axis=-1) @ (h @ p["wv"]) + h
            logits = (mixed @ p["w1"]).relu() @ p["w2"]
            return -(logits.log_softmax(axis=-1) * targets).sum() / np.float32(tokens)

        if compiler == "cpu":  # the reference's cpu compiler has no compiled steps: eager SGD (optim.py:28-64)
            losses = []
            for ids, t in batches:
                opt.zero_grad()
                value = loss(Tensor(ids, copy=False), Tensor(t, copy=False))
                value.backward()
                losses.append(float(value.numpy(compiler="cpu")))
                opt.step(compiler="cpu")
        else:
            step = compile_train_step(loss, opt, Tensor.zeros((tokens, vocab)), Tensor.zeros((tokens, vocab)),
                                      compiler=compiler, return_loss=True)
            losses = [float(step(ids, t).numpy(compiler=compiler)) for ids, t in batches]
        return losses, {k: v.numpy(compiler=compiler) for k, v in p.items()}

    gpu_losses, gpu_params = train(B)
    cpu_losses, cpu_params = train("cpu")
    np.testing.assert_allclose(gpu_losses, cpu_losses, rtol=1e-4)
    assert gpu_losses[-1] < gpu_losses[0]
    for k in shapes:
        np.testing.assert_allclose(gpu_params[k], cpu_params[k], rtol=1e-4, atol=1e-5, err_msg=k)
