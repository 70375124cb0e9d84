"""Training graphs through the planner, on the CPU (plan interpreter vs the parity oracle).

The reference's autograd marks softmax / log_softmax, their backward
contributions, layer_norm and its backward contributions with lowering hints
(chomikgrad/tensor.py:316-450).  The planner lowers each hint to one step
(``softmax``, ``softmax_backward``, ``layer_norm``, ``layer_norm_backward``:
one step for all of a backward's requested input / weight / bias
contributions) and leaves everything else on the generic steps.  These tests
interpret the planned programs step by step and compare them with the
oracle's evaluation of the unrewritten graphs, in the patterns of the
reference's own CUDA tests (tests/test_cuda.py:140-236), and a whole
transformer-style loss with its gradients.  Bars: rtol 2e-5, atol 2e-5.
"""

from __future__ import annotations

from collections import Counter

import numpy as np

from chomikgrad.tensor import Tensor
from cuda_b200.planner import Planner
from plan_interpreter import PlanInterpreter

TOL = dict(rtol=2e-5, atol=2e-5)


def _leaf_dtype(node):
    return np.asarray(node.numpy_value()).dtype


def _plan(outputs):
    return Planner([o._node for o in outputs], [], backend="cuda-b200", leaf_dtype=_leaf_dtype).build()


def _interpret(outputs):
    plan = _plan(outputs)
    it = PlanInterpreter(plan)
    it.run()
    return plan, it.outputs()


def _oracle(outputs):
    from oracle.numpy_compiler import NumpyCompiler

    return [np.asarray(v) for v in NumpyCompiler().compile([o._node for o in outputs]).run()]


def _kinds(plan):
    return Counter(s.name for s in plan.steps)


def test_layer_norm_lowers_to_one_step():
    rng = np.random.default_rng(23)
    source = Tensor(rng.normal(size=(3, 4, 64)).astype(np.float32))
    weight = Tensor(rng.normal(size=64).astype(np.float32))
    bias = Tensor(rng.normal(size=64).astype(np.float32))
    result = source.layer_norm(weight, bias)
    plan, got = _interpret([result])
    assert _kinds(plan)["layer_norm"] == 1 and "layer_norm(" in plan.source
    np.testing.assert_allclose(got[0], _oracle([result])[0], **TOL)


def test_softmax_and_log_softmax_backward_lower_over_the_last_axis():
    rng = np.random.default_rng(29)
    source = Tensor(rng.normal(size=(3, 5, 64)).astype(np.float32), requires_grad=True)
    upstream = Tensor(rng.normal(size=source.shape).astype(np.float32))
    (source.softmax(axis=-1) * upstream).sum().backward()
    plan, got = _interpret([source.grad])
    assert _kinds(plan)["softmax"] == 1 and _kinds(plan)["softmax_backward"] == 1
    np.testing.assert_allclose(got[0], _oracle([source.grad])[0], rtol=1e-5, atol=1e-6)

    log_source = Tensor(rng.normal(size=(4, 7)).astype(np.float32), requires_grad=True)
    log_up = Tensor(rng.normal(size=log_source.shape).astype(np.float32))
    (log_source.log_softmax(axis=-1) * log_up).sum().backward()
    plan, got = _interpret([log_source.grad])
    assert "log_softmax(" in plan.source and "log_softmax_backward(" in plan.source
    np.testing.assert_allclose(got[0], _oracle([log_source.grad])[0], **TOL)

    # another axis: the portable graph on the generic steps, same values
    other = Tensor(rng.normal(size=(2, 3, 4)).astype(np.float32), requires_grad=True)
    other_up = Tensor(rng.normal(size=other.shape).astype(np.float32))
    (other.softmax(axis=1) * other_up).sum().backward()
    plan, got = _interpret([other.grad])
    assert _kinds(plan)["softmax"] == 0 and _kinds(plan)["softmax_backward"] == 0
    np.testing.assert_allclose(got[0], _oracle([other.grad])[0], **TOL)

    empty = Tensor(np.empty((0, 4), dtype=np.float32)).softmax(axis=-1)
    plan, got = _interpret([empty])
    assert got[0].shape == (0, 4)


def test_layer_norm_backward_is_one_step_for_three_gradients():
    rng = np.random.default_rng(31)
    source = Tensor(rng.normal(size=(3, 5, 64)).astype(np.float32), requires_grad=True)
    weight = Tensor(rng.normal(size=64).astype(np.float32), requires_grad=True)
    bias = Tensor(rng.normal(size=64).astype(np.float32), requires_grad=True)
    upstream = Tensor(rng.normal(size=source.shape).astype(np.float32))
    (source.layer_norm(weight, bias) * upstream).sum().backward()
    grads = [source.grad, weight.grad, bias.grad]
    plan, got = _interpret(grads)
    assert plan.source.count("layer_norm_backward(") == 1
    for a, b in zip(got, _oracle(grads)):
        np.testing.assert_allclose(a, b, **TOL)
    # only the weight gradient requested
    plan, got = _interpret([weight.grad])
    assert _kinds(plan)["layer_norm_backward"] == 1
    np.testing.assert_allclose(got[0], _oracle([weight.grad])[0], **TOL)


def test_transformer_style_loss_and_gradients():
    """Embedding rows, layer norm, attention scores with softmax, an MLP with relu, log-softmax
    cross entropy: the loss and every parameter's gradient."""
    rng = np.random.default_rng(5)
    tokens, width, vocab, hidden = 6, 32, 11, 48

    def param(*shape, scale=0.2):
        return Tensor(rng.normal(0, scale, shape).astype(np.float32), requires_grad=True)

    table, ln_w, ln_b = param(vocab, width), param(width, scale=1.0), param(width)
    wq, wk, wv = param(width, width), param(width, width), param(width, width)
    w1, w2 = param(width, hidden), param(hidden, vocab)
    ids = Tensor(rng.integers(0, vocab, (1, tokens)).astype(np.int32), copy=False)
    targets = Tensor(np.eye(vocab, dtype=np.float32)[rng.integers(0, vocab, tokens)])
    x = table.gather(ids).reshape(tokens, width)
    h = x.layer_norm(ln_w, ln_b)
    scores = (h @ wq) @ (h @ wk).transpose(1, 0) / np.float32(np.sqrt(width))
    attended = scores.softmax(axis=-1) @ (h @ wv)
    logits = ((attended + h) @ w1).relu() @ w2
    loss = -(logits.log_softmax(axis=-1) * targets).sum() / np.float32(tokens)
    loss.backward()
    params = [table, ln_w, ln_b, wq, wk, wv, w1, w2]
    outputs = [loss] + [p.grad for p in params]
    plan, got = _interpret(outputs)
    kinds = _kinds(plan)
    assert kinds["layer_norm"] >= 1 and kinds["layer_norm_backward"] == 1
    assert kinds["softmax_backward"] == 2  # the attention softmax and the log-softmax
    for a, b in zip(got, _oracle(outputs)):
        np.testing.assert_allclose(a, b, rtol=1e-4, atol=1e-5)
