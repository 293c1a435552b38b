"""Tree autograd (the host mirror of grad.scm).

CPU: the reference's known answers (tests/test-grad.scm of the reference,
groups 3-19) and its example 9 (linear regression by gradient descent),
with values through the oracle.  GPU: the same gradient trees realized on
the device, bit-exact against the oracle, and example 9 trained on the
device."""
import math

import numpy as np
import pytest

import amcuda as am
import oracle


def fv(vals, shape, rg=True):
    return am.make_var(am.morph_from_list([float(v) for v in vals], tuple(shape), "f64"), rg)


def gl(v):
    return list(np.asarray(oracle.values(am.var_grad(v)), dtype=np.float64).ravel())


def close(a, b, tol=1e-12):
    return len(a) == len(b) and all(abs(x - y) <= tol * max(1.0, abs(y)) for x, y in zip(a, b))


# ------------------------------------------------------------------ state (test-grad.scm:75-135)

def test_variable_state():
    m = am.morph_from_list([1.0, 2.0], (2,), "f64")
    v = am.make_var(m, True)
    assert am.var_value(v) is m and am.var_grad(v) is None and am.var_requires_grad(v)
    assert not am.var_requires_grad(am.make_var(m))
    am.accumulate_grad(v, am.morph_from_list([1.0, 1.0], (2,), "f64"))
    assert gl(v) == [1.0, 1.0]
    am.accumulate_grad(v, am.morph_from_list([2.0, 3.0], (2,), "f64"))
    assert gl(v) == [3.0, 4.0]
    am.zero_grad(v)
    assert am.var_grad(v) is None
    with pytest.raises(ValueError):
        am.make_var([1.0, 2.0])


# ------------------------------------------------------------------ arithmetic rules (test-grad.scm:140-300)

def test_binary_rules():
    v1, v2 = fv([1, 2, 3], [3]), fv([4, 5, 6], [3])
    am.backward(am.var_add(v1, v2))
    assert gl(v1) == [1.0] * 3 and gl(v2) == [1.0] * 3
    v1, v2 = fv([2], [1]), fv([1, 2, 3], [3])
    am.backward(am.var_add(v1, v2))
    assert gl(v1) == [3.0]
    v1, v2 = fv([5, 3], [2]), fv([1, 1], [2])
    am.backward(am.var_sub(v1, v2))
    assert gl(v1) == [1.0, 1.0] and gl(v2) == [-1.0, -1.0]
    v1, v2 = fv([2, 3], [2]), fv([4, 5], [2])
    am.backward(am.var_mul(v1, v2))
    assert gl(v1) == [4.0, 5.0] and gl(v2) == [2.0, 3.0]
    v1, v2 = fv([6, 8], [2]), fv([2, 4], [2])
    am.backward(am.var_div(v1, v2))
    assert gl(v1) == [0.5, 0.25] and gl(v2) == [-1.5, -0.5]


@pytest.mark.parametrize("op,xs,d", [
    (am.var_exp, [0.0, 1.0, 2.0], math.exp),
    (am.var_log, [1.0, 2.0, 4.0], lambda x: 1.0 / x),
    (am.var_sqrt, [1.0, 4.0, 9.0], lambda x: 1.0 / (2.0 * math.sqrt(x))),
    (am.var_sin, [0.0, 1.0, 2.0], math.cos),
    (am.var_cos, [0.0, 1.0, 2.0], lambda x: -math.sin(x)),
    (am.var_negate, [1.0, -2.0, 3.0], lambda x: -1.0),
    (am.var_abs, [1.5, -2.0, 0.0], lambda x: (x > 0) - (x < 0)),
    (am.var_relu, [1.5, -2.0, 0.0], lambda x: 1.0 if x > 0 else 0.0),
    (am.var_sigmoid, [0.0, 1.0, -2.0], lambda x: (1 / (1 + math.exp(-x))) * (1 - 1 / (1 + math.exp(-x)))),
    (am.var_tanh, [0.0, 0.5, -1.0], lambda x: 1.0 - math.tanh(x) ** 2),
])
def test_unary_rules(op, xs, d):
    v = fv(xs, [len(xs)])
    am.backward(op(v))
    assert close(gl(v), [float(d(x)) for x in xs])


def test_pow_rule():
    v1, v2 = fv([2.0, 3.0], [2]), fv([3.0, 2.0], [2])
    am.backward(am.var_pow(v1, v2))
    assert close(gl(v1), [3.0 * 2.0 ** 2, 2.0 * 3.0])
    assert close(gl(v2), [8.0 * math.log(2.0), 9.0 * math.log(3.0)])


# ------------------------------------------------------------------ reductions and structure (test-grad.scm:300-375)

def test_reduction_and_structural_rules():
    v = fv([1, 2, 3], [3])
    am.backward(am.var_sum(v))
    assert gl(v) == [1.0] * 3
    v = fv(range(1, 7), [2, 3])
    am.backward(am.var_sum(v, [0]))
    assert gl(v) == [1.0] * 6
    v = fv([1, 2, 3, 4], [4])
    am.backward(am.var_mean(v))
    assert gl(v) == [0.25] * 4
    v = fv(range(1, 7), [2, 3])
    am.backward(am.var_mean(v, [0]))
    assert gl(v) == [0.5] * 6
    v = fv(range(1, 7), [2, 3])
    am.backward(am.var_sum(v, [1], True))
    assert gl(v) == [1.0] * 6
    v = fv(range(1, 7), [6])
    am.backward(am.var_reshape(v, (2, 3)))
    assert am.var_grad(v).shape == (6,) and gl(v) == [1.0] * 6
    v = fv(range(1, 7), [2, 3])
    am.backward(am.var_transpose(v, (1, 0)))
    assert am.var_grad(v).shape == (2, 3) and gl(v) == [1.0] * 6


# ------------------------------------------------------------------ matmul, chain rule, multi-use, no-grad (test-grad.scm:380-510)

def test_matmul_chain_multiuse_nograd():
    A, B = fv(range(1, 7), [2, 3]), fv(range(1, 13), [3, 4])
    am.backward(am.var_matmul(A, B))
    assert am.var_grad(A).shape == (2, 3) and am.var_grad(B).shape == (3, 4)
    assert gl(A) == [10.0, 26.0, 42.0] * 2
    assert gl(B) == [5.0] * 4 + [7.0] * 4 + [9.0] * 4
    xs = [0.0, 1.0, -1.0]
    v = fv(xs, [3])
    one = am.make_var(am.morph_from_list([1.0], (1,), "f64"))
    am.backward(am.var_sum(am.var_log(am.var_add(am.var_exp(v), one))))
    assert close(gl(v), [math.exp(x) / (math.exp(x) + 1.0) for x in xs])
    v = fv([1, 2, 3], [3])
    am.backward(am.var_mul(v, v))
    assert gl(v) == [2.0, 4.0, 6.0]
    v1, v2 = fv([1, 2], [2]), fv([3, 4], [2], rg=False)
    am.backward(am.var_mul(v1, v2))
    assert am.var_grad(v2) is None and am.var_grad(v1) is not None
    out = am.var_add(fv([1], [1], rg=False), fv([2], [1], rg=False))
    am.backward(out)
    assert not am.var_requires_grad(out)


# ------------------------------------------------------------------ example 9: linear regression by gradient descent

def _example9_data():
    n = 10
    x = [v for i in range(n) for v in (i / 10.0, (9 - i) / 10.0)]
    y = [2.0 * (i / 10.0) + -1.0 * ((9 - i) / 10.0) + 0.5 for i in range(n)]
    return am.morph_from_list(x, (n, 2), "f64"), am.morph_from_list(y, (n, 1), "f64")


def _example9_step(values, realize, X, y, W, b, lr):
    """train-step of the reference's example 9: pred = X W^T + b, loss =
    mean((pred - y)^2), backward, then W -= lr dW, b -= lr db."""
    Wv, bv = am.make_var(W, True), am.make_var(b, True)
    pred = am.var_add(am.var_matmul(am.make_var(X), am.var_transpose(Wv, (1, 0))), bv)
    res = am.var_sub(pred, am.make_var(y))
    loss = am.var_mean(am.var_mul(res, res))
    am.backward(loss)
    dW, db = realize(am.var_grad(Wv)), realize(am.var_grad(bv))
    lr_m = am.morph_from_list([lr], (1,), "f64")
    W2 = realize(am.morph_sub(W, am.morph_mul(lr_m, dW)))
    b2 = realize(am.morph_sub(b, am.morph_mul(lr_m, db)))
    return W2, b2, float(np.asarray(values(am.var_value(loss))).ravel()[0])


def _example9_numpy(steps, lr):
    X = np.array([[i / 10.0, (9 - i) / 10.0] for i in range(10)])
    y = 2.0 * X[:, :1] - X[:, 1:] + 0.5
    W, b = np.zeros((1, 2)), np.zeros((1, 1))
    for _ in range(steps):
        res = X @ W.T + b - y
        g = 2.0 * res / len(X)
        W, b = W - lr * (g.T @ X), b - lr * g.sum(keepdims=True)
    return W.ravel(), b.ravel()


def _run_example9(values, realize):
    X, y = _example9_data()
    W, b = am.morph_from_list([0.0, 0.0], (1, 2), "f64"), am.morph_from_list([0.0], (1, 1), "f64")
    losses = []
    for _ in range(30):
        W, b, loss = _example9_step(values, realize, X, y, W, b, 0.5)
        losses.append(loss)
    return np.asarray(values(W)).ravel(), np.asarray(values(b)).ravel(), losses


def test_example9_linear_regression_oracle():
    W, b, losses = _run_example9(oracle.values, oracle.realize)
    assert abs(losses[0] - 1.645) < 1e-12                  # mean(y^2) at W = 0, b = 0
    assert all(l2 < l1 for l1, l2 in zip(losses, losses[1:])) and losses[-1] < 1e-4
    Wn, bn = _example9_numpy(30, 0.5)
    np.testing.assert_allclose(W, Wn, rtol=1e-10)
    np.testing.assert_allclose(b, bn, rtol=1e-10)


# ------------------------------------------------------------------ device

@pytest.mark.gpu
def test_gradients_on_device_bitwise(amc):
    rng = np.random.default_rng(5)
    x = am.make_var(am.morph_from_numpy(rng.uniform(0.5, 2.0, (6, 5))), True)
    w = am.make_var(am.morph_from_numpy(rng.standard_normal((5, 4))), True)
    b = am.make_var(am.morph_from_numpy(rng.standard_normal((1, 4))), True)
    h = am.var_tanh(am.var_add(am.var_matmul(x, w), b))
    loss = am.var_mean(am.var_mul(am.var_sigmoid(h), am.var_log(am.var_add(h, am.make_var(
        am.morph_from_list([2.0], (1,), "f64"))))))
    am.backward(loss)
    for v in (x, w, b):
        got, ref = np.asarray(amc.realize(am.var_grad(v)).values()), np.asarray(oracle.values(am.var_grad(v)))
        assert got.shape == ref.shape
        assert np.array_equal(got.reshape(-1).view(np.uint8), ref.reshape(-1).view(np.uint8))


@pytest.mark.gpu
def test_example9_linear_regression_device(amc):
    W, b, losses = _run_example9(lambda m: amc.realize(m).values(), amc.realize)
    Wo, bo, lo = _run_example9(oracle.values, oracle.realize)
    assert np.array_equal(W, Wo) and np.array_equal(b, bo) and losses == lo
