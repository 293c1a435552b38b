"""SSA compilation and VJP (the host mirror of ssa.scm).

CPU: the reference's known answers (tests/test-ssa.scm of the reference:
morphism-to-ssa structure, ssa-realize outputs, ssa-vjp gradients, the
aliasing and activation groups), with the program realized by the oracle.
GPU: the same programs realized on the device bit-exact against the
oracle, and ssa_realize_ctx trace / finalize / replay."""
import math

import numpy as np
import pytest

import amcuda as am
from amcuda import ssa as S
import oracle

TOL = 1e-9   # the reference tests' tolerance (test-ssa.scm:37)


def ml(vals, shape):
    return am.morph_from_list([float(v) for v in vals], tuple(shape), "f64")


def param(vals, shape):
    return am.make_var(ml(vals, shape), True)


def inp(vals, shape):
    return am.make_var(ml(vals, shape), False)


def flat(m):
    return list(np.asarray(m.values(), dtype=np.float64).reshape(-1))


def close(a, b, tol=TOL):
    return len(a) == len(b) and all(abs(x - y) <= tol for x, y in zip(a, b))


def joint_of(loss, params):
    """compile-and-realize's first half (test-ssa.scm:80-88)."""
    fwd = S.morphism_to_ssa(loss)
    pv = [v for v in (S.ssa_constant_id(fwd, am.var_value(p)) for p in params) if v is not None]
    return S.ssa_vjp(fwd, pv, S.ssa_loss_binding_val(fwd))


def compile_and_realize(loss, params, realize=oracle.realize):
    return [flat(r) for r in S.ssa_realize(joint_of(loss, params), realize)]


# ------------------------------------------------------------------ group 1: morphism-to-ssa (test-ssa.scm:110-206)

def test_morphism_to_ssa_structure():
    W = ml([1, 2], [2])
    prog = S.morphism_to_ssa(am.make_var(W, True))
    assert prog.bindings == [] and len(prog.constants) == 1
    assert isinstance(S.ssa_constant_id(prog, W), S.ConstRef)
    assert S.ssa_constant_id(prog, ml([1], [1])) is None
    a, b = ml([1, 2], [2]), ml([3, 4], [2])
    prog = S.morphism_to_ssa(am.make_var(am.morph_add(a, b)))
    assert len(prog.bindings) == 1 and isinstance(S.ssa_loss_binding_val(prog), S.BindingRef)
    s = am.morph_add(a, a)
    prog = S.morphism_to_ssa(am.make_var(am.morph_mul(s, s)))      # the shared node is one binding
    assert [bb.op for bb in prog.bindings] == ["add", "mul"]
    prog = S.morphism_to_ssa(am.make_var(am.morph_reduce("mean", ml([1, 2, 3], [3]), [0])))
    assert [bb.op for bb in prog.bindings] == [("reduce", "mean")]
    prog = S.morphism_to_ssa(am.make_var(am.morph_transpose(ml([1, 2, 3, 4], [2, 2]))))
    assert [bb.op for bb in prog.bindings] == ["transpose"]
    W, x = ml([1, 2], [2]), ml([3, 4], [2])
    prog = S.morphism_to_ssa(am.make_var(am.morph_add(am.morph_mul(W, x), W)))
    joint = S.ssa_vjp(prog, [S.ssa_constant_id(prog, W)], S.ssa_loss_binding_val(prog))
    assert len(joint.outputs) == 2


# ------------------------------------------------------------------ group 2: ssa-realize outputs (test-ssa.scm:213-268)

@pytest.mark.parametrize("tree,expect", [
    (lambda: am.morph_add(ml([1, 2, 3], [3]), ml([4, 5, 6], [3])), [5, 7, 9]),
    (lambda: am.morph_mul(ml([1, 2, 3], [3]), ml([4, 5, 6], [3])), [4, 10, 18]),
    (lambda: am.morph_matmul(ml([1, 2, 3, 4], [2, 2]), ml([5, 6, 7, 8], [2, 2])), [19, 22, 43, 50]),
    (lambda: am.morph_reduce("mean", ml([1, 2, 3, 4], [4]), [0]), [2.5]),
    (lambda: am.morph_reduce("sum", ml([1, 2, 3, 4], [4]), [0]), [10]),
    (lambda: am.morph_transpose(ml([1, 2, 3, 4], [2, 2])), [1, 3, 2, 4]),
    (lambda: am.morph_add(am.morph_matmul(ml([1, 0, 0, 1], [2, 2]), ml([2, 3, 4, 5], [2, 2])), ml([1] * 4, [2, 2])),
     [3, 4, 5, 6]),
])
def test_ssa_realize_outputs(tree, expect):
    out = S.ssa_realize(S.morphism_to_ssa(am.make_var(tree())), oracle.realize)
    assert close(flat(out[0]), [float(e) for e in expect])


# ------------------------------------------------------------------ group 3: ssa-vjp gradients (test-ssa.scm:275-336)

def test_ssa_vjp_gradients():
    W, x = param([0.5, 1.0, 1.5, 2.0], [4]), inp([1, 2, 3, 4], [4])
    assert close(compile_and_realize(am.var_sum(am.var_mul(W, x)), [W])[1], [1, 2, 3, 4])
    W = param([0.1, 0.2, 0.3], [3])
    assert close(compile_and_realize(am.var_sum(W), [W])[1], [1, 1, 1])
    Z, b = inp([1, 2, 3, 4], [4]), param([0, 0, 0, 0], [4])
    assert close(compile_and_realize(am.var_sum(am.var_add(Z, b)), [b])[1], [1, 1, 1, 1])
    X, W = inp([1, 2, 3, 4, 5, 6], [3, 2]), param([0.1, 0.2, 0.3, 0.4], [2, 2])
    loss = am.var_mean(am.var_matmul(X, am.var_transpose(W, (1, 0))))
    assert close(compile_and_realize(loss, [W])[1], [1.5, 2.0, 1.5, 2.0])
    W1, W2 = param([1, 2, 3], [3]), param([4, 5, 6], [3])
    res = compile_and_realize(am.var_add(am.var_sum(W1), am.var_sum(W2)), [W1, W2])
    assert close(res[1], [1, 1, 1]) and close(res[2], [1, 1, 1])
    W, x = param([1, 2, 3], [3]), inp([1, 2, 3], [3])
    assert abs(compile_and_realize(am.var_mean(am.var_mul(W, x)), [W])[0][0] - 14.0 / 3.0) <= TOL


def _two_param_loss():
    """loss = sum(W1 * x) + 2 * sum(W2 * x) (test-ssa.scm:522-540)."""
    W1, W2 = param([1, 2, 3, 4], [4]), param([5, 6, 7, 8], [4])
    x = inp([1, 1, 1, 1], [4])
    two = am.make_var(ml([2.0], [1]))
    loss = am.var_add(am.var_sum(am.var_mul(W1, x)), am.var_mul(two, am.var_sum(am.var_mul(W2, x))))
    return loss, [W1, W2]


def test_two_params_distinct_gradients():
    loss, ps = _two_param_loss()
    res = compile_and_realize(loss, ps)
    assert close(res[1], [1, 1, 1, 1]) and close(res[2], [2, 2, 2, 2])


# ------------------------------------------------------------------ E1 / E3 / E4 (test-ssa.scm:917-1121)

def test_activation_gradients():
    xv = am.make_var(ml([-2, -1, 0, 1, 2], [5]), True)
    assert close(compile_and_realize(am.var_mean(am.var_relu(xv)), [xv])[1], [0, 0, 0, 0.2, 0.2])
    sig = lambda t: 1.0 / (1.0 + math.exp(-t))
    xv = am.make_var(ml([1, 2], [2]), True)
    assert close(compile_and_realize(am.var_mean(am.var_sigmoid(xv)), [xv])[1],
                 [0.5 * sig(t) * (1 - sig(t)) for t in (1.0, 2.0)])
    xv = am.make_var(ml([0.5, -0.5], [2]), True)
    assert close(compile_and_realize(am.var_mean(am.var_tanh(xv)), [xv])[1],
                 [0.5 * (1 - math.tanh(t) ** 2) for t in (0.5, -0.5)])


def test_relu_joint_is_smaller_than_its_decomposition():
    x = ml([-1, 0.5, 1, 2], [4])
    x1 = am.make_var(x, True)
    n1 = len(joint_of(am.var_mean(am.var_relu(x1)), [x1]).bindings)
    x2 = am.make_var(x, True)
    relu2 = am.var_mul(am.var_add(x2, am.var_abs(x2)), am.make_var(ml([0.5], [1])))
    n2 = len(joint_of(am.var_mean(relu2), [x2]).bindings)
    assert n1 < n2


def _dense_relu(xs, xshape, ws, wshape, bs):
    xv = am.make_var(ml(xs, xshape))
    Wv, bv = am.make_var(ml(ws, wshape), True), am.make_var(ml(bs, [wshape[1]]), True)
    return am.var_mean(am.var_relu(am.var_add(am.var_matmul(xv, Wv), bv))), [Wv, bv]


def test_dense_relu_gradient():
    loss, ps = _dense_relu([1, 0], [1, 2], [0.5] * 4, [2, 2], [0, 0])
    res = compile_and_realize(loss, ps)
    assert close(res[1], [0.5, 0.5, 0.0, 0.0]) and abs(res[0][0] - 0.5) <= TOL


def test_gradients_agree_with_tree_autograd():
    """The SSA joint program and the tree autograd give the same gradients
    for a small network (different op orders; f64 to 1e-12)."""
    rng = np.random.default_rng(2)
    x = am.make_var(am.morph_from_numpy(rng.uniform(0.5, 2.0, (6, 5))))
    w = am.make_var(am.morph_from_numpy(rng.standard_normal((5, 4))), True)
    b = am.make_var(am.morph_from_numpy(rng.standard_normal((1, 4))), True)
    h = am.var_add(am.var_matmul(x, w), b)
    loss = am.var_mean(am.var_mul(am.var_sigmoid(am.var_tanh(h)), am.var_exp(am.var_sqrt(am.var_abs(h)))))
    res = S.ssa_realize(joint_of(loss, [w, b]), oracle.realize)
    am.backward(loss)
    for got, v in zip(res[1:], (w, b)):
        np.testing.assert_allclose(np.asarray(got.values()), np.asarray(oracle.values(am.var_grad(v))),
                                   rtol=1e-12, atol=1e-14)


# ------------------------------------------------------------------ device

def _bitwise(a, b):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape and np.array_equal(a.reshape(-1).view(np.uint8), b.reshape(-1).view(np.uint8))


@pytest.mark.gpu
def test_ssa_on_device_bitwise(amc):
    """Every output of several joint programs realized on the device equals
    the oracle's bit for bit (arithmetic and matmul only, no libm calls)."""
    X, W = inp([1, 2, 3, 4, 5, 6], [3, 2]), param([0.1, 0.2, 0.3, 0.4], [2, 2])
    cases = [(am.var_mean(am.var_matmul(X, am.var_transpose(W, (1, 0)))), [W]), _two_param_loss(),
             _dense_relu([1, 2, 3, 4, 5, 6], [2, 3], [0.1] * 12, [3, 4], [0.1] * 4)]
    rng = np.random.default_rng(8)
    Xb = am.make_var(am.morph_from_numpy(rng.standard_normal((64, 48))))
    W1 = am.make_var(am.morph_from_numpy(rng.standard_normal((48, 32)) * 0.1), True)
    W2 = am.make_var(am.morph_from_numpy(rng.standard_normal((32, 8)) * 0.1), True)
    h = am.var_relu(am.var_matmul(Xb, W1))
    cases.append((am.var_mean(am.var_mul(am.var_matmul(h, W2), am.var_matmul(h, W2))), [W1, W2]))
    for loss, ps in cases:
        joint = joint_of(loss, ps)
        for got, ref in zip(S.ssa_realize(joint), S.ssa_realize(joint, oracle.realize)):
            _bitwise(got.values(), ref.values())


@pytest.mark.gpu
def test_ssa_realize_ctx_trace_and_replay(amc):
    """ssa-realize/ctx groups (test-ssa.scm:344-680): the trace records
    allocations, replay after finalize gives the trace's values, repeatedly,
    and two same-shape gradients stay distinct (no pool-slot aliasing)."""
    W, x = param([1, 2, 3, 4], [4]), inp([0.1, 0.2, 0.3, 0.4], [4])
    joint = joint_of(am.var_sum(am.var_mul(W, x)), [W])
    ctx = am.make_morphism_context()
    trace = [flat(r) for r in S.ssa_realize_ctx(ctx, joint)]
    assert am.context_stats(ctx)["allocations"] > 0
    am.finalize_context(ctx)
    assert am.context_stats(ctx)["mode"] == "replay"
    for _ in range(3):
        am.reset_context(ctx)
        assert [flat(r) for r in S.ssa_realize_ctx(ctx, joint)] == trace
    loss, ps = _two_param_loss()
    joint = joint_of(loss, ps)
    ctx = am.make_morphism_context()
    res = S.ssa_realize_ctx(ctx, joint)
    assert close(flat(res[1]), [1] * 4) and close(flat(res[2]), [2] * 4)
    am.finalize_context(ctx)
    for _ in range(5):
        am.reset_context(ctx)
        res = S.ssa_realize_ctx(ctx, joint)
        assert close(flat(res[1]), [1] * 4) and close(flat(res[2]), [2] * 4)
    # two-layer model and dense+relu: replay stable and equal to the oracle
    Xm = inp([1, 0, 0, 1], [2, 2])
    W1, W2 = param([0.1 * i for i in range(1, 9)], [4, 2]), param([0.1 * i for i in range(1, 13)], [3, 4])
    z2 = am.var_matmul(am.var_matmul(Xm, am.var_transpose(W1, (1, 0))), am.var_transpose(W2, (1, 0)))
    for loss, ps in ((am.var_mean(z2), [W1, W2]),
                     _dense_relu([1, 2, 3, 4, 5, 6], [2, 3], [0.1] * 12, [3, 4], [0.1] * 4)):
        joint = joint_of(loss, ps)
        ref = [r.values() for r in S.ssa_realize(joint, oracle.realize)]
        ctx = am.make_morphism_context()
        for got, r in zip(S.ssa_realize_ctx(ctx, joint), ref):
            _bitwise(got.values(), r)
        am.finalize_context(ctx)
        for _ in range(5):
            am.reset_context(ctx)
            for got, r in zip(S.ssa_realize_ctx(ctx, joint), ref):
                _bitwise(got.values(), r)


@pytest.mark.parametrize("name", ["add", "sub", "mul", "div", "pow", "negate", "abs", "sqrt", "exp", "log", "sin",
                                  "cos", "relu", "sigmoid", "tanh", "reshape", "transpose", "sum_keep", "mean_axis"])
def test_each_vjp_rule_agrees_with_tree_autograd(name):
    """Every rule of ssa-vjp (ssa.scm:713-983) against the tree autograd's
    rule for the same op (grad.scm), with broadcasting where the op takes
    two operands; gradients through the oracle, f64 to 1e-12."""
    rng = np.random.default_rng(sum(map(ord, name)))
    a = am.make_var(am.morph_from_numpy(rng.uniform(0.5, 2.0, (3, 4))), True)
    b = am.make_var(am.morph_from_numpy(rng.uniform(0.5, 2.0, (1, 4))), True)
    unary = {"negate": am.var_negate, "abs": am.var_abs, "sqrt": am.var_sqrt, "exp": am.var_exp,
             "log": am.var_log, "sin": am.var_sin, "cos": am.var_cos, "relu": am.var_relu,
             "sigmoid": am.var_sigmoid, "tanh": am.var_tanh}
    binary = {"add": am.var_add, "sub": am.var_sub, "mul": am.var_mul, "div": am.var_div, "pow": am.var_pow}
    params = [a, b] if name in binary else [a]
    if name in binary:
        y = binary[name](a, b)
    elif name in unary:
        y = unary[name](am.var_sub(a, am.make_var(ml([1.0], [1]))) if name in ("abs", "relu") else a)
    elif name == "reshape":
        y = am.var_reshape(a, (2, 6))
    elif name == "transpose":
        y = am.var_transpose(a, (1, 0))
    elif name == "sum_keep":
        y = am.var_sum(a, [1], True)
    else:
        y = am.var_mean(a, [0])
    w = am.make_var(am.morph_from_numpy(rng.standard_normal(y.value.shape)))
    loss = am.var_sum(am.var_mul(y, w))            # a non-uniform upstream gradient
    res = S.ssa_realize(joint_of(loss, params), oracle.realize)
    am.backward(loss)
    for got, p in zip(res[1:], params):
        ref = np.asarray(oracle.values(am.var_grad(p)))
        assert np.asarray(got.values()).shape == ref.shape
        np.testing.assert_allclose(np.asarray(got.values()), ref, rtol=1e-12, atol=1e-14, err_msg=name)


# ------------------------------------------------------------------ E2: the element-wise fusion pass (test-ssa.scm:810-870)

def test_fusion_pass_binding_counts_and_values():
    a = ml([-3.0, 2.0], [2])
    p0 = S.morphism_to_ssa(am.make_var(am.morph_negate(am.morph_abs(a))))
    p1 = S.ssa_element_wise_fusion_pass(p0)
    assert len(p0.bindings) - len(p1.bindings) == 1
    assert flat(S.ssa_realize(p1, oracle.realize)[0]) == [-3.0, -2.0]
    a = ml([1.0, 2.0], [2])
    b = am.morph_abs(a)
    p1 = S.ssa_element_wise_fusion_pass(S.morphism_to_ssa(am.make_var(am.morph_add(b, am.morph_negate(b)))))
    assert len(p1.bindings) == 3                       # b has two consumers: nothing merges
    c = am.morph_reduce("sum", am.morph_abs(ml([1.0, -2.0, 3.0, -4.0], [4])), [0])
    assert len(S.ssa_element_wise_fusion_pass(S.morphism_to_ssa(am.make_var(c))).bindings) == 2
    xv = am.make_var(ml([1.0, 2.0, 3.0], [3]), True)
    joint = S.ssa_element_wise_fusion_pass(joint_of(am.var_sum(am.var_negate(xv)), [xv]))
    assert close(flat(S.ssa_realize(joint, oracle.realize)[1]), [-1.0, -1.0, -1.0])


@pytest.mark.parametrize("dt", ["f64", "f32"])
def test_fusion_pass_composes_without_rounding_the_intermediate(dt):
    """A merged chain equals the unfused program in f64; in f32 it equals
    the double-precision composition stored once (compose-flat-combiners)."""
    rng = np.random.default_rng(12)
    xs, ys = rng.uniform(0.5, 2.0, 16), rng.uniform(0.5, 2.0, 16)
    x, y = am.morph_from_numpy(xs, dt), am.morph_from_numpy(ys, dt)
    tree = am.morph_mul(am.morph_sqrt(am.morph_add(am.morph_exp(x), y)), y)
    p0 = S.morphism_to_ssa(am.make_var(tree))
    p1 = S.ssa_element_wise_fusion_pass(p0)
    assert len(p1.bindings) < len(p0.bindings)
    got = np.asarray(S.ssa_realize(p1, oracle.realize)[0].values())
    if dt == "f64":
        np.testing.assert_array_equal(got, np.asarray(S.ssa_realize(p0, oracle.realize)[0].values()))
    else:
        x64, y64 = xs.astype(np.float32).astype(np.float64), ys.astype(np.float32).astype(np.float64)
        np.testing.assert_allclose(got, (np.sqrt(np.exp(x64) + y64) * y64).astype(np.float32), rtol=2e-7)


def test_ssa_mse_step_matches_the_linear_regression_oracle():
    """The C5 program through the SSA compiler: loss = mean((X w - y)^2) and
    its gradient w.r.t. w (2/N X^T (X w - y)), one gradient-descent step of
    which is what the fused linear-regression kernels replay.  The SSA
    gradient and loss agree with the oracle's step to 1e-12."""
    from amcuda import workloads as W
    rows, d, lr = 256, 8, 0.1
    X, y, _ = W.c5_inputs(rows, d)
    w0 = np.random.default_rng(3).standard_normal(d) * 0.1
    Xv = am.make_var(am.morph_from_numpy(X))
    wv = am.make_var(am.morph_from_numpy(w0.reshape(d, 1)), True)
    yv = am.make_var(am.morph_from_numpy(np.asarray(y).reshape(rows, 1)))
    r = am.var_sub(am.var_matmul(Xv, wv), yv)
    res = S.ssa_realize(joint_of(am.var_mean(am.var_mul(r, r)), [wv]), oracle.realize)
    loss, dw = float(np.asarray(res[0].values()).reshape(-1)[0]), np.asarray(res[1].values()).reshape(-1)
    w1, losses = oracle.linreg(X, y, w0, 1, lr)
    np.testing.assert_allclose(loss, losses[0], rtol=1e-12)
    np.testing.assert_allclose(w0 - lr * dw, w1, rtol=1e-12, atol=1e-15)
