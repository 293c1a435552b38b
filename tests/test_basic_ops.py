"""Element-wise and reduction constructors of the host mirror against the
reference's tests/test-basic-ops.scm (file:line per group): node kind,
broadcast shapes, dtype promotion and inference, comparisons, morph-map,
morph-reduce and batch-axis tracking.  CPU only; values through the oracle
where a case states them."""
import numpy as np
import pytest

import amcuda as am
from amcuda import fn
import oracle


def ml(vals, shape, dt="f64", ba=-1):
    return am.morph_from_list(vals, tuple(shape), dt, ba)


# ------------------------------------------------------------------ binary structure (test-basic-ops.scm:44-101)

@pytest.mark.parametrize("ctor,op", [(am.morph_add, "add"), (am.morph_sub, "sub"), (am.morph_mul, "mul"),
                                     (am.morph_div, "div"), (am.morph_pow, "pow")])
def test_binary_structure(ctor, op):
    r = ctor(ml([1, 2, 3], (3,)), ml([4, 5, 6], (3,)))
    assert isinstance(r, am.Expr) and r.op == op and len(r.operands) == 2 and r.shape == (3,)


# ------------------------------------------------------------------ broadcasting (:105-150)

@pytest.mark.parametrize("a,b,ctor,shape", [
    (ml([1, 2, 3], (3,)), ml([4, 5, 6], (3,)), am.morph_add, (3,)),
    (ml([[1, 2], [3, 4]], (2, 2)), ml([10], (1,)), am.morph_add, (2, 2)),
    (ml([[1, 2, 3], [4, 5, 6]], (2, 3)), ml([10, 20, 30], (3,)), am.morph_add, (2, 3)),
    (ml([[1, 2], [3, 4]], (2, 2)), ml([[10], [20]], (2, 1)), am.morph_add, (2, 2)),
    (ml([[[1, 2]]], (1, 1, 2), "f32"), ml([10, 20], (2,), "f32"), am.morph_mul, (1, 1, 2)),
    (ml([[[1]]], (1, 1, 1)), ml([[2, 3, 4]], (1, 3)), am.morph_add, (1, 1, 3)),
])
def test_broadcast_shapes(a, b, ctor, shape):
    assert ctor(a, b).shape == shape


def test_broadcast_values_through_the_oracle():
    r = am.morph_add(ml([[1, 2], [3, 4]], (2, 2)), ml([[10], [20]], (2, 1)))
    assert np.asarray(oracle.values(r)).tolist() == [[11, 12], [23, 24]]


# ------------------------------------------------------------------ promotion and unary dtypes (:154-298)

@pytest.mark.parametrize("d1,d2,out", [("f64", "f32", "f64"), ("f32", "s32", "f32"), ("s64", "s32", "s64"),
                                       ("s32", "f64", "f64"), ("s32", "s32", "s32")])
def test_type_promotion(d1, d2, out):
    assert am.morph_add(ml([1], (1,), d1), ml([2], (1,), d2)).dtype == out


@pytest.mark.parametrize("ctor,op", [(am.morph_sqrt, "sqrt"), (am.morph_exp, "exp"), (am.morph_log, "log"),
                                     (am.morph_sin, "sin"), (am.morph_negate, "negate"), (am.morph_abs, "abs")])
def test_unary_structure(ctor, op):
    r = ctor(ml([4.0, 9.0, 16.0], (3,)))
    assert isinstance(r, am.Expr) and r.op == op and len(r.operands) == 1 and r.shape == (3,)


@pytest.mark.parametrize("ctor,d,out", [(am.morph_sqrt, "s32", "f64"), (am.morph_sqrt, "f32", "f32"),
                                        (am.morph_exp, "s64", "f64"), (am.morph_log, "f64", "f64"),
                                        (am.morph_negate, "s32", "s32"), (am.morph_abs, "f64", "f64"),
                                        (am.morph_floor, "s64", "s64")])
def test_unary_dtype_inference(ctor, d, out):
    assert ctor(ml([1, 2], (2,), d)).dtype == out


# ------------------------------------------------------------------ comparisons (:303-371)

def test_comparisons():
    r = am.morph_gt(ml([3, 1, 4], (3,)), ml([2, 2, 2], (3,)))
    assert r.op == "gt" and len(r.operands) == 2 and r.shape == (3,) and r.dtype == "f64"
    assert np.asarray(oracle.values(r)).tolist() == [1.0, 0.0, 1.0]
    r = am.morph_lt(ml([1, 5], (2,), "s32"), ml([2, 4], (2,), "s32"))
    assert r.op == "lt" and r.dtype == "f64"
    assert am.morph_eq(ml([1, 2], (2,), "f32"), ml([1, 3], (2,), "f32")).op == "eq"
    assert am.morph_ge(ml([3, 2, 1], (3,)), ml([1, 2, 3], (3,))).op == "ge"
    assert am.morph_le(ml([1, 2], (2,), "s64"), ml([2, 1], (2,), "s64")).op == "le"
    assert am.morph_gt(ml([[1, 2], [3, 4]], (2, 2)), ml([2], (1,))).shape == (2, 2)
    assert am.morph_gt(ml([1, 2], (2,), "s32"), ml([2, 1], (2,), "s32")).dtype == "f64"


# ------------------------------------------------------------------ morph-map (:375-414)

def test_morph_map():
    r = am.morph_map(lambda x: x * x, ml([1, 2, 3], (3,)))
    assert r.op == "map" and len(r.operands) == 1 and r.shape == (3,)
    assert am.morph_map(lambda x: x + 10, ml([[1, 2], [3, 4]], (2, 2), "f32")).shape == (2, 2)
    assert am.morph_map(abs, ml([1, 2, 3], (3,), "s32")).dtype == "s32"
    assert am.morph_map(lambda x: x, ml([[1, 2], [3, 4]], (2, 2), ba=0)).batch_axis == 0
    r = am.morph_map(lambda x: fn.sin(x * 3.14159), ml([0.0, 1.0], (2,)))
    assert isinstance(r, am.Expr)
    np.testing.assert_allclose(oracle.values(r), [0.0, np.sin(3.14159)], rtol=0, atol=1e-15)


# ------------------------------------------------------------------ morph-reduce (:418-503)

def test_morph_reduce():
    r = am.morph_reduce("sum", ml([1, 2, 3, 4], (4,)))
    assert r.op == "reduce" and r.meta["op"] == "sum" and r.shape == () and r.dtype == "f64"
    assert am.morph_reduce("sum", ml([[1, 2], [3, 4]], (2, 2)), [0]).shape == (2,)
    assert am.morph_reduce("mean", ml([[1, 2, 3], [4, 5, 6]], (2, 3), "f32"), [1]).shape == (2,)
    assert am.morph_reduce("sum", ml([[1, 2], [3, 4]], (2, 2)), [0], True).shape == (1, 2)
    assert am.morph_reduce("max", ml(list(range(1, 9)), (2, 2, 2)), [0, 2]).shape == (2,)
    assert am.morph_reduce("prod", ml([[1, 2], [3, 4]], (2, 2), "f32")).shape == ()
    assert am.morph_reduce("sum", ml([[1, 2, 3], [4, 5, 6]], (2, 3)), [-1]).shape == (2,)
    assert am.morph_reduce("mean", ml([1, 2, 3, 4], (4,), "s32")).dtype == "f64"
    assert am.morph_reduce("sum", ml([1, 2, 3], (3,), "s64")).dtype == "s64"
    assert float(oracle.values(am.morph_reduce("max", ml(list(range(1, 9)), (2, 2, 2)), [0, 2]))[1]) == 8.0


# ------------------------------------------------------------------ batch axis (:508-571)

def test_batch_axis_tracking():
    b0 = ml([[1, 2], [3, 4]], (2, 2), ba=0)
    assert am.morph_add(ml([1, 2], (2,)), ml([3, 4], (2,))).batch_axis == -1
    assert am.morph_add(b0, ml([10, 20], (2,))).batch_axis == 0
    assert am.morph_add(b0, ml([[5, 6], [7, 8]], (2, 2), ba=0)).batch_axis == 0
    assert am.morph_sqrt(b0).batch_axis == 0
    assert am.morph_exp(ml([1, 2, 3], (3,))).batch_axis == -1
    assert am.morph_reduce("sum", b0, [0]).batch_axis == -1
    assert am.morph_reduce("sum", b0, [1]).batch_axis == 0
    assert am.morph_reduce("sum", b0, [0], True).batch_axis == 0


# ------------------------------------------------------------------ edge cases (:575-620)

def test_edge_cases():
    assert am.morph_reduce("sum", ml([1, 2, 3, 4], (4,)), []).shape == ()
    assert am.morph_reduce("max", ml([42], (1,))).shape == ()
    m = ml([1, 2, 3], (3,))
    assert am.morph_map(lambda x: x, m).shape == m.shape
    final = am.morph_sqrt(am.morph_add(am.morph_map(lambda x: x * x, m), ml([1], (1,))))
    assert final.op == "sqrt"
    np.testing.assert_allclose(oracle.values(final), np.sqrt([2.0, 5.0, 10.0]), rtol=1e-15)
    assert am.morph_mul(ml([[[1, 2]]], (1, 1, 2)), ml([3, 4], (2,))).shape == (1, 1, 2)


# ------------------------------------------------------------------ activation forwards (test-ssa.scm:874-915)

def test_activation_forward_values():
    import math
    vals = lambda m: list(np.asarray(oracle.values(m), dtype=np.float64))
    assert vals(am.morph_relu(ml([1.0, 2.0, 3.0], (3,)))) == [1.0, 2.0, 3.0]
    assert vals(am.morph_relu(ml([-1.0, -2.0, -3.0], (3,)))) == [0.0, 0.0, 0.0]
    assert vals(am.morph_relu(ml([-1.0, 2.0, -3.0, 4.0], (4,)))) == [0.0, 2.0, 0.0, 4.0]
    xs = [-2.0, -1.0, 0.0, 1.0, 2.0]
    np.testing.assert_allclose(vals(am.morph_sigmoid(ml(xs, (5,)))), [1.0 / (1.0 + math.exp(-x)) for x in xs],
                               rtol=0, atol=1e-9)
    xs = [-1.0, 0.0, 1.0]
    np.testing.assert_allclose(vals(am.morph_tanh(ml(xs, (3,)))),
                               [(math.exp(2 * x) - 1) / (math.exp(2 * x) + 1) for x in xs], rtol=0, atol=1e-9)
