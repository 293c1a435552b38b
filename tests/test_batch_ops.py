"""Batch combinators (the host mirror of batch-ops.scm).

CPU: shapes, batch-axis bookkeeping, errors, and values through the oracle,
against the reference's own known answers (tests/test-batch-ops.scm of the
reference, groups 1-5).  GPU: the same trees and deeper fold/scan trees
realized on the device, bit-exact against the oracle."""
import numpy as np
import pytest

import amcuda as am
import oracle


def ml(vals, shape, dt="f64"):
    return am.morph_from_list(vals, shape, dt)


def flat(m):
    return list(np.asarray(oracle.values(m), dtype=np.float64).ravel())


# ------------------------------------------------------------------ group 1: batch dimension management
# (test-batch-ops.scm:58-146)

def test_add_and_remove_batch_dimension():
    m = ml([1.0, 2.0, 3.0], (3,))
    b = am.add_batch_dimension(m)
    assert b.shape == (1, 3) and am.batched(b) and b.batch_axis == 0 and am.batch_size(b) == 1
    assert flat(b) == [1.0, 2.0, 3.0]
    b1 = am.add_batch_dimension(ml([1.0, 2.0, 3.0, 4.0], (2, 2)), 1)
    assert b1.shape == (2, 1, 2) and b1.batch_axis == 1
    m2 = am.remove_batch_dimension(b)
    assert m2.shape == (3,) and not am.batched(m2) and flat(m2) == [1.0, 2.0, 3.0]
    with pytest.raises(ValueError):
        am.add_batch_dimension(b)
    with pytest.raises(ValueError):
        am.remove_batch_dimension(m)


def test_extract_stack_concat():
    data = ml([1.0, 2.0, 3.0, 4.0, 5.0, 6.0], (3, 2))
    e1 = am.extract_batch_element(data, 1)
    assert e1.shape == (2,) and not am.batched(e1)
    assert [flat(am.extract_batch_element(data, i)) for i in range(3)] == [[1.0, 2.0], [3.0, 4.0], [5.0, 6.0]]
    with pytest.raises(ValueError):
        am.extract_batch_element(data, 3)
    s = am.stack_into_batch([ml([1.0, 2.0], (2,)), ml([3.0, 4.0], (2,)), ml([5.0, 6.0], (2,))])
    assert s.shape == (3, 2) and am.batched(s) and s.batch_axis == 0
    assert flat(am.stack_into_batch([ml([1.0, 2.0], (2,)), ml([3.0, 4.0], (2,))])) == [1.0, 2.0, 3.0, 4.0]
    sa = am.stack_into_batch([ml([1.0, 2.0], (2,)), ml([3.0, 4.0], (2,))])
    sb = am.stack_into_batch([ml([5.0, 6.0], (2,)), ml([7.0, 8.0], (2,)), ml([9.0, 10.0], (2,))])
    assert am.concat_batch([sa, sb]).shape == (5, 2)
    with pytest.raises(ValueError):
        am.stack_into_batch([sa])
    with pytest.raises(ValueError):
        am.concat_batch([ml([1.0], (1,))])


# ------------------------------------------------------------------ group 2: core combinators
# (test-batch-ops.scm:148-221)

def test_batch_map_reduce_zip():
    m = ml([1.0, 2.0, 3.0, 4.0, 5.0, 6.0], (3, 2))
    r = am.batch_map(lambda x: x, m)
    assert r.shape == (3, 2) and flat(r) == [1.0, 2.0, 3.0, 4.0, 5.0, 6.0]
    assert flat(am.batch_map(am.morph_negate, ml([1.0, 2.0, 3.0, 4.0], (2, 2)))) == [-1.0, -2.0, -3.0, -4.0]
    s = am.stack_into_batch([ml([1.0, 2.0, 3.0, 4.0], (4,)), ml([5.0, 6.0, 7.0, 8.0], (4,)),
                             ml([9.0, 10.0, 11.0, 12.0], (4,))])
    r = am.batch_map(lambda x: am.morph_reduce("sum", x), s)
    assert r.shape == (3,) and flat(r) == [10.0, 26.0, 42.0]
    assert am.batch_reduce("sum", m).shape == (2,) and flat(am.batch_reduce("sum", m)) == [9.0, 12.0]
    assert am.batch_reduce("sum", ml([1.0, 2.0, 3.0, 4.0], (2, 2)), True).shape == (1, 2)
    z = am.batch_zip(am.morph_add, ml([1.0, 2.0, 3.0, 4.0], (2, 2)), ml([5.0, 6.0, 7.0, 8.0], (2, 2)))
    assert flat(z) == [6.0, 8.0, 10.0, 12.0]
    with pytest.raises(ValueError):
        am.batch_zip(am.morph_add, ml([1.0, 2.0], (2, 1)), ml([1.0, 2.0, 3.0], (3, 1)))


def test_batch_fold_and_scan():
    data = ml([1.0, 2.0, 3.0, 4.0, 5.0, 6.0], (3, 2))
    zero = ml([0.0, 0.0], (2,))
    assert flat(am.batch_fold(am.morph_add, zero, data)) == flat(am.batch_reduce("sum", data))
    s = am.stack_into_batch([ml([1.0, 2.0], (2,)), ml([3.0, 4.0], (2,)), ml([5.0, 6.0], (2,))])
    scan = am.batch_scan(am.morph_add, zero, s)
    assert scan.shape == (3, 2) and flat(scan) == [1.0, 2.0, 4.0, 6.0, 9.0, 12.0]


# ------------------------------------------------------------------ group 3: broadcasting
# (test-batch-ops.scm:223-258)

def test_broadcast_to_batch():
    b = am.broadcast_to_batch(ml([1.0, 2.0, 3.0], (3,)), 4)
    assert am.batched(b) and am.batch_size(b) == 1 and b.shape == (1, 3)
    one = am.add_batch_dimension(ml([1.0, 2.0], (2,)))
    assert am.broadcast_to_batch(one, 8) is one
    two = am.stack_into_batch([ml([1.0, 2.0], (2,)), ml([3.0, 4.0], (2,))])
    assert am.broadcast_to_batch(two, 2) is two
    with pytest.raises(ValueError):
        am.broadcast_to_batch(two, 5)


# ------------------------------------------------------------------ group 4: batch-aware arithmetic
# (test-batch-ops.scm:260-318)

def test_batch_aware_arithmetic():
    assert flat(am.morph_add_batch(ml([1.0, 2.0, 3.0, 4.0], (2, 2)), ml([10.0, 20.0, 30.0, 40.0], (2, 2)))) == \
        [11.0, 22.0, 33.0, 44.0]
    a, b = ml([1.0, 2.0, 3.0, 4.0, 5.0, 6.0], (2, 3)), ml([10.0, 20.0, 30.0], (3,))
    assert flat(am.morph_add_batch(a, b)) == [11.0, 22.0, 33.0, 14.0, 25.0, 36.0]
    assert flat(am.morph_add_batch(b, a)) == [11.0, 22.0, 33.0, 14.0, 25.0, 36.0]
    assert flat(am.morph_add_batch(ml([1.0, 2.0], (2,)), ml([3.0, 4.0], (2,)))) == [4.0, 6.0]
    assert flat(am.morph_mul_batch(ml([1.0, 2.0, 3.0, 4.0], (2, 2)), ml([2.0, 3.0], (2,)))) == [2.0, 6.0, 6.0, 12.0]
    assert flat(am.morph_sub_batch(ml([5.0, 6.0, 7.0, 8.0], (2, 2)), ml([1.0, 2.0, 3.0, 4.0], (2, 2)))) == [4.0] * 4
    assert flat(am.morph_div_batch(ml([6.0, 8.0, 12.0, 16.0], (2, 2)), ml([2.0, 4.0, 3.0, 8.0], (2, 2)))) == \
        [3.0, 2.0, 4.0, 2.0]
    # a batched operand with the other given a size-1 batch axis
    sb = am.stack_into_batch([ml([1.0, 2.0], (2,)), ml([3.0, 4.0], (2,))])
    assert flat(am.morph_add_batch(sb, ml([10.0, 20.0], (2,)))) == [11.0, 22.0, 13.0, 24.0]
    with pytest.raises(ValueError):
        am.morph_add_batch(am.stack_into_batch([ml([1.0, 2.0], (2,))] * 2),
                           am.stack_into_batch([ml([1.0, 2.0], (2,))] * 3))


# ------------------------------------------------------------------ group 5: batched matmul
# (test-batch-ops.scm:320-384)

def test_batch_matmul():
    A = ml([1.0, 2.0, 3.0, 4.0], (2, 2))
    eye = ml([1.0, 0.0, 0.0, 1.0], (2, 2))
    assert flat(am.morph_batch_matmul(A, eye)) == [1.0, 2.0, 3.0, 4.0]
    assert am.morph_batch_matmul(ml([1.0] * 12, (2, 2, 3)), ml([1.0] * 12, (3, 4))).shape == (2, 2, 4)
    A3 = am.stack_into_batch([ml([1.0, 2.0, 3.0, 4.0], (2, 2)), ml([5.0, 6.0, 7.0, 8.0], (2, 2))])
    assert flat(am.morph_batch_matmul(A3, eye)) == [1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0]
    assert am.morph_batch_matmul(ml([1.0] * 24, (3, 2, 4)), ml([1.0] * 60, (3, 4, 5))).shape == (3, 2, 5)
    Ab = am.stack_into_batch([ml([1.0, 2.0], (1, 2)), ml([3.0, 4.0], (1, 2))])
    Bb = am.stack_into_batch([ml([5.0, 6.0], (2, 1)), ml([7.0, 8.0], (2, 1))])
    assert flat(am.morph_batch_matmul(Ab, Bb)) == [17.0, 53.0]
    with pytest.raises(ValueError):
        am.morph_batch_matmul(ml([1.0] * 6, (2, 3)), ml([1.0] * 6, (1, 2, 3)))


# ------------------------------------------------------------------ device realize, bit-exact against the oracle

def _rand(rng, shape, dt):
    if dt in ("f32", "f64"):
        return rng.standard_normal(shape).astype(np.float32 if dt == "f32" else np.float64)
    return rng.integers(-50, 50, size=shape).astype(np.int32 if dt == "s32" else np.int64)


@pytest.mark.gpu
@pytest.mark.parametrize("dt", ["f32", "f64", "s32"])
def test_batch_trees_on_device_bitwise(amc, dt):
    rng = np.random.default_rng(17)
    x = am.morph_from_numpy(_rand(rng, (64, 5, 7), dt))
    w = am.morph_from_numpy(_rand(rng, (7, 3), dt))
    y = am.morph_from_numpy(_rand(rng, (64, 5, 7), dt))
    zero = am.morph_from_numpy(np.zeros((5, 7), dtype=_rand(rng, (1,), dt).dtype))
    exprs = [
        am.batch_map(lambda e: am.morph_map(lambda v: v * v - v, e), x),
        am.batch_reduce("sum", x),
        am.batch_zip(am.morph_mul, x, y),
        am.batch_fold(am.morph_add, zero, x),                     # 64 chained adds
        am.batch_scan(am.morph_add, zero, x),                     # 64 running sums, stacked
        am.batch_scan(lambda acc, e: am.morph_sub(e, acc), zero, x),   # alternating signs
        am.morph_add_batch(x, am.extract_batch_element(y, 3)),
    ]
    if dt != "s32":
        exprs.append(am.morph_batch_matmul(x, w))
    for e in exprs:
        got, ref = np.asarray(amc.realize(e).values()), np.asarray(oracle.values(e))
        assert got.shape == ref.shape and got.dtype == ref.dtype
        assert np.array_equal(got.reshape(-1).view(np.uint8), ref.reshape(-1).view(np.uint8)), "not bit-identical"


# ------------------------------------------------------------------ fold / scan as one SCAN node

_STEPS = {
    "add": am.morph_add,
    "e_minus_acc": lambda acc, e: am.morph_sub(e, acc),
    "decay": lambda acc, e: am.morph_add(am.morph_map(lambda t: t * 0.5 - 1, acc), e),
    "relu_sq": lambda acc, e: am.morph_relu(am.morph_add(acc, am.morph_mul(e, e))),
    "lifted_const": lambda acc, e: acc * 3 + e,
    "max_like": lambda acc, e: am.morph_add(am.morph_mul(am.morph_gt(acc, e), am.morph_sub(acc, e)), e),
}


def _scan_case(rng, dt, shape=(9, 4, 3)):
    x = am.morph_from_numpy(_rand(rng, shape, dt))
    init = am.morph_from_numpy(_rand(rng, shape[1:], dt))
    return x, init


@pytest.mark.parametrize("dt", ["f32", "f64", "s32"])
@pytest.mark.parametrize("name", sorted(_STEPS))
def test_fold_step_program_pinned_by_oracle_steps(dt, name):
    """The compiled step program, applied by the oracle one step at a time
    (acc <- map(prog, acc, x[i]) stored in the accumulator dtype), gives
    bit-for-bit the reference's per-element tree for both fold and scan."""
    from amcuda import batch as B
    rng = np.random.default_rng(3)
    x, init = _scan_case(rng, dt)
    fn = _STEPS[name]
    accs, prog = B._fold_steps(fn, init, x)
    tree_fold = am.batch_fold(fn, init, x)
    if accs[-1].dtype != init.dtype:
        assert prog is None and "scan" not in tree_fold.meta      # the dtype changes: stays a tree
        return
    assert prog is not None and tree_fold.meta["scan"][2] == prog
    acc = init
    steps = []
    for i in range(x.shape[0]):
        e = am.extract_batch_element(x, i)
        acc = oracle.realize(am.Expr("map", [acc, e], acc.shape, init.dtype, {"prog": prog}))
        steps.append(oracle.values(acc))
    ref = oracle.values(tree_fold)
    assert np.array_equal(np.asarray(steps[-1]).view(np.uint8), np.asarray(ref).view(np.uint8))
    scan = am.batch_scan(fn, init, x)
    assert scan.meta["scan"][3] is True
    assert np.array_equal(np.stack(steps).view(np.uint8), np.asarray(oracle.values(scan)).view(np.uint8))


def test_fold_step_program_refusals():
    from amcuda import batch as B
    x = ml([float(i) for i in range(12)], (4, 3))
    init = ml([0.0, 0.0, 0.0], (3,))
    assert B._fold_steps(am.morph_add, init, x)[1] == [(1, 0, 0.0), (1, 1, 0.0), (40, 0, 0.0)]
    # a step that is not element-wise, a shape that broadcasts, the identity on acc
    assert B._fold_steps(lambda a, e: am.morph_add(a, am.morph_reduce("sum", e, [0], True)), init, x)[1] is None
    assert B._fold_steps(am.morph_add, ml([0.0], (1,)), x)[1] is None
    assert B._fold_steps(lambda a, e: a, init, x)[1] is None
    # an operand from outside the step (a full-shape array) is not a constant
    w = ml([1.0, 2.0, 3.0], (3,))
    assert B._fold_steps(lambda a, e: am.morph_add(am.morph_mul(a, w), e), init, x)[1] is None
    # an empty batch: the fold is init itself
    assert am.batch_fold(am.morph_add, init, am.morph_from_numpy(np.zeros((0, 3)))) is init


def _oracle_dag(m, memo):
    """The oracle's value of a tree, each shared node realized once (a step
    that reads the accumulator twice makes the per-element tree a DAG whose
    paths double with every element)."""
    if not isinstance(m, am.Expr):
        return m
    if id(m) not in memo:
        ops = [_oracle_dag(o, memo) for o in m.operands]
        memo[id(m)] = oracle.realize(am.Expr(m.op, ops, m.shape, m.dtype, m.meta, m.batch_axis))
    return memo[id(m)]


def _scan_device_cases(dt):
    rng = np.random.default_rng(11)
    x, init = _scan_case(rng, dt, (37, 33, 5))
    xt = am.morph_transpose(am.morph_from_numpy(_rand(rng, (33, 5, 37), dt)), (2, 0, 1))
    for name in sorted(_STEPS):
        for src in (x, xt):
            for tree in (am.batch_fold(_STEPS[name], init, src), am.batch_scan(_STEPS[name], init, src)):
                yield name, tree, np.asarray(oracle.values(_oracle_dag(tree, {})))
    # one element, and a strided init (every other column of a wider array)
    one = am.morph_from_numpy(_rand(rng, (1, 33, 5), dt))
    wide = am.morph_from_numpy(_rand(rng, (33, 10), dt))
    init_s = am.morph_slice(wide, [0, 0], [33, 10], [1, 2])
    for tree in (am.batch_scan(am.morph_add, init, one), am.batch_fold(am.morph_sub, init_s, x)):
        yield "edge", tree, np.asarray(oracle.values(_oracle_dag(tree, {})))


@pytest.mark.parametrize("dt", ["f32", "f64", "s32"])
def test_scan_device_cases_oracle_cost(dt):
    """The references of the device test below come from the oracle in
    linear time (shared nodes realized once)."""
    n = sum(1 for _ in _scan_device_cases(dt))
    assert n == len(_STEPS) * 4 + 2


@pytest.mark.gpu
@pytest.mark.parametrize("dt", ["f32", "f64", "s32"])
def test_scan_node_on_device_bitwise(amc, dt):
    """Fold and scan of element-wise steps run as one SCAN launch, bit-exact
    against the oracle's per-element tree; a strided (transposed) batch and
    a dtype-changing step (left as a tree) too."""
    for name, tree, ref in _scan_device_cases(dt):
        p = amc.Plan(tree)
        if "scan" in tree.meta:
            assert p.stats()["launches"] == 1, name
        p.execute()
        got = np.asarray(p.result().values())
        assert got.shape == ref.shape and got.dtype == ref.dtype
        assert np.array_equal(got.reshape(-1).view(np.uint8), ref.reshape(-1).view(np.uint8)), name
