"""Parity of the device realize path (libamcuda through its C ABI) with the
oracle and with the reference's known answers."""
import json
from pathlib import Path

import numpy as np
import pytest

import oracle
from golden_dsl import build

pytestmark = pytest.mark.gpu

CASES = json.loads((Path(__file__).parent / "golden" / "known_answers.json").read_text())["cases"]


@pytest.mark.parametrize("c", CASES, ids=[c["name"] for c in CASES])
def test_device_known_answer(amc, c):
    res = amc.realize(build(c["expr"]))
    if c["shape"] is not None:
        assert list(res.shape) == c["shape"]
    if c["dtype"] is not None:
        assert res.dtype == c["dtype"]
    if c["values"] is not None:
        got = np.asarray(res.values(), dtype=np.float64).reshape(-1)
        exp = np.asarray(c["values"], dtype=np.float64).reshape(-1)
        np.testing.assert_allclose(got, exp, rtol=0, atol=c["tol"] if c["tol"] else 0)
    # and bit-for-bit (or within the case tolerance) equal to the oracle
    ref = oracle.realize(build(c["expr"]))
    np.testing.assert_allclose(np.asarray(res.values(), np.float64), np.asarray(ref.values(), np.float64),
                               rtol=c["tol"] if c["tol"] else 0, atol=0)


def _same(a, b):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape and a.dtype == b.dtype
    a, b = a.reshape(-1), b.reshape(-1)
    assert np.array_equal(a.view(np.uint8), b.view(np.uint8)), np.max(np.abs(a.astype(np.float64) - b))


@pytest.mark.parametrize("dtype", ["f64", "s32"])
def test_c1_fused_view_map_reduce_bit_exact(amc, dtype):
    """Config 1 at full size: sum_j x[2048j+i]^2 + y[2048j+i] (1024 outputs)."""
    from amcuda import workloads as W
    xm, ym = W.c1_inputs_morph(dtype)
    tree = W.c1_tree(xm, ym)
    dev = amc.realize(tree).values()
    ref = oracle.realize(W.c1_tree(xm, ym)).values()
    _same(dev, ref)
    assert dev.shape == (1024,)


def test_c1_plan_is_one_fused_launch(amc):
    from amcuda import workloads as W
    xm, ym = W.c1_inputs_morph("f64")
    p = amc.Plan(W.c1_tree(xm, ym))
    st = p.stats()
    assert st["launches"] == 1 and st["buffers"] == 1


@pytest.mark.parametrize("batch,length", [(2, 1 << 14), (3, 4096 + 64 * 37)])
def test_c2_filter_bank_bit_exact_small(amc, batch, length):
    from amcuda import workloads as W
    x = np.stack([W.c2_signal(s, length) for s in range(batch)])
    h = W.c2_prototype()
    xm, hm = amc.morph_from_numpy(x), amc.morph_from_numpy(h)
    tree = W.c2_tree(xm, hm)
    p = amc.Plan(tree)
    p.execute()
    dev = p.result().values()
    ref = oracle.realize(W.c2_tree(xm, hm)).values()
    _same(dev, ref)
    assert dev.shape == (batch, W.c2_frames(length), 64)


def test_c2_streaming_kernel_matches_generic_reduction(amc):
    """The FIR kernel against the generic ordered reduction of the same tree
    (forced by an identity map that hides the pattern): bitwise equal."""
    from amcuda import workloads as W
    L = 1 << 17
    x = np.stack([W.c2_signal(s, L) for s in range(2)])
    h = W.c2_prototype()
    xm, hm = amc.morph_from_numpy(x), amc.morph_from_numpy(h)
    fast = W.c2_tree(xm, hm)
    prod = fast.operands[0]
    slow = amc.morph_reduce("sum", amc.morph_map(lambda v: v * 1.0, prod), (2,))
    pf, ps = amc.Plan(fast), amc.Plan(slow)
    pf.execute(), ps.execute()
    _same(pf.result().values(), ps.result().values())


def _rand(rng, shape, dtype):
    if dtype in ("f32", "f64"):
        return rng.standard_normal(shape).astype(np.float32 if dtype == "f32" else np.float64)
    return rng.integers(-50, 50, size=shape).astype(np.int32 if dtype == "s32" else np.int64)


@pytest.mark.parametrize("dtype", ["f32", "f64", "s32", "s64"])
def test_fused_chains_match_oracle_bitwise(amc, dtype):
    rng = np.random.default_rng(3)
    a = amc.morph_from_numpy(_rand(rng, (37, 19), dtype))
    b = amc.morph_from_numpy(_rand(rng, (19,), dtype))
    c = amc.morph_from_numpy(_rand(rng, (37, 1), dtype))
    exprs = [
        amc.morph_add(amc.morph_mul(a, b), c),
        amc.morph_sub(amc.morph_transpose(amc.morph_mul(a, a)), amc.morph_transpose(a)),
        amc.morph_reduce("sum", amc.morph_mul(amc.morph_add(a, b), c), (0,)),
        amc.morph_reduce("sum", amc.morph_slice(amc.morph_add(a, c), (1, 2), (37, 19), (3, 2)), (1,), True),
        amc.morph_reduce("prod", amc.morph_slice(a, (0, 0), (37, 19), (9, 5)), (0, 1)),
        amc.morph_reduce("mean", amc.morph_abs(a), (1,)),
        amc.morph_map(lambda v: v * v - 3 * v + 1, amc.morph_transpose(a)),
        amc.morph_gt(a, b),
        amc.morph_reshape(amc.morph_transpose(a), (19 * 37,)),
        amc.morph_reduce("sum", amc.morph_pad(a, [(1, 2), (3, 0)], "reflect"), (0,)),
    ]
    if dtype in ("f32", "f64"):
        exprs.append(amc.morph_reduce("max", amc.morph_div(a, amc.morph_add(amc.morph_abs(c), c)), (0,)))
        exprs.append(amc.morph_reduce("min", a, (0, 1), True))
    for e in exprs:
        _same(amc.realize(e).values(), oracle.realize(e).values())


@pytest.mark.parametrize("dtype", ["f32", "f64", "s32", "s64"])
@pytest.mark.parametrize("R,O", [(1, 5), (7, 8), (512, 13), (3000, 1000)])
def test_staged_reduction_bitwise(amc, dtype, R, O):
    """Reductions over the leading axis of an (R, O) tree with few outputs
    (the staged ordered reduction: 8 adjacent outputs per CTA, leaf values
    copied into shared memory, ascending fold); R = 3000 takes several
    chunks.  Bit-exact against the oracle."""
    rng = np.random.default_rng(R + O)
    x = amc.morph_from_numpy(_rand(rng, (R, O), dtype))
    y = amc.morph_from_numpy(_rand(rng, (R, O), dtype))
    exprs = [
        amc.morph_reduce("sum", amc.morph_add(amc.morph_mul(x, x), y), (0,)),
        amc.morph_reduce("mean", amc.morph_abs(x), (0,)),
        amc.morph_reduce("sum", amc.morph_map(lambda v: v - 3, x), (0,), True),
    ]
    if dtype in ("f32", "f64"):
        exprs.append(amc.morph_reduce("max", amc.morph_sub(x, y), (0,)))
    for e in exprs:
        _same(amc.realize(e).values(), oracle.realize(e).values())


def test_transcendentals_within_f64_tolerance(amc):
    rng = np.random.default_rng(5)
    a = amc.morph_from_numpy(rng.uniform(0.1, 3.0, (64, 33)))
    for f in (amc.morph_sqrt, amc.morph_exp, amc.morph_log, amc.morph_sin, amc.morph_cos, amc.morph_tan,
              amc.morph_sigmoid, amc.morph_tanh, amc.morph_relu):
        e = amc.morph_reduce("sum", f(a), (1,))
        np.testing.assert_allclose(amc.realize(e).values(), oracle.realize(e).values(), rtol=1e-12, atol=0)


def test_integer_max_reduction_is_rejected(amc):
    a = amc.morph_from_numpy(np.arange(6, dtype=np.int32))
    with pytest.raises(amc.AmcError):
        amc.realize(amc.morph_reduce("max", a))


def test_long_reduction_tree_path(amc):
    rng = np.random.default_rng(9)
    x = rng.standard_normal(1 << 21)
    e = amc.morph_reduce("sum", amc.morph_map(lambda v: v * v, amc.morph_from_numpy(x)))
    got = float(amc.realize(e).values())
    ref = float(oracle.realize(e).values())
    assert abs(got - ref) <= 1e-12 * abs(ref)


def test_structural_gathers_match_oracle(amc):
    rng = np.random.default_rng(11)
    img = amc.morph_from_numpy(rng.standard_normal((2, 3, 7, 6)))
    for e in [
        amc.im2col_morph(img, (3, 2), (2, 1), (1, 2)),
        amc.col2im_morph(amc.im2col_morph(img, (3, 3), 1, 1), (2, 3, 7, 6), (3, 3), 1, 1),
        amc.morph_pad(amc.morph_transpose(img, (0, 2, 1, 3)), [(0, 0), (2, 1), (1, 1), (0, 3)], "edge"),
        amc.morph_pad(img, [(0, 0), (1, 0), (0, 2), (3, 3)], "constant", -7.5),
        amc.morph_stack([amc.morph_slice(img, (0, 0, 0, 0), (2, 3, 6, 6), (1, 1, 2, 3)),
                         amc.morph_slice(img, (0, 0, 1, 1), (2, 3, 7, 6), (1, 1, 2, 3))], 2),
        amc.morph_concat([img, amc.morph_mul(img, img)], 3),
    ]:
        _same(amc.realize(e).values(), oracle.realize(e).values())


def test_matmul_family_matches_oracle_bitwise(amc):
    rng = np.random.default_rng(13)
    for dt in ("f64", "f32"):
        A = amc.morph_from_numpy(_rand(rng, (70, 45), dt))
        B = amc.morph_from_numpy(_rand(rng, (45, 66), dt))
        v = amc.morph_from_numpy(_rand(rng, (45,), dt))
        for e in [amc.morph_matmul(A, B), amc.morph_matmul(amc.morph_transpose(B), amc.morph_transpose(A)),
                  amc.morph_matvec(A, v), amc.morph_dot(v, v)]:
            _same(amc.realize(e).values(), oracle.realize(e).values())


def test_attention_node_matches_oracle(amc):
    rng = np.random.default_rng(17)
    for dt, tol in (("f64", 1e-12), ("f32", 1e-5)):
        q = amc.morph_from_numpy(_rand(rng, (2, 3, 40, 8), dt))
        k = amc.morph_from_numpy(_rand(rng, (2, 3, 40, 8), dt))
        v = amc.morph_from_numpy(_rand(rng, (2, 3, 40, 5), dt))
        e = amc.attention_morphism(q, k, v)
        got, ref = amc.realize(e).values(), oracle.realize(e).values()
        assert np.max(np.abs(got.astype(np.float64) - ref)) <= tol * np.max(np.abs(ref))


def test_attention_node_tensor_core_shape(amc):
    """A contiguous f32 attention with head dim 64 and n % 128 == 0 plans the
    tcgen05 kernel (TF32 operands): within 2e-3 of the output scale."""
    rng = np.random.default_rng(18)
    q, k, v = (rng.standard_normal((1, 2, 256, 64)).astype(np.float32) for _ in range(3))
    e = amc.attention_morphism(amc.morph_from_numpy(q), amc.morph_from_numpy(k), amc.morph_from_numpy(v))
    plan = amc.Plan(e)
    assert plan.stats()["launches"] == 3
    plan.execute()
    got, ref = plan.result().values(), oracle.realize(e).values()
    assert np.max(np.abs(got.astype(np.float64) - ref)) <= 2e-3 * np.max(np.abs(ref))


@pytest.mark.parametrize("C,H,W,K,ksz,stride,pad,tol", [
    (64, 16, 16, 64, 3, 1, 1, 2e-3),     # implicit-GEMM tensor-core kernel (TF32)
    (3, 9, 7, 5, 3, 2, 1, 1e-6),         # direct kernel, double accumulation
    (2, 6, 6, 4, 2, 1, 0, 1e-6),
])
def test_conv_pattern_lowering(amc, C, H, W, K, ksz, stride, pad, tol):
    """reshape(matmul(W, im2col(X))) on one image is planned as a convolution
    (detect-conv2d-pattern, realization.scm:136-164), no column matrix."""
    rng = np.random.default_rng(19)
    x = rng.standard_normal((C, H, W)).astype(np.float32)
    w = (rng.standard_normal((K, C * ksz * ksz)) * np.sqrt(2.0 / (C * ksz * ksz))).astype(np.float32)
    oh, ow = 1 + (H + 2 * pad - ksz) // stride, 1 + (W + 2 * pad - ksz) // stride
    e = amc.morph_reshape(amc.morph_matmul(amc.morph_from_numpy(w),
                                           amc.im2col_morph(amc.morph_from_numpy(x), ksz, stride, pad)), (K, oh, ow))
    got = np.asarray(amc.realize(e).values(), np.float64)
    ref = np.asarray(oracle.realize(e).values(), np.float64)
    assert got.shape == (K, oh, ow)
    assert np.max(np.abs(got - ref)) <= tol * np.max(np.abs(ref))


@pytest.mark.parametrize("shape,perm,dt", [((100, 70), (1, 0), "f64"), ((3, 50, 40), (0, 2, 1), "s32"),
                                           ((20, 33, 45), (2, 0, 1), "f32"), ((7, 5, 64, 3), (1, 3, 0, 2), "s64")])
def test_transposed_view_copy(amc, shape, perm, dt):
    """A reshape of a transposed view copies it in logical row-major order
    (execute-affine-morphism, realization.scm:849-862); the copy goes through
    shared-memory tiles when the source's unit-stride axis is not innermost.
    Bit-exact against the oracle."""
    rng = np.random.default_rng(21)
    x = _rand(rng, shape, dt)
    n = int(np.prod(shape))
    e = amc.morph_reshape(amc.morph_transpose(amc.morph_from_numpy(x), perm), (n,))
    got, ref = amc.realize(e).values(), oracle.realize(e).values()
    assert np.array_equal(np.asarray(got), np.asarray(ref))
    assert np.array_equal(np.asarray(got).reshape(-1), np.transpose(x, perm).reshape(-1))


def test_plan_rejects_bad_trees(amc):
    a = amc.morph_from_numpy(np.zeros((4, 4)))
    with pytest.raises(ValueError):
        amc.morph_slice(a, (0, 0), (5, 4))
    bad = amc.morph_reshape(a, (16,))
    bad.shape = (17,)  # corrupt the node: the planner must refuse it
    with pytest.raises(amc.AmcError):
        amc.realize(bad)


def test_leaf_residency_and_host_changed(amc):
    """A concrete leaf is uploaded once and stays on the device across
    realizes; after an in-place host write, host_changed() makes the next
    realize see the new values (the in-place parameter updates of the
    reference's training loops)."""
    x = amc.morph_from_numpy(np.arange(6, dtype=np.float64))
    e = amc.morph_reduce("sum", amc.morph_mul(x, x))
    assert float(amc.realize(e).values()) == 55.0
    dev = x._dev
    assert dev is not None
    assert float(amc.realize(e).values()) == 55.0 and x._dev is dev   # no re-upload
    x.data[0] = 10.0
    assert float(amc.realize(e).values()) == 55.0                     # device copy unchanged
    x.host_changed()
    assert float(amc.realize(e).values()) == 155.0
    # a device-produced value is downloaded only when the host reads it
    y = amc.realize(amc.morph_add(x, x))
    assert y._data is None and list(y.values()) == [20.0, 2.0, 4.0, 6.0, 8.0, 10.0]


def _gemm_epilogue_trees(amc, dt):
    """(name, tree, launches) for map-over-GEMM trees; launches is the plan's
    launch count with the epilogue folded into the GEMM where it may be."""
    rng = np.random.default_rng(23)
    npdt = np.float32 if dt == "f32" else np.float64
    A = amc.morph_from_numpy(rng.standard_normal((37, 29)).astype(npdt))
    B = amc.morph_from_numpy(rng.standard_normal((29, 45)).astype(npdt))
    b1 = amc.morph_from_numpy(rng.standard_normal((45,)).astype(npdt))
    W2 = amc.morph_from_numpy(rng.standard_normal((45, 19)).astype(npdt))
    b2 = amc.morph_from_numpy(rng.standard_normal((1, 19)).astype(npdt))
    S = amc.morph_from_numpy(rng.standard_normal((40, 40)).astype(npdt))
    v = amc.morph_from_numpy(rng.standard_normal((29,)).astype(npdt))
    x = amc.morph_from_numpy(rng.standard_normal((300,)).astype(npdt))
    X = amc.morph_from_numpy(rng.standard_normal((37, 45, 3)).astype(npdt))
    h = amc.morph_matmul(A, B)
    hs = amc.morph_matmul(S, S)
    return [
        ("relu_bias", amc.morph_relu(amc.morph_add(amc.morph_matmul(A, B), b1)), 1),
        ("sigmoid_scale", amc.morph_sigmoid(amc.morph_map(lambda t: t * 0.5 - 0.25, amc.morph_matmul(A, B))), 1),
        ("int_consts", amc.morph_map(lambda t: t * 2 + 1, amc.morph_matmul(A, B)), 1),
        ("two_layers", amc.morph_relu(amc.morph_add(amc.morph_matmul(
            amc.morph_relu(amc.morph_add(amc.morph_matmul(A, B), b1)), W2), b2)), 2),
        ("matvec_tanh", amc.morph_tanh(amc.morph_map(lambda t: t - 1.5, amc.morph_matvec(A, v))), 1),
        ("dot_exp", amc.morph_exp(amc.morph_map(lambda t: t * 0.001, amc.morph_dot(x, x))), 1),
        # the GEMM result also read transposed: not folded
        ("plus_transpose", amc.morph_add(hs, amc.morph_transpose(hs, (1, 0))), 2),
        # two readers of the result (a map and a reduction): not folded
        ("two_readers", amc.morph_add(amc.morph_relu(h), amc.morph_reduce("sum", h, [1], True)), None),
        # a launch between the GEMM and the map: not folded
        ("step_between", amc.morph_add(amc.morph_matmul(A, B), amc.morph_reduce("sum", X, [2])), 3),
        # an empty contraction (K = 0): the epilogue sees zeros
        ("k_zero", amc.morph_relu(amc.morph_add(amc.morph_matmul(
            amc.morph_from_numpy(np.zeros((5, 0), npdt)), amc.morph_from_numpy(np.zeros((0, 7), npdt))),
            amc.morph_from_numpy(np.arange(7, dtype=npdt) - 3))), 1),
        # a comparison: the epilogue's output dtype (f64) differs from the GEMM's
        ("compare", amc.morph_gt(amc.morph_matmul(A, B), amc.morph_from_list([0.0], (1,), dt)), 1),
    ]


def _gemms_realized_first(amc, m, memo):
    """The same tree with every GEMM node realized on its own beforehand, so
    that no epilogue can be folded into it."""
    if not isinstance(m, amc.Expr):
        return m
    if id(m) not in memo:
        ops = [_gemms_realized_first(amc, o, memo) for o in m.operands]
        e = amc.Expr(m.op, ops, m.shape, m.dtype, m.meta, m.batch_axis)
        memo[id(m)] = amc.realize(e) if m.op in ("matmul", "matvec", "dot") else e
    return memo[id(m)]


_TRANSCENDENTAL_TREES = {"sigmoid_scale", "matvec_tanh", "dot_exp"}


@pytest.mark.parametrize("dt", ["f32", "f64"])
def test_gemm_epilogue_fusion_bitwise(amc, dt):
    """An element-wise map whose only input path to a GEMM result is through
    single-use map nodes runs in the GEMM's store (one launch fewer).  Values
    are bit-identical to the device's separate GEMM and map launches, and to
    the oracle (f64 transcendentals within 1e-12, CUDA's exp/tanh against
    libm's, as for every map); trees that must not be folded keep the
    separate launches."""
    for name, tree, launches in _gemm_epilogue_trees(amc, dt):
        p = amc.Plan(tree)
        if launches is not None:
            assert p.stats()["launches"] == launches, name
        p.execute()
        got = p.result().values()
        _same(got, amc.realize(_gemms_realized_first(amc, tree, {})).values())
        ref = oracle.realize(tree).values()
        if dt == "f64" and name in _TRANSCENDENTAL_TREES:
            np.testing.assert_allclose(np.asarray(got), np.asarray(ref), rtol=1e-12, atol=0, err_msg=name)
        else:
            _same(got, ref)
