"""The column fold: ordered sums over a strided axis of outputs adjacent in
memory, with the element program evaluated in its closed form and the leaves
moved by TMA.  Every case is bit-exact against the oracle, and each one
checks that the column-fold kernel is what ran (its launch counter moves)."""
import ctypes as C

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def _launches():
    from amcuda import _abi as A
    n = C.c_int64(0)
    A.call("amc_colfold_launch_count", C.byref(n))
    return n.value


def _same(a, b):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape and a.dtype == b.dtype
    a, b = a.reshape(-1), b.reshape(-1)
    assert np.array_equal(a.view(np.uint8), b.view(np.uint8)), np.max(np.abs(a.astype(np.float64) - b))


def _rand(rng, shape, dtype):
    if dtype in ("f32", "f64"):
        return rng.uniform(-1.0, 1.0, shape).astype(np.float32 if dtype == "f32" else np.float64)
    return rng.integers(-3000, 3000, shape).astype(np.int32)


def _forms(amc, x, y):
    """Programs of every closed form: A, A op B, (A op B) op C, C op (A op B),
    with leaves and constants in each place."""
    return {
        "x": x,
        "x+y": amc.morph_add(x, y),
        "x-y": amc.morph_sub(x, y),
        "x*y": amc.morph_mul(x, y),
        "x*x+y": amc.morph_add(amc.morph_mul(x, x), y),
        "x*x-y": amc.morph_sub(amc.morph_mul(x, x), y),
        "y-x*x": amc.morph_sub(y, amc.morph_mul(x, x)),
        "x*(x+y)": amc.morph_mul(x, amc.morph_add(x, y)),
        "x-3": amc.morph_map(lambda v: v - 3, x),
        "3-x": amc.morph_map(lambda v: 3 - v, x),
        "2*x+y": amc.morph_add(amc.morph_map(lambda v: v * 2, x), y),
    }


@pytest.mark.parametrize("dtype", ["f64", "f32", "s32"])
@pytest.mark.parametrize("R,O", [(1, 8), (31, 16), (64, 1000), (65, 1024), (600, 1024), (1500, 2048)])
def test_colfold_forms_bit_exact(amc, dtype, R, O):
    """Sums over axis 0 of (R, O) trees: R = 1 and 31 leave a partial first
    step, 65 a partial chunk, 600 and 1500 wrap the 8-slot ring; O = 1000
    and 2048 leave a partial last CTA / two fold warps per CTA."""
    rng = np.random.default_rng(7 * R + O)
    x = amc.morph_from_numpy(_rand(rng, (R, O), dtype))
    y = amc.morph_from_numpy(_rand(rng, (R, O), dtype))
    for name, e in _forms(amc, x, y).items():
        for op in (("sum", "mean") if dtype != "s32" else ("sum",)):
            tree = amc.morph_reduce(op, e, (0,))
            before = _launches()
            dev = amc.realize(tree).values()
            assert _launches() == before + 1, f"{name} {op}: the column fold did not run"
            _same(dev, oracle.realize(amc.morph_reduce(op, e, (0,))).values())


@pytest.mark.parametrize("dtype", ["f64", "s32"])
def test_colfold_config1(amc, dtype):
    """Config 1 itself (x^2 + y over the step-2 slice of a transposed
    1024 x 1024 reshape) goes through the column fold."""
    from amcuda import workloads as W
    xm, ym = W.c1_inputs_morph(dtype)
    before = _launches()
    dev = amc.realize(W.c1_tree(xm, ym)).values()
    assert _launches() == before + 1
    _same(dev, oracle.realize(W.c1_tree(xm, ym)).values())


def test_colfold_declines_other_kinds(amc):
    """Shapes outside the column fold keep their own kernels and stay exact:
    a unary program, a pitch that is not a multiple of 16 bytes, a max."""
    rng = np.random.default_rng(3)
    x = amc.morph_from_numpy(rng.uniform(-1, 1, (100, 13)))
    z = amc.morph_from_numpy(rng.uniform(-1, 1, (100, 16)))
    for tree in (amc.morph_reduce("sum", amc.morph_abs(z), (0,)),
                 amc.morph_reduce("sum", amc.morph_mul(x, x), (0,)),
                 amc.morph_reduce("max", z, (0,))):
        before = _launches()
        dev = amc.realize(tree).values()
        assert _launches() == before
        _same(dev, oracle.realize(tree).values())
