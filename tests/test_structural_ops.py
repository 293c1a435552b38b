"""Structural constructors of the host mirror against the reference's
tests/test-structural-ops.scm (file:line per group): node kind, shapes,
dtypes, batch-axis tracking and the errors the reference raises; the pad
index functions through the oracle's values.  CPU only."""
import numpy as np
import pytest

import amcuda as am
import oracle


def ml(vals, shape, dt="f64", ba=-1):
    return am.morph_from_list(vals, tuple(shape), dt, ba)


def ones(n, shape, dt="f64", ba=-1):
    return ml([1.0] * n, shape, dt, ba)


# ------------------------------------------------------------------ reshape (test-structural-ops.scm:44-131)

def test_reshape():
    r = am.morph_reshape(ml([[1, 2, 3], [4, 5, 6]], (2, 3)), (6,))
    assert isinstance(r, am.Expr) and r.op == "reshape" and len(r.operands) == 1
    assert am.morph_reshape(ml([1, 2, 3, 4, 5, 6], (6,)), (2, 3)).shape == (2, 3)
    assert am.morph_reshape(ml([1, 2, 3, 4], (4,), "s32"), (2, 2)).dtype == "s32"
    assert am.morph_reshape(ml([1, 2, 3, 4, 5, 6], (6,)), (2, -1)).shape == (2, 3)
    assert am.morph_reshape(ml([[1, 2], [3, 4]], (2, 2)), (-1,)).shape == (4,)
    assert am.morph_reshape(ones(24, (2, 3, 4)), (2, -1, 4)).shape == (2, 3, 4)
    for bad in ((ml([1, 2, 3, 4], (4,)), (-1, -1)), (ml([1, 2, 3, 4, 5], (5,)), (2, -1)),
                (ml([1, 2, 3, 4], (4,)), (5,))):
        with pytest.raises(ValueError):
            am.morph_reshape(*bad)
    m = ml([1, 2, 3, 4, 5, 6], (6,))
    assert all(isinstance(am.morph_reshape(m, s), am.Expr) for s in ((2, 3), (3, 2), (1, 6)))
    assert am.morph_reshape(ml([[1, 2], [3, 4], [5, 6]], (3, 2), ba=0), (3, 2)).batch_axis == 0
    assert am.morph_reshape(ml([[1, 2], [3, 4]], (2, 2), ba=0), (4,)).batch_axis == -1
    assert am.morph_reshape(ones(12, (3, 4), ba=0), (3, 2, 2)).batch_axis == 0


# ------------------------------------------------------------------ transpose (:137-227)

def test_transpose():
    t = am.morph_transpose(ml([[1, 2], [3, 4]], (2, 2)))
    assert isinstance(t, am.Expr) and t.op == "transpose" and t.batch_axis == -1
    assert am.morph_transpose(ml([[1, 2], [3, 4]], (2, 2), "s32")).dtype == "s32"
    assert am.morph_transpose(ml([[1, 2, 3], [4, 5, 6]], (2, 3))).shape == (3, 2)
    assert am.morph_transpose(ones(24, (2, 3, 4))).shape == (4, 3, 2)
    assert am.morph_transpose(ml([1, 2, 3], (3,))).shape == (3,)
    assert am.morph_transpose(ml([[1, 2, 3], [4, 5, 6]], (2, 3)), (1, 0)).shape == (3, 2)
    assert am.morph_transpose(ones(24, (2, 3, 4)), (0, 2, 1)).shape == (2, 4, 3)
    assert am.morph_transpose(ones(24, (2, 3, 4)), (2, 0, 1)).shape == (4, 2, 3)
    assert am.morph_transpose(ml([[1, 2], [3, 4]], (2, 2)), (0, 1)).shape == (2, 2)
    for perm in ((0,), (0, 2), (0, 0)):
        with pytest.raises(ValueError):
            am.morph_transpose(ml([[1, 2], [3, 4]], (2, 2)), perm)
    assert am.morph_transpose(ones(12, (3, 2, 2), ba=0), (1, 0, 2)).batch_axis == 1
    assert am.morph_transpose(ones(12, (3, 2, 2), ba=0), (1, 2, 0)).batch_axis == 2


# ------------------------------------------------------------------ slice (:233-327)

def test_slice():
    s = am.morph_slice(ml([1, 2, 3, 4, 5], (5,)), (1,), (4,))
    assert isinstance(s, am.Expr) and s.op == "slice"
    assert am.morph_slice(ml([1, 2, 3, 4, 5], (5,), "s32"), (1,), (4,)).dtype == "s32"
    assert am.morph_slice(ml(list(range(6)), (6,)), (1,), (4,)).shape == (3,)
    assert am.morph_slice(ml(list(range(10)), (10,)), (0,), (10,), 2).shape == (5,)
    assert am.morph_slice(ml(list(range(5)), (5,)), (-2,), (-1,)).shape == (1,)
    assert am.morph_slice(ml([1, 2, 3, 4], (4,)), (0,), (4,)).shape == (4,)
    m33 = ml([[1, 2, 3], [4, 5, 6], [7, 8, 9]], (3, 3))
    assert am.morph_slice(m33, (0, 1), (2, 3)).shape == (2, 2)
    assert am.morph_slice(ml([[1, 2, 3], [4, 5, 6]], (2, 3)), (1, 0), (2, 3)).shape == (1, 3)
    assert am.morph_slice(ones(20, (4, 5)), (0, 0), (4, 5), (2, 2)).shape == (2, 3)
    for args in ((ml([[1, 2], [3, 4]], (2, 2)), (0,), (2, 2)), (ml([1, 2, 3], (3,)), (0,), (3,), -1),
                 (ml([1, 2, 3], (3,)), (0,), (5,)), (ml([1, 2, 3], (3,)), (2,), (1,))):
        with pytest.raises(ValueError):
            am.morph_slice(*args)
    assert am.morph_slice(ones(12, (3, 4), ba=0), (0, 1), (3, 3)).batch_axis == 0
    assert am.morph_slice(ones(12, (3, 4), ba=0), (1, 0), (2, 4)).batch_axis == -1
    assert am.morph_slice(ones(12, (4, 3), ba=0), (0, 0), (4, 3), (2, 1)).batch_axis == -1


# ------------------------------------------------------------------ squeeze, unsqueeze, pad (:332-455)

def test_squeeze_unsqueeze():
    assert am.morph_squeeze(ml([[[1, 2]]], (1, 1, 2))).shape == (2,)
    assert am.morph_squeeze(ones(6, (1, 2, 1, 3)), [0, 2]).shape == (2, 3)
    with pytest.raises(ValueError):
        am.morph_squeeze(ml([[1, 2]], (1, 2)), [1])
    assert am.morph_squeeze(ml([[1, 2], [3, 4]], (2, 2))).shape == (2, 2)
    assert am.morph_unsqueeze(ml([1, 2, 3], (3,)), 0).shape == (1, 3)
    assert am.morph_unsqueeze(ml([1, 2, 3], (3,)), 1).shape == (3, 1)
    assert am.morph_unsqueeze(ml([[1, 2], [3, 4]], (2, 2)), 1).shape == (2, 1, 2)
    assert am.morph_unsqueeze(ml([1, 2], (2,)), -1).shape == (2, 1)
    with pytest.raises(ValueError):
        am.morph_unsqueeze(ml([1, 2], (2,)), 3)


def test_pad_shapes_and_index_functions():
    x = ml([1, 2, 3], (3,))
    assert isinstance(am.morph_pad(x, [(1, 1)]), am.Expr)
    assert am.morph_pad(ml([[1, 2], [3, 4]], (2, 2)), [(1, 1), (2, 2)]).shape == (4, 6)
    with pytest.raises(ValueError):
        am.morph_pad(ml([[1, 2], [3, 4]], (2, 2)), [(1, 1)])
    assert am.morph_pad(x, [(1, 1)], "edge").shape == (5,)
    assert am.morph_pad(ml([[1, 2], [3, 4]], (2, 2)), [(1, 1), (1, 1)], "reflect").shape == (4, 4)
    # the index functions of :407-455, as the values they select from [1 2 3]
    vals = lambda m: list(np.asarray(oracle.values(m), dtype=np.float64))
    assert vals(am.morph_pad(x, [(2, 1)], "constant", 0.0)) == [0, 0, 1, 2, 3, 0]
    assert vals(am.morph_pad(x, [(2, 1)], "edge")) == [1, 1, 1, 2, 3, 3]       # indices 0 0 0 1 2 2
    assert vals(am.morph_pad(x, [(2, 2)], "reflect")) == [2, 1, 1, 2, 3, 3, 2]  # indices 1 0 0 1 2 2 1


# ------------------------------------------------------------------ im2col, col2im (:461-582)

def test_im2col_col2im():
    c = am.im2col_morph(ones(18, (2, 3, 3)), (2, 2))
    assert isinstance(c, am.Expr) and c.op == "im2col" and c.shape == (8, 4) and c.batch_axis == -1
    assert am.im2col_morph(ones(18, (2, 3, 3), "f32"), (2, 2)).dtype == "f32"
    assert am.im2col_morph(ones(18, (2, 3, 3)), (2, 2), 1, 0).shape == (8, 4)
    b = am.im2col_morph(ones(72, (4, 2, 3, 3), ba=0), (2, 2), 1, 0)
    assert b.shape == (4, 8, 4) and b.batch_axis == 0
    assert am.im2col_morph(ones(50, (2, 5, 5)), (3, 3), 2, 0).shape == (18, 4)
    assert am.im2col_morph(ones(18, (2, 3, 3)), (3, 3), 1, 1).shape == (18, 9)
    assert am.im2col_morph(ones(18, (2, 3, 3)), 2).shape == (8, 4)
    assert am.im2col_morph(ones(32, (2, 4, 4)), (2, 3), (1, 2), (0, 1)).shape == (12, 6)
    assert am.im2col_morph(ones(32, (2, 4, 4)), (3, 3), 1, 1).shape == (18, 16)
    col = ones(32, (8, 4))
    im = am.col2im_morph(col, (2, 3, 3), (2, 2))
    assert isinstance(im, am.Expr) and im.op == "col2im" and im.shape == (2, 3, 3) and im.batch_axis == -1
    assert am.col2im_morph(ones(32, (8, 4), "f32"), (2, 3, 3), (2, 2)).dtype == "f32"
    assert am.col2im_morph(ones(128, (4, 8, 4), ba=0), (4, 2, 3, 3), (2, 2)).batch_axis == 0
    with pytest.raises(ValueError):
        am.col2im_morph(col, (4, 2, 3, 3), (2, 2))


# ------------------------------------------------------------------ stack, concat, split (:588-705)

def test_stack_concat_split():
    a, b, c = ml([1, 2], (2,)), ml([3, 4], (2,)), ml([5, 6], (2,))
    assert isinstance(am.morph_stack([a, b]), am.Expr)
    assert am.morph_stack([a, b, c]).shape == (3, 2)
    assert am.morph_stack([a, b], 1).shape == (2, 2)
    assert am.morph_stack([ml([[1, 2], [3, 4]], (2, 2)), ml([[5, 6], [7, 8]], (2, 2))], 0).shape == (2, 2, 2)
    with pytest.raises(ValueError):
        am.morph_stack([a, ml([3, 4, 5], (3,))])
    assert am.morph_stack([ml([1, 2], (2,), "s32"), ml([3.0, 4.0], (2,))]).dtype == "f64"
    assert am.morph_stack([a, b], 0).batch_axis == 0
    assert am.morph_concat([a, ml([3, 4, 5], (3,))], 0).shape == (5,)
    assert am.morph_concat([ml([[1, 2], [3, 4]], (2, 2)), ml([[5, 6]], (1, 2))], 0).shape == (3, 2)
    assert am.morph_concat([ml([[1, 2], [3, 4]], (2, 2)), ml([[5], [6]], (2, 1))], 1).shape == (2, 3)
    with pytest.raises(ValueError):
        am.morph_concat([ml([[1, 2]], (1, 2)), ml([[3, 4, 5]], (1, 3))], 0)
    assert am.morph_concat([ml([1, 2], (2,), "s32"), ml([3.0, 4.0], (2,))]).dtype == "f64"
    m6 = ml([1, 2, 3, 4, 5, 6], (6,))
    assert [s.shape for s in am.morph_split(m6, 3)] == [(2,)] * 3
    assert [s.shape for s in am.morph_split(m6, [1, 2, 3])] == [(1,), (2,), (3,)]
    assert [s.shape for s in am.morph_split(ml([[1, 2], [3, 4], [5, 6], [7, 8]], (4, 2)), 2, 0)] == [(2, 2)] * 2
    with pytest.raises(ValueError):
        am.morph_split(ml([1, 2, 3, 4, 5], (5,)), 2)
    with pytest.raises(ValueError):
        am.morph_split(ml([1, 2, 3, 4], (4,)), [2, 3])


# ------------------------------------------------------------------ chained (:709-745)

def test_chained_shapes():
    m = ml([1, 2, 3, 4, 5, 6], (6,))
    assert am.morph_transpose(am.morph_reshape(m, (2, 3))).shape == (3, 2)
    assert am.morph_slice(am.morph_transpose(ml([[1, 2, 3], [4, 5, 6]], (2, 3))), (0, 0), (2, 1)).shape == (2, 1)
    assert am.morph_unsqueeze(am.morph_squeeze(ml([[[1, 2]]], (1, 1, 2))), 0).shape == (1, 2)
    st = am.morph_stack([ml([1, 2], (2,)), ml([3, 4], (2,)), ml([5, 6], (2,))])
    assert [s.shape for s in am.morph_split(st, 3)] == [(1, 2)] * 3
