"""Host-side constructors: shapes, dtypes and errors as the reference's."""
import pytest

import amcuda as am


def m(vals, shape, dt="f64"):
    return am.morph_from_list(vals, shape, dt)


def test_binary_promotion_and_broadcast():
    a = m([1, 2, 3], (3,), "s32")
    b = m([1.5], (1,), "f32")
    c = am.morph_add(a, b)
    assert c.shape == (3,) and c.dtype == "f32"
    assert am.morph_gt(a, a).dtype == "f64"
    with pytest.raises(ValueError):
        am.morph_add(m([1, 2], (2,)), m([1, 2, 3], (3,)))


def test_unary_dtype_rules():
    a = m([1, 4], (2,), "s32")
    assert am.morph_sqrt(a).dtype == "f64"
    assert am.morph_abs(a).dtype == "s32"
    assert am.morph_map(lambda x: x * x, a).dtype == "s32"


def test_reduce_shapes():
    a = m(list(range(24)), (2, 3, 4))
    assert am.morph_reduce("sum", a, (1,)).shape == (2, 4)
    assert am.morph_reduce("sum", a, (1,), True).shape == (2, 1, 4)
    assert am.morph_reduce("sum", a).shape == ()
    assert am.morph_reduce("mean", m([1, 2], (2,), "s32")).dtype == "f64"


def test_structural_shapes_and_errors():
    a = m(list(range(12)), (12,))
    assert am.morph_reshape(a, (3, -1)).shape == (3, 4)
    with pytest.raises(ValueError):
        am.morph_reshape(a, (5, -1))
    with pytest.raises(ValueError):
        am.morph_reshape(a, (-1, -1))
    b = am.morph_reshape(a, (3, 4))
    assert am.morph_transpose(b).shape == (4, 3)
    with pytest.raises(ValueError):
        am.morph_transpose(b, (0, 0))
    assert am.morph_slice(b, (0, 1), (3, 4), (2, 2)).shape == (2, 2)
    with pytest.raises(ValueError):
        am.morph_slice(b, (0, 0), (4, 4))
    with pytest.raises(ValueError):
        am.morph_slice(b, (0, 0), (3, 4), 0)
    assert am.morph_pad(b, [(1, 1), (0, 2)]).shape == (5, 6)
    x = m([0.0] * 48, (3, 4, 4))
    assert am.im2col_morph(x, (3, 3), 1, 1).shape == (27, 16)
    assert am.col2im_morph(am.im2col_morph(x, (2, 2), 2, 0), (3, 4, 4), (2, 2), 2, 0).shape == (3, 4, 4)
    assert am.morph_stack([a, a], 1).shape == (12, 2)
    assert am.morph_concat([b, b], 1).shape == (3, 8)
    assert [s.shape for s in am.morph_split(b, 2, 1)] == [(3, 2), (3, 2)]


def test_blas_constructors_reject_batched_operands():
    a3 = m([0.0] * 8, (2, 2, 2))
    a2 = m([0.0] * 4, (2, 2))
    with pytest.raises(ValueError):
        am.morph_matmul(a3, a2)
    assert am.morph_matmul(a2, m([0.0] * 6, (2, 3), "f32")).dtype == "f64"
    assert am.morph_dot(m([1.0, 2.0], (2,)), m([1.0, 2.0], (2,))).shape == ()


def test_attention_default_scale():
    q = m([0.0] * 12, (3, 4))
    att = am.attention_morphism(q, q, q)
    assert att.meta["scale"] == 0.5 and att.shape == (3, 4)


def test_attention_constructor():
    """test-attention.scm:151-196: output (n, dv) from V, dtype, scale in the
    metadata, and the shape errors."""
    q = m([0.0] * 12, (3, 4))
    assert am.attention_morphism(q, q, m([0.0] * 18, (3, 6))).shape == (3, 6)
    assert am.attention_morphism(q, q, q).dtype == "f64"
    assert am.attention_morphism(q, q, q, 0.25).meta["scale"] == 0.25
    with pytest.raises(ValueError):
        am.attention_morphism(q, m([0.0] * 15, (3, 5)), q)
    with pytest.raises(ValueError):
        am.attention_morphism(q, q, m([0.0] * 8, (2, 4)))
