"""Core helpers of the host mirror against the reference's tests/test-core.scm
(file:line per group): strides, axes, broadcasting, dtype rules, concrete
array construction and batch accessors.  CPU only."""
import numpy as np
import pytest

import amcuda as am
from amcuda import morph as M


def test_shape_utilities():                                         # test-core.scm:41-100
    assert M.shape_size((2, 3, 4)) == 24
    assert M.compute_strides((5,)) == (1,)
    assert M.compute_strides((3, 4)) == (4, 1)
    assert M.compute_strides((3, 4, 5)) == (20, 5, 1)
    assert M.compute_strides((2, 3, 4, 10)) == (120, 40, 10, 1)
    assert M.normalize_axis(1, 3) == 1 and M.normalize_axis(-1, 3) == 2 and M.normalize_axis(-2, 3) == 1


def test_broadcasting():                                            # test-core.scm:168-214
    assert M.broadcast_shapes((3, 4), (3, 4)) == (3, 4)
    assert M.broadcast_shapes((3, 1, 5), (4, 5)) == (3, 4, 5)
    assert M.broadcast_shapes((3, 4, 5), (1,)) == (3, 4, 5)
    assert M.broadcast_shapes((3, 1, 5), (1, 4, 1)) == (3, 4, 5)
    with pytest.raises(ValueError):
        M.broadcast_shapes((3, 4), (5, 6))


def test_type_system():                                             # test-core.scm:222-290
    assert M.dtype_floating("f64") and not M.dtype_floating("s32")
    assert M.promote_types("f32", "f64") == "f64" and M.promote_types("f32", "s32") == "f32"
    assert M.promote_types("f32", "f32") == "f32" and M.promote_types("s32", "s64") == "s64"
    assert M.infer_reduction_dtype("sum", "f32") == "f32"
    assert M.infer_reduction_dtype("mean", "s32") == "f64" and M.infer_reduction_dtype("mean", "f32") == "f32"
    assert M.infer_reduction_dtype("argmax", "f64") == "s32"


def test_construction_and_accessors():                             # test-core.scm:332-480
    m = am.morph_from_list([[1, 2, 3], [4, 5, 6]], (2, 3), "f32")
    assert isinstance(m, am.Concrete) and m.shape == (2, 3) and m.dtype == "f32"
    assert m.size() == 6 and m.rank() == 2 and m.batch_axis == -1 and not am.batched(m)
    assert am.morph_from_list([1, 2, 3, 4], (2, 2), "s32").dtype == "s32"
    with pytest.raises(ValueError):
        am.morph_from_list([1, 2, 3], (2, 2), "f32")
    b = am.morph_from_list([[1, 2], [3, 4], [5, 6]], (3, 2), "f64", 0)
    assert am.batched(b) and am.batch_size(b) == 3
    assert am.morph_from_list([1, 2, 3], (3,), "f32").values().tolist() == [1.0, 2.0, 3.0]
    assert am.morph_from_list([[[1, 2], [3, 4]], [[5, 6], [7, 8]]], (2, 2, 2), "f32").values().tolist() == \
        [[[1.0, 2.0], [3.0, 4.0]], [[5.0, 6.0], [7.0, 8.0]]]
    assert am.morph_from_numpy(np.zeros((2, 2), np.float32), batch_axis=0).batch_axis == 0
