"""Lazy array morphisms: the host data model of the reference, in Python.

Mirrors the public constructors of array-morphisms (core.scm, basic-ops.scm,
structural-ops.scm, blas-exec.scm): they only build a tree; nothing is
computed until realize().  Names follow the reference with Scheme
punctuation mapped to Python (morph+ -> morph_add, morph-reduce ->
morph_reduce, im2col-morph -> im2col_morph, ...).

Element-wise combiners are carried as postfix programs (include/amc.h
AMC_OP_*).  morph_map traces its Python function on a symbolic operand, the
counterpart of capturing the Scheme lambda's source: the function may use
+ - * / ** with numbers, comparisons, and the functions in amcuda.fn.
"""
from __future__ import annotations

import itertools
import math
from typing import Iterable, Sequence

import numpy as np

from . import _abi as A

DTYPES = {"f32": A.F32, "f64": A.F64, "s32": A.S32, "s64": A.S64, "u32": A.U32, "u64": A.U64}
NP_DTYPES = {"f32": np.float32, "f64": np.float64, "s32": np.int32, "s64": np.int64, "u32": np.uint32,
             "u64": np.uint64}
FROM_NP = {np.dtype(v): k for k, v in NP_DTYPES.items()}
FLOAT = ("f32", "f64")

_ids = itertools.count()


def dtype_floating(d: str) -> bool:
    return d in FLOAT


def promote_types(d1: str, d2: str) -> str:
    """promote-types (core.scm:585-605): f64 > f32 > s64 > s32 > u64 > u32."""
    if d1 == d2:
        return d1
    for d in ("f64", "f32", "s64", "s32", "u64"):
        if d1 == d or d2 == d:
            return d
    return "u32"


def infer_reduction_dtype(op: str, dtype: str) -> str:
    """infer-reduction-dtype (core.scm:607-621): mean promotes integers to
    f64, argmax/argmin give s32 indices, the rest keep the dtype."""
    if op == "mean":
        return dtype if dtype_floating(dtype) else "f64"
    if op in ("argmax", "argmin"):
        return "s32"
    return dtype


def compute_strides(shape: Sequence[int]) -> tuple:
    """compute-strides (core.scm:441-456): row-major element strides."""
    st, s = [], 1
    for d in reversed(shape):
        st.append(s)
        s *= d
    return tuple(reversed(st))


def shape_size(shape: Sequence[int]) -> int:
    n = 1
    for d in shape:
        n *= d
    return n


def broadcast_shapes(s1: Sequence[int], s2: Sequence[int]) -> tuple:
    """broadcast-shapes (core.scm:519-545)."""
    r = max(len(s1), len(s2))
    a = (1,) * (r - len(s1)) + tuple(s1)
    b = (1,) * (r - len(s2)) + tuple(s2)
    out = []
    for x, y in zip(a, b):
        if x != y and x != 1 and y != 1:
            raise ValueError(f"Shapes not compatible for broadcasting {tuple(s1)} {tuple(s2)}")
        out.append(max(x, y))
    return tuple(out)


def normalize_axis(ax: int, rank: int) -> int:
    a = ax + rank if ax < 0 else ax
    if not 0 <= a < max(rank, 1):
        raise ValueError(f"axis {ax} out of range for rank {rank}")
    return a


# ---------------------------------------------------------------------------- ADT
class Morphism:
    """array-morphism (core.scm:238-269)."""
    shape: tuple
    dtype: str
    batch_axis: int

    def rank(self) -> int:
        return len(self.shape)

    def size(self) -> int:
        return shape_size(self.shape)

    # operator sugar (not in the reference; convenient in Python)
    def __add__(self, o): return morph_add(self, _lift(o, self))
    def __sub__(self, o): return morph_sub(self, _lift(o, self))
    def __mul__(self, o): return morph_mul(self, _lift(o, self))
    def __truediv__(self, o): return morph_div(self, _lift(o, self))


class Concrete(Morphism):
    """concrete-array: a typed vector with shape, strides and offset.

    `data` is the host typed vector; a value produced on the device may keep
    only its device buffer until the host reads `data` (then it is
    downloaded once)."""

    def __init__(self, data, shape, strides=None, offset=0, dtype="f64", batch_axis=-1, dev=None):
        self.shape = tuple(int(s) for s in shape)
        self.dtype = dtype
        self.strides = tuple(int(s) for s in (strides if strides is not None else compute_strides(self.shape)))
        self.offset = int(offset)
        self.batch_axis = batch_axis
        self._data = data
        self._dev = dev          # DeviceBuffer or None
        self.alloc_id = -1

    @property
    def data(self) -> np.ndarray:
        if self._data is None:
            self._data = self._dev.download()
        return self._data

    def host_changed(self) -> None:
        """Declare that the host vector was written in place (as the reference
        does with typed-vector-set! or the optimizer's in-place parameter
        updates).  The device copy, uploaded once by the first realize that
        read this array, is dropped, so the next realize uploads the new
        values.  Views created before the call keep the old device copy."""
        if self._data is None:
            raise ValueError("host_changed: the array has no host vector yet (read .data first)")
        self._dev = None

    def values(self) -> np.ndarray:
        """Logical values as a numpy array of this shape (a copy)."""
        flat = self.data
        if not self.shape:
            return np.array(flat[self.offset], dtype=flat.dtype)
        item = flat.itemsize
        v = np.lib.stride_tricks.as_strided(flat[self.offset:] if self.offset else flat, shape=self.shape,
                                            strides=tuple(s * item for s in self.strides))
        return np.array(v)

    def __repr__(self):
        return f"Concrete(shape={self.shape}, dtype={self.dtype})"


class Expr(Morphism):
    """morphism-expr / reduction-morphism: an unrealized node."""

    def __init__(self, op: str, operands: list, shape, dtype: str, meta: dict | None = None, batch_axis=-1):
        self.op = op
        self.operands = operands
        self.shape = tuple(int(s) for s in shape)
        self.dtype = dtype
        self.meta = meta or {}
        self.batch_axis = batch_axis
        self.morph_id = next(_ids)

    def __repr__(self):
        return f"Expr({self.op}, shape={self.shape}, dtype={self.dtype})"


def _lift(x, like: Morphism) -> Morphism:
    if isinstance(x, Morphism):
        return x
    dt = like.dtype if isinstance(x, (int, np.integer)) or dtype_floating(like.dtype) else "f64"
    return morph_from_list([x], (1,), dt)


# ---------------------------------------------------------------------------- construction
def morph_from_numpy(arr, dtype: str | None = None, batch_axis: int = -1) -> Concrete:
    a = np.asarray(arr)
    if dtype is None:
        dtype = FROM_NP.get(a.dtype)
        if dtype is None:
            dtype = "f64" if a.dtype.kind == "f" else "s64"
    if dtype not in DTYPES:
        raise ValueError(f"Unsupported dtype {dtype}")
    flat = np.ascontiguousarray(a, dtype=NP_DTYPES[dtype]).reshape(-1)
    return Concrete(flat, a.shape, dtype=dtype, batch_axis=batch_axis)


def morph_from_list(values, shape, dtype: str = "f64", batch_axis: int = -1) -> Concrete:
    """morph-from-list: nested or flat values with an explicit shape."""
    flat = np.array(values, dtype=np.float64 if dtype_floating(dtype) else np.int64).reshape(-1)
    shape = tuple(shape)
    if flat.size != shape_size(shape):
        raise ValueError(f"morph-from-list: {flat.size} values for shape {shape}")
    if not dtype_floating(dtype):
        flat = np.trunc(flat).astype(np.int64)
        if dtype.startswith("u"):
            flat = np.abs(flat)
    return Concrete(flat.astype(NP_DTYPES[dtype]), shape, dtype=dtype, batch_axis=batch_axis)


# ---------------------------------------------------------------------------- combiner programs
L0 = (A.OP["LOAD"], 0, 0.0)
L1 = (A.OP["LOAD"], 1, 0.0)


def _binary(opname: str, m1: Morphism, m2: Morphism, dtype: str | None = None) -> Expr:
    """create-binary-morphism (basic-ops.scm:40-82)."""
    shape = broadcast_shapes(m1.shape, m2.shape)
    dt = dtype or promote_types(m1.dtype, m2.dtype)
    ba = m1.batch_axis if m1.batch_axis >= 0 else m2.batch_axis
    return Expr(opname.lower(), [m1, m2], shape, dt, {"prog": [L0, L1, (A.OP[opname], 0, 0.0)]}, ba)


def morph_add(m1, m2): return _binary("ADD", m1, m2)
def morph_sub(m1, m2): return _binary("SUB", m1, m2)
def morph_mul(m1, m2): return _binary("MUL", m1, m2)
def morph_div(m1, m2): return _binary("DIV", m1, m2)
def morph_pow(m1, m2): return _binary("POW", m1, m2)


# comparisons -> f64 0.0/1.0 (basic-ops.scm:381-435)
def morph_gt(m1, m2): return _binary("GT", m1, m2, "f64")
def morph_lt(m1, m2): return _binary("LT", m1, m2, "f64")
def morph_eq(m1, m2): return _binary("EQ", m1, m2, "f64")
def morph_ge(m1, m2): return _binary("GE", m1, m2, "f64")
def morph_le(m1, m2): return _binary("LE", m1, m2, "f64")


_TRANSCENDENTAL = ("sqrt", "exp", "log", "sin", "cos", "tan", "relu", "sigmoid", "tanh")


def _unary(name: str, m: Morphism) -> Expr:
    """create-unary-morphism (basic-ops.scm:207-256); infer-unary-dtype (:286-302)."""
    dt = m.dtype
    if name in _TRANSCENDENTAL and not dtype_floating(dt):
        dt = "f64"
    opname = {"ceiling": "CEIL"}.get(name, name.upper())
    return Expr(name, [m], m.shape, dt, {"prog": [L0, (A.OP[opname], 0, 0.0)]}, m.batch_axis)


def morph_sqrt(m): return _unary("sqrt", m)
def morph_exp(m): return _unary("exp", m)
def morph_log(m): return _unary("log", m)
def morph_sin(m): return _unary("sin", m)
def morph_cos(m): return _unary("cos", m)
def morph_tan(m): return _unary("tan", m)
def morph_negate(m): return Expr("negate", [m], m.shape, m.dtype, {"prog": [L0, (A.OP["NEG"], 0, 0.0)]}, m.batch_axis)
def morph_abs(m): return _unary("abs", m)
def morph_floor(m): return _unary("floor", m)
def morph_ceiling(m): return _unary("ceiling", m)
def morph_relu(m): return _unary("relu", m)
def morph_sigmoid(m): return _unary("sigmoid", m)
def morph_tanh(m): return _unary("tanh", m)


class Sym:
    """Symbolic operand for tracing morph_map functions into programs."""

    def __init__(self, prog):
        self.prog = prog

    @staticmethod
    def _c(x) -> "Sym":
        if isinstance(x, Sym):
            return x
        if isinstance(x, bool):
            x = int(x)
        if isinstance(x, (int, np.integer)):
            return Sym([(A.OP["ICONST"], 0, float(x))])
        if isinstance(x, (float, np.floating)):
            return Sym([(A.OP["CONST"], 0, float(x))])
        raise TypeError(f"morph_map: cannot trace constant {x!r}")

    def _b(self, other, op, rev=False):
        o = Sym._c(other)
        a, b = (o, self) if rev else (self, o)
        return Sym(a.prog + b.prog + [(A.OP[op], 0, 0.0)])

    def __add__(self, o): return self._b(o, "ADD")
    def __radd__(self, o): return self._b(o, "ADD", True)
    def __sub__(self, o): return self._b(o, "SUB")
    def __rsub__(self, o): return self._b(o, "SUB", True)
    def __mul__(self, o): return self._b(o, "MUL")
    def __rmul__(self, o): return self._b(o, "MUL", True)
    def __truediv__(self, o): return self._b(o, "DIV")
    def __rtruediv__(self, o): return self._b(o, "DIV", True)
    def __pow__(self, o): return self._b(o, "POW")
    def __rpow__(self, o): return self._b(o, "POW", True)
    def __gt__(self, o): return self._b(o, "GT")
    def __lt__(self, o): return self._b(o, "LT")
    def __ge__(self, o): return self._b(o, "GE")
    def __le__(self, o): return self._b(o, "LE")
    def __neg__(self): return Sym(self.prog + [(A.OP["NEG"], 0, 0.0)])
    def __abs__(self): return Sym(self.prog + [(A.OP["ABS"], 0, 0.0)])


def morph_map(fn, m: Morphism) -> Expr:
    """morph-map (basic-ops.scm:475-507): element-wise function, dtype kept."""
    r = fn(Sym([L0]))
    prog = Sym._c(r).prog
    if len(prog) > A.PROG_MAX:
        raise ValueError("morph_map: function too long for one fused program")
    return Expr("map", [m], m.shape, m.dtype, {"prog": list(prog)}, m.batch_axis)


# ---------------------------------------------------------------------------- reductions
def morph_reduce(op: str, m: Morphism, axes: Iterable[int] = (), keepdims: bool = False) -> Expr:
    """morph-reduce (basic-ops.scm:522-608)."""
    if op not in A.RED:
        raise ValueError(f"Unknown reduction operation {op}")
    rank = m.rank()
    axes = list(axes)
    norm = sorted({normalize_axis(a, rank) for a in axes}) if axes else list(range(rank))
    if keepdims:
        shape = tuple(1 if i in norm else m.shape[i] for i in range(rank))
    else:
        shape = tuple(m.shape[i] for i in range(rank) if i not in norm)
    ba = m.batch_axis
    if ba >= 0:
        if ba in norm:
            ba = ba if keepdims else -1
        elif not keepdims:
            ba -= sum(1 for a in norm if a < ba)
    return Expr("reduce", [m], shape, infer_reduction_dtype(op, m.dtype), {"op": op, "axes": norm, "keepdims": keepdims}, ba)


# ---------------------------------------------------------------------------- structural
def morph_reshape(m: Morphism, new_shape) -> Expr:
    """morph-reshape (structural-ops.scm:49-137): at most one -1."""
    tgt = list(new_shape)
    size = m.size()
    if tgt.count(-1) > 1:
        raise ValueError(f"At most one -1 allowed in reshape {tgt}")
    if -1 in tgt:
        known = shape_size([d for d in tgt if d > 0])
        inf = size // known if known else 0
        if known * inf != size:
            raise ValueError("Cannot infer reshape dimension - sizes incompatible")
        tgt = [inf if d == -1 else d for d in tgt]
    if shape_size(tgt) != size:
        raise ValueError(f"Reshape size mismatch {size} {shape_size(tgt)}")
    ba = m.batch_axis
    if ba >= 0:
        if not (ba < len(tgt) and m.shape[ba] == tgt[ba]):
            bs = m.shape[ba]
            ba = next((i for i, d in enumerate(tgt) if d == bs), -1)
    return Expr("reshape", [m], tgt, m.dtype, {"original-shape": m.shape}, ba)


def morph_transpose(m: Morphism, perm=None) -> Expr:
    """morph-transpose (structural-ops.scm:167-226); default reverses axes."""
    rank = m.rank()
    perm = list(perm) if perm is not None else list(reversed(range(rank)))
    if sorted(perm) != list(range(rank)):
        raise ValueError(f"Invalid permutation {perm}")
    shape = [m.shape[p] for p in perm]
    ba = perm.index(m.batch_axis) if m.batch_axis >= 0 else -1
    return Expr("transpose", [m], shape, m.dtype, {"permutation": perm}, ba)


def morph_slice(m: Morphism, start, end, step=None) -> Expr:
    """morph-slice (structural-ops.scm:245-335)."""
    rank = m.rank()
    start, end = list(start), list(end)
    if step is None:
        step = [1] * rank
    elif isinstance(step, (int, np.integer)):
        step = [int(step)] * rank
    else:
        step = list(step)
    if not (len(start) == len(end) == len(step) == rank):
        raise ValueError("morph-slice: start/end/step length must equal rank")
    ns = [s + d if s < 0 else s for s, d in zip(start, m.shape)]
    ne = [e + d if e < 0 else e for e, d in zip(end, m.shape)]
    for s, e, d, st in zip(ns, ne, m.shape, step):
        if st <= 0:
            raise ValueError(f"Step must be positive {st}")
        if not 0 <= s < d:
            raise ValueError(f"Start index out of range {s} {d}")
        if not (s < e <= d):
            raise ValueError(f"End index out of range or not > start {e} {d} {s}")
    shape = [(e - s + st - 1) // st for s, e, st in zip(ns, ne, step)]
    ba = m.batch_axis
    if ba >= 0 and not (ns[ba] == 0 and ne[ba] == m.shape[ba] and step[ba] == 1):
        ba = -1
    return Expr("slice", [m], shape, m.dtype, {"start": ns, "end": ne, "step": step}, ba)


def morph_squeeze(m: Morphism, axes=None) -> Expr:
    """morph-squeeze (structural-ops.scm:350-385)."""
    rank = m.rank()
    rm = [normalize_axis(a, rank) for a in axes] if axes is not None else [i for i in range(rank) if m.shape[i] == 1]
    for a in rm:
        if m.shape[a] != 1:
            raise ValueError(f"Cannot squeeze non-singular dimension {a}")
    return morph_reshape(m, [m.shape[i] for i in range(rank) if i not in rm])


def morph_unsqueeze(m: Morphism, axis: int) -> Expr:
    """morph-unsqueeze (structural-ops.scm:387-409)."""
    rank = m.rank()
    a = rank + 1 + axis if axis < 0 else axis
    if not 0 <= a <= rank:
        raise ValueError("Unsqueeze axis out of range")
    s = list(m.shape)
    return morph_reshape(m, s[:a] + [1] + s[a:])


def morph_pad(m: Morphism, padding, mode: str = "constant", value: float = 0.0) -> Expr:
    """morph-pad (structural-ops.scm:411-447): list of (before, after) per axis."""
    padding = [tuple(p) for p in padding]
    if len(padding) != m.rank():
        raise ValueError("Padding length must match rank")
    if mode not in A.PAD:
        raise ValueError(f"Unknown padding mode {mode}")
    shape = [d + b + a for d, (b, a) in zip(m.shape, padding)]
    return Expr("pad", [m], shape, m.dtype, {"padding": padding, "mode": mode, "value": float(value)}, m.batch_axis)


def _pair(x):
    if isinstance(x, (list, tuple)):
        return (int(x[0]), int(x[1] if len(x) > 1 else x[0]))
    return (int(x), int(x))


def im2col_morph(m: Morphism, kernel_size, stride=1, padding=0) -> Expr:
    """im2col-morph (structural-ops.scm:513-579)."""
    batched = m.rank() == 4
    if m.rank() not in (3, 4):
        raise ValueError("im2col: input must be (C,H,W) or (N,C,H,W)")
    N, C, H, W = (m.shape if batched else (1,) + m.shape)
    KH, KW = _pair(kernel_size)
    SH, SW = _pair(stride)
    PH, PW = _pair(padding)
    OH = 1 + (H + 2 * PH - KH) // SH
    OW = 1 + (W + 2 * PW - KW) // SW
    shape = (N, C * KH * KW, OH * OW) if batched else (C * KH * KW, OH * OW)
    meta = {"kernel-size": (KH, KW), "stride": (SH, SW), "padding": (PH, PW), "spatial-output": (OH, OW)}
    return Expr("im2col", [m], shape, m.dtype, meta, 0 if batched else -1)


def col2im_morph(col: Morphism, output_shape, kernel_size, stride=1, padding=0) -> Expr:
    """col2im-morph (structural-ops.scm:629-686)."""
    output_shape = tuple(output_shape)
    if not ((col.rank() == 2 and len(output_shape) == 3) or (col.rank() == 3 and len(output_shape) == 4)):
        raise ValueError("Batch mismatch between col and output shape")
    KH, KW = _pair(kernel_size)
    SH, SW = _pair(stride)
    PH, PW = _pair(padding)
    meta = {"kernel-size": (KH, KW), "stride": (SH, SW), "padding": (PH, PW)}
    return Expr("col2im", [col], output_shape, col.dtype, meta, 0 if len(output_shape) == 4 else -1)


def morph_stack(ms: Sequence[Morphism], axis: int = 0) -> Expr:
    """morph-stack (structural-ops.scm:729-790)."""
    ms = list(ms)
    if not ms:
        raise ValueError("morph-stack requires at least one morphism")
    s0 = ms[0].shape
    if any(m.shape != s0 for m in ms):
        raise ValueError("All morphisms must have same shape for stack")
    a = len(s0) + 1 + axis if axis < 0 else axis
    if not 0 <= a <= len(s0):
        raise ValueError("stack axis out of range")
    dt = ms[0].dtype
    for m in ms[1:]:
        dt = promote_types(dt, m.dtype)
    shape = list(s0[:a]) + [len(ms)] + list(s0[a:])
    return Expr("stack", ms, shape, dt, {"axis": a}, a)


def morph_unstack(m: Morphism, axis: int = 0) -> list:
    a = normalize_axis(axis, m.rank())
    out = []
    for i in range(m.shape[a]):
        st = [0] * m.rank()
        en = list(m.shape)
        st[a], en[a] = i, i + 1
        out.append(morph_squeeze(morph_slice(m, st, en), [a]))
    return out


def morph_concat(ms: Sequence[Morphism], axis: int = 0) -> Expr:
    """morph-concat (structural-ops.scm:860-928)."""
    ms = list(ms)
    if not ms:
        raise ValueError("morph-concat requires at least one morphism")
    rank = ms[0].rank()
    a = normalize_axis(axis, rank)
    for m in ms:
        if m.rank() != rank or any(m.shape[i] != ms[0].shape[i] for i in range(rank) if i != a):
            raise ValueError("concat: shapes must match except along the axis")
    dt = ms[0].dtype
    for m in ms[1:]:
        dt = promote_types(dt, m.dtype)
    shape = list(ms[0].shape)
    shape[a] = sum(m.shape[a] for m in ms)
    return Expr("concat", ms, shape, dt, {"axis": a}, ms[0].batch_axis)


def morph_split(m: Morphism, sections, axis: int = 0) -> list:
    """morph-split (structural-ops.scm:792-858): equal parts or explicit sizes."""
    a = normalize_axis(axis, m.rank())
    d = m.shape[a]
    if isinstance(sections, int):
        if d % sections:
            raise ValueError("split: axis not divisible")
        sizes = [d // sections] * sections
    else:
        sizes = list(sections)
        if sum(sizes) != d:
            raise ValueError("split: sizes must sum to the axis length")
    out, pos = [], 0
    for s in sizes:
        st = [0] * m.rank()
        en = list(m.shape)
        st[a], en[a] = pos, pos + s
        out.append(morph_slice(m, st, en))
        pos += s
    return out


# ---------------------------------------------------------------------------- BLAS-shaped
def morph_matmul(a: Morphism, b: Morphism) -> Expr:
    """morph-matmul (blas-exec.scm:227-258): 2-D only, dtype promoted."""
    if a.rank() != 2:
        raise ValueError(f"morph-matmul: A must be 2-D {a.shape}")
    if b.rank() != 2:
        raise ValueError(f"morph-matmul: B must be 2-D {b.shape}")
    if a.shape[1] != b.shape[0]:
        raise ValueError("morph-matmul: inner dimensions must match")
    return Expr("matmul", [a, b], (a.shape[0], b.shape[1]), promote_types(a.dtype, b.dtype))


def morph_matvec(a: Morphism, v: Morphism) -> Expr:
    """morph-matvec (blas-exec.scm:260-285)."""
    if a.rank() != 2 or v.rank() != 1 or a.shape[1] != v.shape[0]:
        raise ValueError("morph-matvec: shapes must be (M,N) x (N)")
    return Expr("matvec", [a, v], (a.shape[0],), promote_types(a.dtype, v.dtype))


def morph_dot(v1: Morphism, v2: Morphism) -> Expr:
    """morph-dot (blas-exec.scm:287-310)."""
    if v1.rank() != 1 or v2.rank() != 1 or v1.shape[0] != v2.shape[0]:
        raise ValueError("morph-dot: vectors must be 1-D of the same length")
    return Expr("dot", [v1, v2], (), promote_types(v1.dtype, v2.dtype))


def attention_morphism(Q: Morphism, K: Morphism, V: Morphism, scale: float | None = None) -> Expr:
    """attention-morphism (blas-exec.scm:334-398): rank 2..4, default scale 1/sqrt(dk)."""
    r = Q.rank()
    if r < 2 or K.rank() != r or V.rank() != r:
        raise ValueError("attention-morphism: Q, K, V must share rank >= 2")
    n, dk = Q.shape[-2], Q.shape[-1]
    if K.shape[-2] != n or K.shape[-1] != dk or V.shape[-2] != n:
        raise ValueError("attention-morphism: shape mismatch")
    if scale is None:
        scale = 1.0 / math.sqrt(dk)
    shape = tuple(Q.shape[:-1]) + (V.shape[-1],)
    meta = {"scale": float(scale), "n": n, "dk": dk, "dv": V.shape[-1], "n-leading": r - 2}
    return Expr("attention", [Q, K, V], shape, Q.dtype, meta, Q.batch_axis)
