"""Tree autograd: the host side of the reference's grad.scm.

A variable wraps a morphism with gradient state.  Each operation builds its
forward morphism and, when a parent requires a gradient, a backward closure
that adds lazy gradient morphisms to its parents.  backward() seeds the root
with ones and runs the closures root first.  Every gradient is a lazy tree of
the same constructors (`morph`), so realizing it runs on the device through
the planner; nothing here computes values.

Names, rules, accumulation order and errors follow grad.scm (file:line on
each function); errors raise ValueError where the reference calls `error`.
"""
from __future__ import annotations

import itertools
from typing import Callable, Iterable, Optional

import numpy as np

from .morph import (Morphism, dtype_floating, morph_add, morph_cos, morph_div, morph_exp, morph_from_list,
                    morph_from_numpy, morph_log, morph_map, morph_matmul, morph_mul, morph_negate, morph_pow,
                    morph_reduce, morph_relu, morph_reshape, morph_sigmoid, morph_sin, morph_sqrt, morph_sub,
                    morph_tanh, morph_transpose, morph_abs, normalize_axis, NP_DTYPES)

__all__ = [
    "Var", "make_var", "var_name", "var_value", "var_grad", "var_requires_grad", "zero_grad", "accumulate_grad",
    "var_add", "var_sub", "var_mul", "var_div", "var_pow", "var_sqrt", "var_exp", "var_log", "var_sin", "var_cos",
    "var_negate", "var_abs", "var_relu", "var_sigmoid", "var_tanh", "var_sum", "var_mean", "var_reshape",
    "var_transpose", "var_matmul", "var_parents", "var_grad_fn", "topo_sort", "backward",
]

_names = itertools.count()


class Var:
    """morph-variable (grad.scm:113-119)."""
    __slots__ = ("name", "value", "grad", "requires_grad", "grad_fn", "parents")

    def __init__(self, value: Morphism, requires_grad: bool):
        self.name = f"morph-var{next(_names)}"
        self.value = value
        self.grad: Optional[Morphism] = None
        self.requires_grad = bool(requires_grad)
        self.grad_fn: Optional[Callable[[Morphism], None]] = None
        self.parents: list = []


# ------------------------------------------------------------------ constructors, accessors, gradient state

def make_var(m: Morphism, requires_grad: bool = False) -> Var:
    """make-var (grad.scm:126-131)."""
    if not isinstance(m, Morphism):
        raise ValueError("make-var: value must be an array morphism")
    return Var(m, requires_grad)


def var_name(v: Var) -> str: return v.name                                # grad.scm:133-135
def var_value(v: Var) -> Morphism: return v.value                         # grad.scm:137-139
def var_grad(v: Var) -> Optional[Morphism]: return v.grad                 # grad.scm:141-143
def var_requires_grad(v: Var) -> bool: return v.requires_grad             # grad.scm:145-147
def var_parents(v: Var) -> list: return v.parents                         # grad.scm:699
def var_grad_fn(v: Var): return v.grad_fn                                 # grad.scm:700


def zero_grad(v: Var) -> None:
    """zero-grad! (grad.scm:154-156)."""
    v.grad = None


def accumulate_grad(v: Var, g: Morphism) -> None:
    """accumulate-grad! (grad.scm:158-164): the first contribution is taken as
    it is, later ones are added lazily (existing + g)."""
    v.grad = g if v.grad is None else morph_add(v.grad, g)


def _requires(vs: Iterable[Var]) -> bool:
    """grad-requires? (grad.scm:166-168)."""
    return any(v.requires_grad for v in vs)


# ------------------------------------------------------------------ helpers

def _grad_dtype(dtype: str) -> str:
    """effective-grad-dtype (grad.scm:175-180): integers accumulate in f64."""
    return dtype if dtype_floating(dtype) else "f64"


def _ones_like(m: Morphism) -> Morphism:
    """morph-ones-like (grad.scm:190-203): a concrete array of ones."""
    dt = _grad_dtype(m.dtype)
    return morph_from_numpy(np.ones(m.shape, dtype=NP_DTYPES[dt]), dt)


def _reduce_sum_to(g: Morphism, target_shape) -> Morphism:
    """reduce-sum-to (grad.scm:213-245): sum g over leading extra axes, then
    (keeping them) over axes the target broadcasts from size 1."""
    target = tuple(target_shape)
    extra = g.rank() - len(target)
    cur = morph_reduce("sum", g, list(range(extra))) if extra > 0 else g
    for k, t in enumerate(target):
        if t == 1 and cur.shape[k] > 1:
            cur = morph_reduce("sum", cur, [k], True)
    return cur


def _broadcast_grad(g: Morphism, x: Morphism, axes: list, keepdims: bool) -> Morphism:
    """broadcast-grad (grad.scm:253-275): g back to x's shape, by multiplying
    with ones of that shape (after reinserting the reduced axes)."""
    ones = _ones_like(x)
    if keepdims:
        return morph_mul(g, ones)
    expanded = [1 if i in axes else x.shape[i] for i in range(x.rank())]
    return morph_mul(morph_reshape(g, expanded), ones)


def _sign(m: Morphism) -> Morphism:
    """morph-sign (grad.scm:288-295): 1, -1 or 0 (also for NaN), dtype kept."""
    return morph_map(lambda v: (v > 0.0) - (v < 0.0), m)


def _link(out: Var, parents: list, fn: Callable[[Morphism], None]) -> Var:
    out.parents = [p for p in parents if p.requires_grad]
    out.grad_fn = fn
    return out


# ------------------------------------------------------------------ binary operations

def var_add(v1: Var, v2: Var) -> Var:
    """var+ (grad.scm:301-318)."""
    x1, x2 = v1.value, v2.value
    rg = _requires([v1, v2])
    out = make_var(morph_add(x1, x2), rg)
    if rg:
        def fn(g):
            if v1.requires_grad:
                accumulate_grad(v1, _reduce_sum_to(g, x1.shape))
            if v2.requires_grad:
                accumulate_grad(v2, _reduce_sum_to(g, x2.shape))
        _link(out, [v1, v2], fn)
    return out


def var_sub(v1: Var, v2: Var) -> Var:
    """var- (grad.scm:320-338)."""
    x1, x2 = v1.value, v2.value
    rg = _requires([v1, v2])
    out = make_var(morph_sub(x1, x2), rg)
    if rg:
        def fn(g):
            if v1.requires_grad:
                accumulate_grad(v1, _reduce_sum_to(g, x1.shape))
            if v2.requires_grad:
                accumulate_grad(v2, _reduce_sum_to(morph_negate(g), x2.shape))
        _link(out, [v1, v2], fn)
    return out


def var_mul(v1: Var, v2: Var) -> Var:
    """var* (grad.scm:340-361): product rule."""
    rg = _requires([v1, v2])
    out = make_var(morph_mul(v1.value, v2.value), rg)
    if rg:
        def fn(g):
            x1, x2 = v1.value, v2.value
            if v1.requires_grad:
                accumulate_grad(v1, _reduce_sum_to(morph_mul(g, x2), x1.shape))
            if v2.requires_grad:
                accumulate_grad(v2, _reduce_sum_to(morph_mul(g, x1), x2.shape))
        _link(out, [v1, v2], fn)
    return out


def var_div(v1: Var, v2: Var) -> Var:
    """var/ (grad.scm:363-387): quotient rule, d/dx2 = -g * x1 / (x2 * x2)."""
    rg = _requires([v1, v2])
    out = make_var(morph_div(v1.value, v2.value), rg)
    if rg:
        def fn(g):
            x1, x2 = v1.value, v2.value
            if v1.requires_grad:
                accumulate_grad(v1, _reduce_sum_to(morph_div(g, x2), x1.shape))
            if v2.requires_grad:
                d2 = morph_mul(morph_negate(g), morph_div(x1, morph_mul(x2, x2)))
                accumulate_grad(v2, _reduce_sum_to(d2, x2.shape))
        _link(out, [v1, v2], fn)
    return out


def var_pow(v1: Var, v2: Var) -> Var:
    """var-pow (grad.scm:389-418): d/dx1 = g * x2 * x1^(x2 - 1),
    d/dx2 = g * x1^x2 * log(x1)."""
    rg = _requires([v1, v2])
    out = make_var(morph_pow(v1.value, v2.value), rg)
    if rg:
        def fn(g):
            x1, x2 = v1.value, v2.value
            if v1.requires_grad:
                one = morph_from_list([1.0], (1,), "f64")
                d1 = morph_mul(g, morph_mul(x2, morph_pow(x1, morph_sub(x2, one))))
                accumulate_grad(v1, _reduce_sum_to(d1, x1.shape))
            if v2.requires_grad:
                d2 = morph_mul(g, morph_mul(morph_pow(x1, x2), morph_log(x1)))
                accumulate_grad(v2, _reduce_sum_to(d2, x2.shape))
        _link(out, [v1, v2], fn)
    return out


# ------------------------------------------------------------------ unary operations

def _unary(v: Var, fwd: Callable[[Morphism], Morphism], bwd: Callable[[Morphism, Morphism, Var], Morphism]) -> Var:
    out = make_var(fwd(v.value), v.requires_grad)
    if v.requires_grad:
        _link(out, [v], lambda g: accumulate_grad(v, bwd(g, v.value, out)))
    return out


def var_sqrt(v: Var) -> Var:
    """var-sqrt (grad.scm:424-440): d/dx = g / (2 sqrt(x)), sqrt(x) rebuilt lazily."""
    two = morph_from_list([2.0], (1,), "f64")
    return _unary(v, morph_sqrt, lambda g, x, out: morph_div(g, morph_mul(two, morph_sqrt(x))))


def var_exp(v: Var) -> Var:
    """var-exp (grad.scm:442-456): d/dx = g * exp(x)."""
    return _unary(v, morph_exp, lambda g, x, out: morph_mul(g, morph_exp(x)))


def var_log(v: Var) -> Var:
    """var-log (grad.scm:458-470): d/dx = g / x."""
    return _unary(v, morph_log, lambda g, x, out: morph_div(g, x))


def var_sin(v: Var) -> Var:
    """var-sin (grad.scm:472-484): d/dx = g * cos(x)."""
    return _unary(v, morph_sin, lambda g, x, out: morph_mul(g, morph_cos(x)))


def var_cos(v: Var) -> Var:
    """var-cos (grad.scm:486-498): d/dx = -(g * sin(x))."""
    return _unary(v, morph_cos, lambda g, x, out: morph_negate(morph_mul(g, morph_sin(x))))


def var_negate(v: Var) -> Var:
    """var-negate (grad.scm:504-515): d/dx = -g."""
    return _unary(v, morph_negate, lambda g, x, out: morph_negate(g))


def var_abs(v: Var) -> Var:
    """var-abs (grad.scm:517-528): d/dx = g * sign(x)."""
    return _unary(v, morph_abs, lambda g, x, out: morph_mul(g, _sign(x)))


def var_relu(v: Var) -> Var:
    """var-relu (grad.scm:532-544): d/dx = g * (x > 0 ? 1 : 0)."""
    return _unary(v, morph_relu, lambda g, x, out: morph_mul(g, morph_map(lambda t: t > 0.0, x)))


def var_sigmoid(v: Var) -> Var:
    """var-sigmoid (grad.scm:546-558): d/dx = g * s (1 - s), s the forward value."""
    return _unary(v, morph_sigmoid, lambda g, x, out: morph_mul(g, morph_map(lambda s: s * (1.0 - s), out.value)))


def var_tanh(v: Var) -> Var:
    """var-tanh (grad.scm:560-572): d/dx = g * (1 - t t), t the forward value."""
    return _unary(v, morph_tanh, lambda g, x, out: morph_mul(g, morph_map(lambda t: 1.0 - t * t, out.value)))


# ------------------------------------------------------------------ reductions

def _norm_axes(x: Morphism, axes) -> list:
    axes = list(axes)
    return list(range(x.rank())) if not axes else [normalize_axis(a, x.rank()) for a in axes]


def var_sum(v: Var, axes=(), keepdims: bool = False) -> Var:
    """var-sum (grad.scm:579-596): the gradient is broadcast back to x."""
    x = v.value
    norm = _norm_axes(x, axes)
    return _unary(v, lambda m: morph_reduce("sum", m, list(axes), keepdims),
                  lambda g, xx, out: _broadcast_grad(g, x, norm, keepdims))


def var_mean(v: Var, axes=(), keepdims: bool = False) -> Var:
    """var-mean (grad.scm:598-621): broadcast back, divided by the number of
    reduced elements (an f64 constant)."""
    x = v.value
    norm = _norm_axes(x, axes)
    n = 1
    for a in norm:
        n *= x.shape[a]
    n_m = morph_from_list([float(n)], (1,), "f64")
    return _unary(v, lambda m: morph_reduce("mean", m, list(axes), keepdims),
                  lambda g, xx, out: morph_div(_broadcast_grad(g, x, norm, keepdims), n_m))


# ------------------------------------------------------------------ structural and linear algebra

def var_reshape(v: Var, new_shape) -> Var:
    """var-reshape (grad.scm:629-641): the gradient is reshaped back."""
    shape = v.value.shape
    return _unary(v, lambda m: morph_reshape(m, new_shape), lambda g, x, out: morph_reshape(g, shape))


def var_transpose(v: Var, perm) -> Var:
    """var-transpose (grad.scm:643-657): the gradient is transposed by the
    inverse permutation."""
    perm = list(perm)
    inv = [0] * len(perm)
    for i, p in enumerate(perm):
        inv[p] = i
    return _unary(v, lambda m: morph_transpose(m, perm), lambda g, x, out: morph_transpose(g, inv))


def var_matmul(va: Var, vb: Var) -> Var:
    """var-matmul (grad.scm:668-693): dA = g B^T, dB = A^T g (transposes are views)."""
    rg = _requires([va, vb])
    out = make_var(morph_matmul(va.value, vb.value), rg)
    if rg:
        def fn(g):
            a, b = va.value, vb.value
            if va.requires_grad:
                accumulate_grad(va, morph_matmul(g, morph_transpose(b, [1, 0])))
            if vb.requires_grad:
                accumulate_grad(vb, morph_matmul(morph_transpose(a, [1, 0]), g))
        _link(out, [va, vb], fn)
    return out


# ------------------------------------------------------------------ backward pass

def topo_sort(root: Var) -> list:
    """topo-sort (grad.scm:713-724): depth-first over parents, each node put in
    front of everything visited below it, so the root comes first."""
    visited = set()

    def visit(v: Var, order: list) -> list:
        if v.name in visited:
            return order
        visited.add(v.name)
        for p in v.parents:
            order = visit(p, order)
        return [v] + order

    return visit(root, [])


def backward(var: Var, seed: Optional[Morphism] = None) -> None:
    """backward! (grad.scm:726-745): seed the root (ones by default), then run
    every node's backward closure in topo-sort order."""
    accumulate_grad(var, seed if seed is not None else _ones_like(var.value))
    for v in topo_sort(var):
        if v.grad_fn is not None and v.grad is not None:
            v.grad_fn(v.grad)
