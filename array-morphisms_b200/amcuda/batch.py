"""Batch combinators: the host side of the reference's batch-ops.scm.

Every combinator builds a lazy expression tree out of the structural and
arithmetic constructors in `morph`, exactly as the reference does (slice +
squeeze views per element, then a stack), so `realize` plans and runs the
whole tree on the device.  Names, argument meaning, batch-axis bookkeeping
and errors follow batch-ops.scm; errors raise ValueError where the
reference calls `error`.

Batch convention (batch-ops.scm:9-11): the batch axis is dimension 0 by
default, and a batched morphism carries batch_axis >= 0 (core.scm:847-856).
"""
from __future__ import annotations

from typing import Callable, Sequence

from . import _abi as A
from .morph import (DTYPES, Concrete, Expr, Morphism, morph_add, morph_concat, morph_div, morph_matmul, morph_mul,
                    morph_reduce, morph_slice, morph_squeeze, morph_stack, morph_sub, morph_unsqueeze)

__all__ = [
    "batched", "batch_size",
    "add_batch_dimension", "remove_batch_dimension", "extract_batch_element", "stack_into_batch", "concat_batch",
    "broadcast_to_batch",
    "batch_map", "batch_reduce", "batch_zip", "batch_fold", "batch_scan",
    "make_batch_aware_binop", "morph_add_batch", "morph_sub_batch", "morph_mul_batch", "morph_div_batch",
    "morph_batch_matmul",
]


def batched(m: Morphism) -> bool:
    """batched? (core.scm:847-849): the morphism carries a batch axis."""
    return m.batch_axis != -1


def batch_size(m: Morphism) -> int:
    """batch-size (core.scm:851-856): extent of the batch axis; error if not batched."""
    if not batched(m):
        raise ValueError("Morphism is not batched")
    return m.shape[m.batch_axis]


# --------------------------------------------------------------- batch dimension management

def add_batch_dimension(m: Morphism, axis: int = 0) -> Expr:
    """add-batch-dimension (batch-ops.scm:60-90): insert a size-1 axis and mark
    it as the batch axis."""
    if batched(m):
        raise ValueError("add-batch-dimension: morphism already has a batch dimension")
    rank = m.rank()
    norm = rank + 1 + axis if axis < 0 else axis
    if not 0 <= norm <= rank:
        raise ValueError(f"add-batch-dimension: axis out of range {axis} {rank}")
    out = morph_unsqueeze(m, axis)
    out.batch_axis = norm
    return out


def remove_batch_dimension(m: Morphism) -> Expr:
    """remove-batch-dimension (batch-ops.scm:92-110): squeeze a size-1 batch axis."""
    if not batched(m):
        raise ValueError("remove-batch-dimension: morphism has no batch dimension")
    if m.shape[m.batch_axis] != 1:
        raise ValueError(f"remove-batch-dimension: batch dimension must have size 1 ({m.shape[m.batch_axis]})")
    out = morph_squeeze(m, [m.batch_axis])
    out.batch_axis = -1
    return out


def extract_batch_element(m: Morphism, i: int, batch_axis: int = 0) -> Expr:
    """extract-batch-element (batch-ops.scm:112-141): element i along batch_axis
    as a non-batched zero-copy view (slice, then squeeze)."""
    rank = m.rank()
    n = m.shape[batch_axis]
    if i < 0 or i >= n:
        raise ValueError(f"extract-batch-element: index out of range {i} {n}")
    start = [i if ax == batch_axis else 0 for ax in range(rank)]
    end = [i + 1 if ax == batch_axis else m.shape[ax] for ax in range(rank)]
    out = morph_squeeze(morph_slice(m, start, end), [batch_axis])
    out.batch_axis = -1
    return out


def stack_into_batch(ms: Sequence[Morphism], axis: int = 0) -> Expr:
    """stack-into-batch (batch-ops.scm:143-160): stack non-batched morphisms
    into a batch (morph-stack marks `axis` as the batch axis)."""
    ms = list(ms)
    if not ms:
        raise ValueError("stack-into-batch: requires at least one morphism")
    if any(batched(m) for m in ms):
        raise ValueError("stack-into-batch: input morphisms must not be batched")
    return morph_stack(ms, axis)


def concat_batch(ms: Sequence[Morphism], axis: int = 0) -> Expr:
    """concat-batch (batch-ops.scm:162-180): concatenate batched morphisms along
    the batch axis."""
    ms = list(ms)
    if not ms:
        raise ValueError("concat-batch: requires at least one morphism")
    if not all(batched(m) for m in ms):
        raise ValueError("concat-batch: all morphisms must be batched")
    return morph_concat(ms, axis)


def broadcast_to_batch(m: Morphism, target_batch_size: int, batch_axis: int = 0) -> Morphism:
    """broadcast-to-batch (batch-ops.scm:184-211): a non-batched morphism gets a
    size-1 batch axis (element broadcasting expands it); a batched one of size
    1 or of the target size is returned as it is; any other size is an error."""
    if not batched(m):
        return add_batch_dimension(m, batch_axis)
    n = batch_size(m)
    if n in (1, target_batch_size):
        return m
    raise ValueError(f"broadcast-to-batch: batch size mismatch {n} {target_batch_size}")


# --------------------------------------------------------------- core combinators

def batch_map(fn: Callable[[Morphism], Morphism], m: Morphism, batch_axis: int = 0) -> Expr:
    """batch-map (batch-ops.scm:222-239): fn on every element along batch_axis,
    results stacked back at batch_axis."""
    n = m.shape[batch_axis]
    return morph_stack([fn(extract_batch_element(m, i, batch_axis)) for i in range(n)], batch_axis)


def batch_reduce(op: str, m: Morphism, keepdims: bool = False) -> Expr:
    """batch-reduce (batch-ops.scm:241-254): morph-reduce over the batch axis
    (axis 0 when the morphism is not batched)."""
    axis = m.batch_axis if batched(m) else 0
    return morph_reduce(op, m, [axis], keepdims)


def batch_zip(fn: Callable[[Morphism, Morphism], Morphism], m1: Morphism, m2: Morphism) -> Expr:
    """batch-zip (batch-ops.scm:256-276): fn on each pair of elements along
    axis 0, stacked."""
    n = m1.shape[0]
    if m2.shape[0] != n:
        raise ValueError(f"batch-zip: batch size mismatch {n} {m2.shape[0]}")
    return morph_stack([fn(extract_batch_element(m1, i, 0), extract_batch_element(m2, i, 0)) for i in range(n)], 0)


class _NotElementwise(Exception):
    pass


def _step_program(r: Morphism, acc: Morphism, e: Morphism, shape: tuple) -> list:
    """The program of one fold step r = fn(acc, e) over LOAD 0 = acc and
    LOAD 1 = e, spliced the way realize fuses map nodes (an inner map node's
    value is rounded to its dtype with CVT).  Raises _NotElementwise unless r
    is built from acc, e, size-1 constants and map nodes of the element shape
    only."""
    if r is acc:
        return [(A.OP["LOAD"], 0, 0.0)]
    if r is e:
        return [(A.OP["LOAD"], 1, 0.0)]
    if isinstance(r, Concrete) and r.size() == 1 and r.shape == (1,) * len(r.shape):
        v = r.values().reshape(-1)[0]
        if r.dtype in ("f32", "f64"):
            return [(A.OP["CONST"], 0, float(v))]
        if abs(int(v)) >= 1 << 53:
            raise _NotElementwise
        return [(A.OP["ICONST"], 0, float(int(v)))]
    if not (isinstance(r, Expr) and "prog" in r.meta and "scan" not in r.meta and r.shape == shape):
        raise _NotElementwise
    prog = []
    for (op, a, imm) in r.meta["prog"]:
        if op == A.OP["LOAD"]:
            o = r.operands[a]
            prog += _step_program(o, acc, e, shape)
            if isinstance(o, Expr) and o is not acc and o is not e:
                prog.append((A.OP["CVT"], DTYPES[o.dtype], 0.0))
        else:
            prog.append((op, a, imm))
    return prog


def _fold_steps(fn, init, m: Morphism):
    """Run batch-fold's loop (batch-ops.scm:278-300), returning every
    accumulator and, when every step is the same element-wise program of
    (acc, element) that keeps init's shape and dtype, that program (else
    None): realize then runs the whole fold as one SCAN node."""
    acc, accs, progs = init, [], []
    elem = tuple(m.shape[1:])
    ok = isinstance(init, Morphism) and tuple(init.shape) == elem
    for i in range(m.shape[0]):
        e = extract_batch_element(m, i, 0)
        r = fn(acc, e)
        if ok:
            try:
                if not isinstance(r, Expr) or r.shape != elem or r.dtype != init.dtype:
                    raise _NotElementwise
                p = _step_program(r, acc, e, elem)
                ok = not progs or p == progs[0]
                progs.append(p)
            except _NotElementwise:
                ok = False
        acc = r
        accs.append(acc)
    prog = progs[0] if ok and progs else None
    if prog is not None:
        sp = depth = 0
        for (op, _, _) in prog:
            sp += 1 if op in (A.OP["LOAD"], A.OP["CONST"], A.OP["ICONST"]) else (-1 if op >= A.OP["ADD"] else 0)
            depth = max(depth, sp)
        if len(prog) > A.PROG_MAX or depth > A.STACK_MAX:
            prog = None
    return accs, prog


def batch_fold(fn: Callable[[Morphism, Morphism], Morphism], init, m: Morphism):
    """batch-fold (batch-ops.scm:278-300): acc = fn(acc, element i) for i in
    order along axis 0, starting from init; returns the final accumulator.
    The returned tree is the reference's; when the step is element-wise it
    also records (init, m, step program) so realize runs one SCAN kernel."""
    accs, prog = _fold_steps(fn, init, m)
    if not accs:
        return init
    acc = accs[-1]
    if prog is not None:
        acc = Expr(acc.op, acc.operands, acc.shape, acc.dtype, dict(acc.meta, scan=(init, m, prog, False)),
                   acc.batch_axis)
    return acc


def batch_scan(fn: Callable[[Morphism, Morphism], Morphism], init, m: Morphism) -> Expr:
    """batch-scan (batch-ops.scm:302-322): every intermediate accumulator of
    batch-fold, stacked along axis 0 (one SCAN kernel when the step is
    element-wise, as for batch_fold)."""
    accs, prog = _fold_steps(fn, init, m)
    out = morph_stack(accs, 0)
    if prog is not None and out.dtype == init.dtype:
        out.meta["scan"] = (init, m, prog, True)
    return out


# --------------------------------------------------------------- batch-aware arithmetic

def make_batch_aware_binop(base_op: Callable[[Morphism, Morphism], Morphism]):
    """make-batch-aware-binop (batch-ops.scm:333-366): a non-batched operand is
    given a size-1 batch axis at the other operand's batch axis; two batched
    operands must have the same batch size."""
    def op(m1: Morphism, m2: Morphism):
        b1, b2 = batched(m1), batched(m2)
        if b1 and b2:
            if batch_size(m1) != batch_size(m2):
                raise ValueError(f"batch arithmetic: batch size mismatch {batch_size(m1)} {batch_size(m2)}")
            return base_op(m1, m2)
        if b1:
            return base_op(m1, broadcast_to_batch(m2, batch_size(m1), m1.batch_axis))
        if b2:
            return base_op(broadcast_to_batch(m1, batch_size(m2), m2.batch_axis), m2)
        return base_op(m1, m2)
    return op


morph_add_batch = make_batch_aware_binop(morph_add)   # morph+/batch
morph_sub_batch = make_batch_aware_binop(morph_sub)   # morph-/batch
morph_mul_batch = make_batch_aware_binop(morph_mul)   # morph*/batch
morph_div_batch = make_batch_aware_binop(morph_div)   # morph-div/batch


# --------------------------------------------------------------- batched matmul

def morph_batch_matmul(a: Morphism, b: Morphism) -> Expr:
    """morph-batch-matmul (batch-ops.scm:372-422): (M,K)x(K,P) is a plain
    matmul; (N,M,K)x(K,P) maps matmul over the batch (shared weight);
    (N,M,K)x(N,K,P) zips it (per-element weight)."""
    ra, rb = a.rank(), b.rank()
    if ra == 2 and rb == 2:
        return morph_matmul(a, b)
    if ra == 3 and rb == 2:
        if a.shape[2] != b.shape[0]:
            raise ValueError(f"morph-batch-matmul: inner dimensions must match {a.shape[2]} {b.shape[0]}")
        return batch_map(lambda x: morph_matmul(x, b), a, 0)
    if ra == 3 and rb == 3:
        if a.shape[0] != b.shape[0]:
            raise ValueError(f"morph-batch-matmul: batch size mismatch {a.shape[0]} {b.shape[0]}")
        if a.shape[2] != b.shape[1]:
            raise ValueError(f"morph-batch-matmul: inner dimensions must match {a.shape[2]} {b.shape[1]}")
        return batch_zip(morph_matmul, a, b)
    raise ValueError(f"morph-batch-matmul: unsupported shape combination {a.shape} {b.shape}")
