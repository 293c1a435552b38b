"""SSA compilation of a variable graph: the host side of the reference's ssa.scm.

morphism_to_ssa flattens the value tree of a variable into an SSA program of
bindings in topological order (concrete arrays become constants, shared
nodes one binding); ssa_vjp appends the reverse-mode bindings with the
reference's rules and makes the outputs (loss, gradient of each parameter).
Running a program rebuilds every binding as a lazy morphism of the same
constructors (`morph`) over its inputs, so realize plans and runs the joint
forward and backward trees on the device.  There the planner fuses the
element-wise bindings that the reference's psi-composition pass
(ssa.scm:372-426) merges; values equal the reference's per-binding realize,
since every fused map node is still rounded to its dtype.

Names, program structure and rules follow ssa.scm (file:line on each
function).  The outputs of a program are planned together, so each
binding runs once.  ssa-realize/ctx traces the program through the context
(allocations recorded, finalize_context colours them into one arena), then
compiles the replay plan once against the arena and re-runs it each step
without re-planning (ssa.scm:1390-1654).
"""
from __future__ import annotations

import itertools
from typing import Callable, Optional

import numpy as np

from .morph import (Concrete, Expr, Morphism, morph_add, morph_cos, morph_div, morph_from_numpy, morph_map,
                    morph_matmul, morph_mul, morph_negate, morph_pow, morph_reduce, morph_reshape, morph_sin,
                    morph_sub, morph_transpose, NP_DTYPES)

__all__ = [
    "ConstRef", "BindingRef", "SSABinding", "SSAProgram", "morphism_to_ssa", "ssa_constant_id",
    "ssa_loss_binding_val", "ssa_vjp", "ssa_element_wise_fusion_pass", "rebuild_morphism", "ssa_realize",
    "ssa_realize_ctx",
]

_ids = itertools.count()


class ConstRef:
    """const-ref of ssa-value (ssa.scm:104-106): a constant array."""
    __slots__ = ("cid",)

    def __init__(self, cid: str):
        self.cid = cid

    def __repr__(self):
        return f"ConstRef({self.cid})"


class BindingRef:
    """binding-ref of ssa-value (ssa.scm:104-106): a binding's result."""
    __slots__ = ("id",)

    def __init__(self, bid: str):
        self.id = bid

    def __repr__(self):
        return f"BindingRef({self.id})"


def _vid(v) -> str:
    return v.cid if isinstance(v, ConstRef) else v.id


class SSABinding:
    """ssa-binding (ssa.scm:132): name, op ('add', ('reduce', 'sum'), ...),
    inputs (ssa values), shape, dtype, meta.  `build` turns realized or lazy
    inputs into the binding's lazy morphism (rebuild-morphism)."""
    __slots__ = ("name", "op", "inputs", "shape", "dtype", "meta", "build")

    def __init__(self, name, op, inputs, shape, dtype, meta, build: Callable[[list], Morphism]):
        self.name, self.op, self.inputs = name, op, list(inputs)
        self.shape, self.dtype, self.meta, self.build = tuple(shape), dtype, dict(meta), build

    def __repr__(self):
        return f"SSABinding({self.name}, {self.op}, shape={self.shape})"


class SSAProgram:
    """ssa-program (ssa.scm:144-145): constants (cid -> concrete array),
    morph_to_val (morphism identity -> ssa value), bindings in topological
    order, outputs (loss first, then parameter gradients), n_params."""

    def __init__(self, constants: dict, morph_to_val: dict, bindings: list, outputs: list, n_params: int):
        self.constants, self.morph_to_val = constants, morph_to_val
        self.bindings, self.outputs, self.n_params = bindings, outputs, n_params


def _const(value: float, shape, dtype: str) -> Concrete:
    return morph_from_numpy(np.full(tuple(shape), value, dtype=NP_DTYPES[dtype]), dtype)


# ------------------------------------------------------------------ phase 1: morphism-to-ssa

def _ssa_op(m: Expr):
    if m.op == "reduce":
        return ("reduce", m.meta["op"])
    return m.op


def morphism_to_ssa(loss_var) -> SSAProgram:
    """morphism-to-ssa (ssa.scm:437-491): one constant per concrete array and
    one binding per expression node of the variable's value tree, each shared
    node once, in topological order."""
    from .grad import var_value
    constants: dict = {}
    visited: dict = {}
    bindings: list = []

    def visit(m: Morphism):
        key = id(m)
        if key in visited:
            return visited[key][0]
        if isinstance(m, Concrete):
            v = ConstRef(f"cid-{next(_ids)}")
            constants[v.cid] = m
        else:
            ins = [visit(o) for o in m.operands]
            meta = dict(m.meta)
            if m.op == "transpose":
                meta["perm"] = tuple(m.meta["permutation"])
            if m.op == "reduce":
                meta["src-shape"] = tuple(m.operands[0].shape)
            op, shape, dtype, em, ba = m.op, m.shape, m.dtype, dict(m.meta), m.batch_axis
            build = (lambda xs, op=op, shape=shape, dtype=dtype, em=em, ba=ba: Expr(op, list(xs), shape, dtype,
                                                                                   dict(em), ba))
            b = SSABinding(f"bid-{next(_ids)}", _ssa_op(m), ins, m.shape, m.dtype, meta, build)
            bindings.append(b)
            v = BindingRef(b.name)
        visited[key] = (v, m)      # the morphism is kept alive so its identity stays unique
        return v

    loss_val = visit(var_value(loss_var))
    return SSAProgram(constants, {k: v for k, (v, _) in visited.items()}, bindings, [loss_val], 0)


def ssa_constant_id(prog: SSAProgram, m: Morphism) -> Optional[ConstRef]:
    """ssa-constant-id (ssa.scm:498-501): the constant of morphism m, or None."""
    v = prog.morph_to_val.get(id(m))
    return v if isinstance(v, ConstRef) and prog.constants.get(v.cid) is m else None


def ssa_loss_binding_val(prog: SSAProgram):
    """ssa-loss-binding-val (ssa.scm:503-505): the first output."""
    return prog.outputs[0]


# ------------------------------------------------------------------ phase 2: ssa-vjp

def _transpose_perm(rank: int) -> tuple:
    """transpose-perm (ssa.scm:1047-1052): (1 0), or the last two axes swapped."""
    return (1, 0) if rank == 2 else tuple(range(rank - 2)) + (rank - 1, rank - 2)


def ssa_vjp(fwd: SSAProgram, param_vals: list, loss_val) -> SSAProgram:
    """ssa-vjp (ssa.scm:517-1033): reverse sweep over the forward bindings,
    emitting backward bindings with the reference's rules and accumulating
    adjoints by `add` in the order they arrive.  Outputs are add(loss, 0)
    followed by each parameter's gradient (parameters with none are
    dropped, as filter-map does)."""
    sd: dict = {}
    for b in fwd.bindings:
        sd[b.name] = (b.shape, b.dtype)
    for cid, m in fwd.constants.items():
        sd[cid] = (tuple(m.shape), m.dtype)
    bwd: list = []
    adjoint: dict = {}
    param_grad: dict = {}
    params = {_vid(v) for v in param_vals}

    def shape_of(v):
        return sd[_vid(v)][0]

    def emit(op, inputs, shape, dtype, build, meta=None):
        name = f"adj-{next(_ids)}"
        bwd.append(SSABinding(name, op, inputs, shape, dtype, meta or {}, build))
        sd[name] = (tuple(shape), dtype)
        return BindingRef(name)

    def const(value, shape, dtype):
        m = _const(value, shape, dtype)
        cid = f"cid-{next(_ids)}"
        fwd.constants[cid] = m
        sd[cid] = (tuple(shape), dtype)
        return ConstRef(cid)

    def accumulate(table: dict, key: str, new, shape, dtype):
        old = table.get(key)
        table[key] = new if old is None else emit("add", [old, new], shape, dtype, lambda x: morph_add(x[0], x[1]))

    def accumulate_input(iv, new):
        shape, dtype = sd[_vid(iv)]
        if isinstance(iv, BindingRef):
            accumulate(adjoint, iv.id, new, shape, dtype)
        elif iv.cid in params:
            accumulate(param_grad, iv.cid, new, shape, dtype)

    def reduce_sum_to(g, g_shape, target, dtype):
        """emit-reduce-sum-to! (ssa.scm:589-628)."""
        target = tuple(target)
        extra = len(g_shape) - len(target)
        cur, cur_shape = g, tuple(g_shape)
        if extra > 0:
            axes = list(range(extra))
            cur_shape = cur_shape[extra:]
            cur = emit(("reduce", "sum"), [cur], cur_shape, dtype,
                       lambda x, axes=axes: morph_reduce("sum", x[0], axes, False))
        for k in range(len(target)):
            if target[k] == 1 and cur_shape[k] > 1:
                cur_shape = cur_shape[:k] + (1,) + cur_shape[k + 1:]
                cur = emit(("reduce", "sum"), [cur], cur_shape, dtype,
                           lambda x, k=k: morph_reduce("sum", x[0], [k], True))
        return cur

    def broadcast_grad(g, src_shape, axes, keepdims, dtype):
        """emit-broadcast-grad! (ssa.scm:643-669): reshape to the keepdims
        shape, then multiply by a ones constant of the source shape."""
        kd = tuple(1 if i in axes else s for i, s in enumerate(src_shape))
        gk = g if keepdims else emit("reshape", [g], kd, dtype, lambda x, kd=kd: morph_reshape(x[0], kd))
        ones = const(1.0, src_shape, dtype)
        return emit("mul", [gk, ones], src_shape, dtype, lambda x: morph_mul(x[0], x[1]))

    mul = lambda x: morph_mul(x[0], x[1])
    div = lambda x: morph_div(x[0], x[1])
    neg = lambda x: morph_negate(x[0])

    # seed: dL/dL = ones of the loss shape, a constant (ssa.scm:672-685)
    loss_b = next(b for b in fwd.bindings if b.name == _vid(loss_val))
    adjoint[loss_b.name] = const(1.0, loss_b.shape, loss_b.dtype)

    for b in reversed(fwd.bindings):
        g = adjoint.get(b.name)
        if g is None:
            continue
        op, ins, dtype, gs = b.op, b.inputs, b.dtype, shape_of(g)
        x = ins[0] if ins else None
        if op in ("add", "sub"):                                        # ssa.scm:714-738
            y = ins[1]
            accumulate_input(x, reduce_sum_to(g, gs, shape_of(x), dtype))
            gy = g if op == "add" else emit("negate", [g], gs, dtype, neg)
            accumulate_input(y, reduce_sum_to(gy, gs, shape_of(y), dtype))
        elif op == "mul":                                               # ssa.scm:740-753
            y = ins[1]
            accumulate_input(x, reduce_sum_to(emit("mul", [g, y], gs, dtype, mul), gs, shape_of(x), dtype))
            accumulate_input(y, reduce_sum_to(emit("mul", [g, x], gs, dtype, mul), gs, shape_of(y), dtype))
        elif op == "div":                                               # ssa.scm:755-777
            y = ins[1]
            accumulate_input(x, reduce_sum_to(emit("div", [g, y], gs, dtype, div), gs, shape_of(x), dtype))
            y2 = emit("mul", [y, y], shape_of(y), dtype, lambda v: morph_mul(v[0], v[1]))
            xy2 = emit("div", [x, y2], gs, dtype, div)
            ndy = emit("negate", [emit("mul", [g, xy2], gs, dtype, mul)], gs, dtype, neg)
            accumulate_input(y, reduce_sum_to(ndy, gs, shape_of(y), dtype))
        elif op == "pow":                                               # ssa.scm:779-797
            n = ins[1]
            one = const(1.0, (1,), dtype)
            nm1 = emit("sub", [n, one], shape_of(n), dtype, lambda v: morph_sub(v[0], v[1]))
            xp = emit("pow", [x, nm1], gs, dtype, lambda v: morph_pow(v[0], v[1]))
            nxp = emit("mul", [n, xp], gs, dtype, mul)
            accumulate_input(x, reduce_sum_to(emit("mul", [g, nxp], gs, dtype, mul), gs, shape_of(x), dtype))
        elif op == "negate":                                            # ssa.scm:799-806
            accumulate_input(x, reduce_sum_to(emit("negate", [g], gs, dtype, neg), gs, shape_of(x), dtype))
        elif op == "abs":                                               # ssa.scm:808-821
            sx = emit("map", [x], shape_of(x), dtype, lambda v: morph_map(lambda t: (t > 0.0) - (t < 0.0), v[0]))
            accumulate_input(x, reduce_sum_to(emit("mul", [g, sx], gs, dtype, mul), gs, shape_of(x), dtype))
        elif op == "sqrt":                                              # ssa.scm:823-836
            two = const(2.0, (1,), dtype)
            to = emit("mul", [two, BindingRef(b.name)], gs, dtype, mul)
            accumulate_input(x, reduce_sum_to(emit("div", [g, to], gs, dtype, div), gs, shape_of(x), dtype))
        elif op == "exp":                                               # ssa.scm:838-846
            d = emit("mul", [g, BindingRef(b.name)], gs, dtype, mul)
            accumulate_input(x, reduce_sum_to(d, gs, shape_of(x), dtype))
        elif op == "log":                                               # ssa.scm:848-855
            accumulate_input(x, reduce_sum_to(emit("div", [g, x], gs, dtype, div), gs, shape_of(x), dtype))
        elif op == "sin":                                               # ssa.scm:857-866
            c = emit("cos", [x], shape_of(x), dtype, lambda v: morph_cos(v[0]))
            accumulate_input(x, reduce_sum_to(emit("mul", [g, c], gs, dtype, mul), gs, shape_of(x), dtype))
        elif op == "cos":                                               # ssa.scm:868-879
            s = emit("sin", [x], shape_of(x), dtype, lambda v: morph_sin(v[0]))
            ns = emit("negate", [s], shape_of(x), dtype, neg)
            accumulate_input(x, reduce_sum_to(emit("mul", [g, ns], gs, dtype, mul), gs, shape_of(x), dtype))
        elif op == "relu":                                              # ssa.scm:881-894
            h = emit("map", [x], shape_of(x), dtype, lambda v: morph_map(lambda t: t > 0.0, v[0]))
            accumulate_input(x, reduce_sum_to(emit("mul", [g, h], gs, dtype, mul), gs, shape_of(x), dtype))
        elif op in ("sigmoid", "tanh"):                                 # ssa.scm:896-920
            f = (lambda t: t * (1.0 - t)) if op == "sigmoid" else (lambda t: 1.0 - t * t)
            d = emit("map", [BindingRef(b.name)], gs, dtype, lambda v, f=f: morph_map(f, v[0]))
            accumulate_input(x, reduce_sum_to(emit("mul", [g, d], gs, dtype, mul), gs, shape_of(x), dtype))
        elif op == "matmul":                                            # ssa.scm:922-940
            y = ins[1]
            xs, ys = shape_of(x), shape_of(y)
            perm = _transpose_perm(len(xs))
            yt = emit("transpose", [y], tuple(ys[p] for p in perm), dtype,
                      lambda v, perm=perm: morph_transpose(v[0], perm), {"perm": perm})
            xt = emit("transpose", [x], tuple(xs[p] for p in perm), dtype,
                      lambda v, perm=perm: morph_transpose(v[0], perm), {"perm": perm})
            da = emit("matmul", [g, yt], xs, dtype, lambda v: morph_matmul(v[0], v[1]))
            db = emit("matmul", [xt, g], ys, dtype, lambda v: morph_matmul(v[0], v[1]))
            accumulate_input(x, da)
            accumulate_input(y, db)
        elif op == "transpose":                                         # ssa.scm:942-950
            perm = b.meta["perm"]
            inv = tuple(int(i) for i in np.argsort(perm))
            accumulate_input(x, emit("transpose", [g], shape_of(x), dtype,
                                     lambda v, inv=inv: morph_transpose(v[0], inv), {"perm": inv}))
        elif op == "reshape":                                           # ssa.scm:952-957
            xs = shape_of(x)
            accumulate_input(x, emit("reshape", [g], xs, dtype, lambda v, xs=xs: morph_reshape(v[0], xs)))
        elif op in (("reduce", "mean"), ("reduce", "sum")):             # ssa.scm:959-983
            src = b.meta["src-shape"]
            axes, keepdims = list(b.meta["axes"]), bool(b.meta["keepdims"])
            gg = g
            if op == ("reduce", "mean"):
                n = float(np.prod([src[a] for a in axes])) if axes else 1.0
                nv = const(n, (1,), dtype)
                gg = emit("div", [g, nv], gs, dtype, div)
            accumulate_input(x, broadcast_grad(gg, src, axes, keepdims, dtype))
        # reduce max, map and every other op: no gradient (ssa.scm:985-995)

    # the loss output: add(loss, zero) keeps the loss buffer live to the end
    # in the context's lifetime analysis (ssa.scm:999-1020)
    zero = const(0.0, loss_b.shape, loss_b.dtype)
    loss_out = emit("add", [loss_val, zero], loss_b.shape, loss_b.dtype, lambda v: morph_add(v[0], v[1]))
    grads = [param_grad[_vid(p)] for p in param_vals if _vid(p) in param_grad]
    # the joint forward + backward program goes through the psi-composition
    # fusion pass, as ssa.scm:1024-1032 does
    return ssa_element_wise_fusion_pass(
        SSAProgram(fwd.constants, fwd.morph_to_val, fwd.bindings + bwd, [loss_out] + grads, len(param_vals)))


# ------------------------------------------------------------------ element-wise fusion pass

class _Shape(Morphism):
    """An operand stand-in with only shape and dtype: enough for a
    constructor to give the node's program."""

    def __init__(self, shape, dtype):
        self.shape, self.dtype, self.batch_axis = tuple(shape), dtype, -1


def _binding_program(b: SSABinding, sd: dict):
    """The element-wise program of a binding (its constructor's `prog`), or
    None for matmul, reductions and structural bindings."""
    if b.op in ("matmul", "matvec", "dot", "reshape", "transpose", "slice") or isinstance(b.op, tuple):
        return None
    m = b.build([_Shape(*sd[_vid(v)]) for v in b.inputs])
    return list(m.meta["prog"]) if isinstance(m, Expr) and "prog" in m.meta else None


def _depth(prog) -> int:
    """The deepest stack a postfix program reaches."""
    from . import _abi as A
    sp = depth = 0
    for (op, _, _) in prog:
        sp += 1 if op in (A.OP["LOAD"], A.OP["CONST"], A.OP["ICONST"]) else (-1 if op >= A.OP["ADD"] else 0)
        depth = max(depth, sp)
    return depth


def ssa_element_wise_fusion_pass(prog: SSAProgram) -> SSAProgram:
    """ssa-element-wise-fusion-pass (ssa.scm:372-426): a greedy scan that
    merges a producer binding into the binding right after it when the
    producer has one use, is that binding's first input, has its shape,
    reads only operands of its own shape, and both are element-wise.  The
    merged binding keeps the consumer's name and computes
    consumer(producer(...), ...) in double with no rounding of the
    intermediate (compose-flat-combiners), stored to the consumer's dtype.

    ssa_vjp applies this pass to the joint program, as the reference does,
    so a merged chain runs on the device as one map node whose program
    rounds only its final value; in f32 programs that differs from the
    unfused node-by-node rounding, in f64 it does not.  A producer that is
    also a program output is not merged away.  A merge is skipped when the
    result would exceed a map node's 4 operands or program limits."""
    from . import _abi as A
    sd: dict = {}
    for cid, m in prog.constants.items():
        sd[cid] = (tuple(m.shape), m.dtype)
    for b in prog.bindings:
        sd[b.name] = (b.shape, b.dtype)
    uses: dict = {b.name: 0 for b in prog.bindings}
    for b in prog.bindings:
        for v in b.inputs:
            if isinstance(v, BindingRef) and v.id in uses:
                uses[v.id] += 1
    # a program output is read after the program: it keeps its binding
    # (ssa-compute-use-counts counts binding inputs only; a producer that is
    # also an output would otherwise vanish into its consumer)
    for v in prog.outputs:
        if isinstance(v, BindingRef) and v.id in uses:
            uses[v.id] += 1
    bs, out = list(prog.bindings), []
    while bs:
        p = bs.pop(0)
        if bs:
            c = bs[0]
            pp, cp = _binding_program(p, sd), _binding_program(c, sd)
            ok = (pp is not None and cp is not None and uses.get(p.name) == 1 and c.inputs
                  and isinstance(c.inputs[0], BindingRef) and c.inputs[0].id == p.name and p.shape == c.shape
                  and all(sd[_vid(v)][0] == p.shape for v in p.inputs)
                  and len(p.inputs) + len(c.inputs) - 1 <= A.NODE_MAX_IN)
            if ok:
                n_p = len(p.inputs)
                fused = []
                for (op, a, imm) in cp:
                    if op == A.OP["LOAD"] and a == 0:
                        fused += pp
                    elif op == A.OP["LOAD"]:
                        fused.append((op, n_p + a - 1, imm))
                    else:
                        fused.append((op, a, imm))
                if len(fused) <= A.PROG_MAX and _depth(fused) <= A.STACK_MAX:
                    shape, dtype = c.shape, c.dtype
                    build = (lambda xs, shape=shape, dtype=dtype, fused=fused:
                             Expr("map", list(xs), shape, dtype, {"prog": list(fused)}))
                    merged = SSABinding(c.name, c.op, p.inputs + c.inputs[1:], shape, dtype,
                                        dict(c.meta, fused=True), build)
                    bs[0] = merged            # the merged binding may absorb the next one too
                    continue
        out.append(p)
    return SSAProgram(prog.constants, prog.morph_to_val, out, prog.outputs, prog.n_params)


# ------------------------------------------------------------------ phase 3: realization

def rebuild_morphism(b: SSABinding, inputs: list) -> Morphism:
    """rebuild-morphism (ssa.scm:1066-1128): the binding's lazy morphism over
    its inputs (concrete or lazy).  ssa-vjp records some bindings with the
    adjoint's shape where the constructor broadcasts a rank-0 value against a
    (1,) constant; such a result is reshaped to the recorded shape (same
    elements), so later rules see the shapes the program states."""
    m = b.build(inputs)
    if tuple(m.shape) != b.shape:
        if int(np.prod(m.shape)) != int(np.prod(b.shape)):
            raise ValueError(f"rebuild-morphism: {b.op} gives shape {tuple(m.shape)}, binding has {b.shape}")
        m = morph_reshape(m, b.shape)
    return m


def _output_trees(prog: SSAProgram) -> list:
    vals: dict = dict(prog.constants)
    for b in prog.bindings:
        vals[b.name] = rebuild_morphism(b, [vals[_vid(v)] for v in b.inputs])
    return [vals[_vid(o)] for o in prog.outputs]


def ssa_realize(prog: SSAProgram, realize: Optional[Callable[[Morphism], Concrete]] = None) -> list:
    """ssa-realize (ssa.scm:1130-1156): the outputs as concrete arrays.  On
    the device the outputs' trees are planned and run together, so every
    binding is computed once, as the reference's binding loop computes it
    (the loss and the gradients share the forward bindings).  A `realize`
    given (e.g. the oracle's) is applied to each output tree in turn."""
    trees = _output_trees(prog)
    if realize is None:
        from .realize import realize_many
        return realize_many(trees)
    return [o if isinstance(o, Concrete) else realize(o) for o in trees]


def _const_devs(prog: SSAProgram) -> tuple:
    """Identity of each constant's device copy: a constant whose host vector
    was rewritten (host_changed) gets a new device copy, and a replay plan
    compiled over the old one is stale."""
    return tuple(id(m._dev) for m in prog.constants.values())


def ssa_realize_ctx(ctx, prog: SSAProgram, stream=None) -> list:
    """ssa-realize/ctx (ssa.scm:1661-1749).

    Trace mode: the outputs are realized together through the context (each
    binding once), every output pinned (context-pin-output! applies while
    tracing only, ssa.scm:1716-1717), and returned on the host.

    Replay mode (after finalize_context and reset_context): the first call
    compiles the replay plan, i.e. plans the program once against the
    context's arena (compile-replay-plan, ssa.scm:1390-1512); this and every
    later call runs it without re-planning or allocating
    (execute-replay-plan, ssa.scm:1519-1654).  The outputs are returned as
    the arena buffers themselves, as the reference returns its pool vectors:
    read them before the next replay overwrites them.  A constant rewritten
    through host_changed() makes the next call compile the plan again.
    The compiling call also captures the plan's launches into a CUDA graph,
    which every later replay launches as one.  `stream` (a CUDA stream pointer) orders the replay's
    launches."""
    from .context import context_stats, realize_ctx_many, replay_plan
    from .realize import Plan
    trace = context_stats(ctx)["mode"] == "trace"
    if trace:
        trees = _output_trees(prog)
        lazy = [o for o in trees if not isinstance(o, Concrete)]
        if not lazy:
            return trees
        _, res = realize_ctx_many(ctx, lazy, pin_output=True)
        it = iter(res)
        return [o if isinstance(o, Concrete) else next(it) for o in trees]
    cache = prog.__dict__.setdefault("_replay", {})
    key = ctx.handle
    entry = cache.get(key)
    if entry is not None and entry[2] != _const_devs(prog):
        entry = None
    if entry is None:
        trees = _output_trees(prog)
        lazy = [o for o in trees if not isinstance(o, Concrete)]
        plan = Plan(lazy, ctx) if lazy else None
        if plan is not None:
            plan.execute(stream)
            if plan.stats()["launches"] > 1:
                plan.capture_graph(stream)   # later replays launch one graph (captured, not run, here)
        entry = (plan, trees, _const_devs(prog))
        cache[key] = entry
    else:
        plan = entry[0]
        if plan is not None:
            replay_plan(ctx, plan, stream)
    plan, trees = entry[0], entry[1]
    if plan is None:
        return list(trees)
    it = iter(plan.results(arena=True))
    return [o if isinstance(o, Concrete) else next(it) for o in trees]
