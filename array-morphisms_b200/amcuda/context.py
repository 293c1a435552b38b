"""realize/ctx: memory-reuse contexts backed by one device arena.

Mirrors context.scm's public API (make-morphism-context, realize/ctx,
finalize-context!, reset-context!, context-stats, context-pin-output!).
In trace mode every buffer a realize allocates is recorded; finalize colours
the records greedily into one device arena; in replay mode (after reset)
realize/ctx of the same tree takes its buffers from the arena and allocates
nothing.  Results of replay live in the arena and are copied to the host
before the next replay can overwrite them.
"""
from __future__ import annotations

import ctypes as C

from . import _abi as A
from .morph import Concrete, Morphism
from .realize import Plan, _ensure_init


class MorphismContext:
    def __init__(self):
        _ensure_init()
        h = C.c_uint64(0)
        A.call("amc_ctx_create", C.byref(h))
        self.handle = h.value

    def __del__(self):
        try:
            if self.handle and A._lib is not None:
                A._lib.amc_ctx_destroy(self.handle)
        except Exception:
            pass
        self.handle = 0


def make_morphism_context() -> MorphismContext:
    return MorphismContext()


def realize_ctx(ctx: MorphismContext, m: Morphism, pin_output: bool = False) -> Concrete:
    """realize/ctx (context.scm:125-131).  pin_output marks the result's
    allocation output-pinned (context-pin-output!, :190-200) while tracing."""
    if isinstance(m, Concrete):
        return m
    p = Plan(m, ctx)
    p.execute()
    if pin_output:
        A.call("amc_ctx_pin_output", ctx.handle, p.handle)
    return p.result(keep_device=False)


def realize_ctx_many(ctx: MorphismContext, ms: list, pin_output: bool = False) -> tuple:
    """The lazy morphisms of `ms` realized together through the context in
    one plan (each shared node once); pin_output pins every result while
    tracing.  Returns (plan, results)."""
    p = Plan(ms, ctx)
    p.execute()
    if pin_output:
        A.call("amc_ctx_pin_output", ctx.handle, p.handle)
    return p, p.results(keep_device=False)


def replay_plan(ctx: MorphismContext, plan: Plan, stream: int | None = None) -> None:
    """Run a plan created in the context's replay mode again on its arena
    buffers, without re-planning (amc_ctx_replay; execute-replay-plan,
    ssa.scm:1519-1654)."""
    A.call("amc_ctx_replay", ctx.handle, plan.handle, C.c_void_p(stream or 0))


def plan_ctx(ctx: MorphismContext, m: Morphism) -> Plan:
    """A replayable plan bound to the context (for repeated execution or
    CUDA-graph capture without re-planning)."""
    return Plan(m, ctx)


def finalize_context(ctx: MorphismContext) -> None:
    A.call("amc_ctx_finalize", ctx.handle)


def reset_context(ctx: MorphismContext) -> None:
    A.call("amc_ctx_reset", ctx.handle)


def context_stats(ctx: MorphismContext) -> dict:
    """context-stats (context.scm:167-183) plus the arena size."""
    a, b, by, mode = C.c_int32(), C.c_int32(), C.c_int64(), C.c_int32()
    A.call("amc_ctx_stats", ctx.handle, C.byref(a), C.byref(b), C.byref(by), C.byref(mode))
    st = {"mode": "replay" if mode.value else "trace", "allocations": a.value}
    if mode.value:
        st["buffers"] = b.value
        st["arena_bytes"] = by.value
    return st


def colour(dtypes, sizes, inputs, pinned=None):
    """The context's greedy colouring on explicit allocation records:
    returns (assignment, n_buffers)."""
    n = len(dtypes)
    off = [0]
    flat = []
    for ins in inputs:
        flat.extend(ins)
        off.append(len(flat))
    DT = (C.c_int32 * max(n, 1))(*dtypes)
    SZ = (C.c_int64 * max(n, 1))(*sizes)
    OF = (C.c_int32 * (n + 1))(*off)
    IN = (C.c_int32 * max(len(flat), 1))(*flat)
    PN = (C.c_int32 * max(n, 1))(*(pinned or [0] * n))
    AS = (C.c_int32 * max(n, 1))()
    NB = C.c_int32()
    A.call("amc_colour", n, DT, SZ, OF, IN, PN, AS, C.byref(NB))
    return list(AS)[:n], NB.value
