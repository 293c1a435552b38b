"""realize/ctx on the device against the reference's tests/test-context.scm
(file:line per group): trace recording, zero-copy transparency,
finalization, replay correctness, buffer reuse, repeated replays,
reductions, mixed dtypes and pinning errors.

One deliberate difference: the planner fuses a chain of element-wise nodes
into one kernel, so a chain records one allocation where the reference,
realizing node by node, records one per node (test-context.scm:59-67).
Buffer counts therefore only get smaller."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def ml(amc, vals, shape, dt="f64"):
    return amc.morph_from_list(vals, tuple(shape), dt)


def stats(amc, ctx):
    return amc.context_stats(ctx)


def replay_equals_reference(amc, tree, tol=0.0, runs=1):
    ref = np.asarray(oracle.values(tree), dtype=np.float64)
    ctx = amc.make_morphism_context()
    amc.realize_ctx(ctx, tree)
    amc.finalize_context(ctx)
    for _ in range(runs):
        amc.reset_context(ctx)
        got = np.asarray(amc.realize_ctx(ctx, tree).values(), dtype=np.float64)
        np.testing.assert_allclose(got, ref, rtol=tol, atol=0)
    return ctx


def test_trace_recording_and_zero_copy(amc):                    # test-context.scm:45-105
    ctx = amc.make_morphism_context()
    assert stats(amc, ctx)["mode"] == "trace"
    a, b = ml(amc, [1, 2, 3], [3]), ml(amc, [4, 5, 6], [3])
    amc.realize_ctx(ctx, amc.morph_add(a, b))
    assert stats(amc, ctx)["allocations"] == 1
    ctx = amc.make_morphism_context()
    x, two = ml(amc, [1, 2], [2]), ml(amc, [2, 2], [2])
    amc.realize_ctx(ctx, amc.morph_mul(amc.morph_add(x, x), two))
    assert stats(amc, ctx)["allocations"] == 1          # fused: one kernel, one output
    ctx = amc.make_morphism_context()
    amc.realize_ctx(ctx, a)
    assert stats(amc, ctx)["allocations"] == 0
    ctx = amc.make_morphism_context()
    amc.realize_ctx(ctx, amc.morph_reshape(ml(amc, [1, 2, 3, 4, 5, 6], [6]), (2, 3)))
    amc.realize_ctx(ctx, amc.morph_transpose(ml(amc, [1, 2, 3, 4], [2, 2])))
    assert stats(amc, ctx)["allocations"] == 0
    r = amc.morph_reshape(ml(amc, [1, 2, 3, 4], [4]), (2, 2))
    amc.realize_ctx(ctx, amc.morph_add(r, r))
    assert stats(amc, ctx)["allocations"] == 1


def test_finalization_and_state_errors(amc):                    # test-context.scm:108-135, 244-248
    ctx = amc.make_morphism_context()
    with pytest.raises(amc.AmcError):
        amc.reset_context(ctx)
    a = ml(amc, [1, 2], [2])
    amc.realize_ctx(ctx, amc.morph_add(a, a))
    amc.finalize_context(ctx)
    st = stats(amc, ctx)
    assert st["mode"] == "replay" and st["buffers"] >= 1
    with pytest.raises(amc.AmcError):
        amc.finalize_context(ctx)
    amc.reset_context(ctx)
    with pytest.raises(amc.AmcError):
        amc.realize_ctx(ctx, amc.morph_add(a, a), pin_output=True)   # pinning is for tracing only


def test_replay_correctness(amc):                               # test-context.scm:140-190
    a = ml(amc, [1, 2, 3, 4], [4])
    replay_equals_reference(amc, amc.morph_add(ml(amc, [1, 2, 3], [3]), ml(amc, [10, 20, 30], [3])))
    replay_equals_reference(amc, amc.morph_mul(amc.morph_add(a, a), ml(amc, [0.5] * 4, [4])))
    r = amc.morph_reshape(a, (2, 2))
    replay_equals_reference(amc, amc.morph_add(r, r))
    replay_equals_reference(amc, amc.morph_sqrt(ml(amc, [1, 4, 9], [3])), tol=1e-12)


def test_memory_reduction(amc):                                 # test-context.scm:193-222
    a, two = ml(amc, [1, 2, 3, 4], [4]), ml(amc, [2, 2], [2])
    b = amc.morph_add(a, a)
    d = amc.morph_add(amc.morph_mul(b, b), a)
    ctx = replay_equals_reference(amc, d)
    assert stats(amc, ctx)["buffers"] <= stats(amc, ctx)["allocations"]
    x = ml(amc, [1, 2], [2])
    e = amc.morph_add(amc.morph_add(amc.morph_add(amc.morph_add(x, two), two), two), two)
    ctx = replay_equals_reference(amc, e)
    assert stats(amc, ctx)["buffers"] <= 2


def test_repeated_replays(amc):                                 # test-context.scm:226-268
    a = ml(amc, [1, 2, 3], [3])
    replay_equals_reference(amc, amc.morph_add(a, a), runs=3)
    b = ml(amc, [1, 2, 3, 4], [4])
    replay_equals_reference(amc, amc.morph_add(amc.morph_mul(b, b), ml(amc, [1] * 4, [4])), runs=5)


def test_reductions(amc):                                       # test-context.scm:271-316
    a = ml(amc, [[1, 2], [3, 4]], [2, 2])
    ctx = amc.make_morphism_context()
    amc.realize_ctx(ctx, amc.morph_reduce("sum", a, [1]))
    assert stats(amc, ctx)["allocations"] == 1
    replay_equals_reference(amc, amc.morph_reduce("sum", a, [1]))
    replay_equals_reference(amc, amc.morph_reduce("mean", ml(amc, [2, 4, 6, 8], [4]), [0]))
    s = amc.morph_reduce("sum", ml(amc, [[1, 3], [5, 7]], [2, 2]), [0])
    replay_equals_reference(amc, amc.morph_mul(s, ml(amc, [2, 2], [2])))


def test_mixed_dtypes(amc):                                     # test-context.scm:319-363
    a32, a64 = ml(amc, [1, 2, 3], [3], "f32"), ml(amc, [1, 2], [2])
    replay_equals_reference(amc, amc.morph_add(a32, a32))
    c32, c64 = amc.make_morphism_context(), amc.make_morphism_context()
    b32, b64 = amc.morph_add(ml(amc, [1, 2], [2], "f32"), ml(amc, [1, 2], [2], "f32")), amc.morph_add(a64, a64)
    amc.realize_ctx(c32, b32)
    amc.realize_ctx(c64, b64)
    amc.finalize_context(c32)
    amc.finalize_context(c64)
    amc.reset_context(c32)
    amc.reset_context(c64)
    r32, r64 = amc.realize_ctx(c32, b32), amc.realize_ctx(c64, b64)
    assert r32.dtype == "f32" and r32.values().tolist() == [2.0, 4.0]
    assert r64.dtype == "f64" and r64.values().tolist() == [2.0, 4.0]


def test_example8_polyphase_allocations(amc):
    """examples/example-08-polyphase-filter-bank.scm:57-83: the four strided
    branches and a nested decimation allocate nothing under a context; the
    4-tap average allocates its result only (the reference's product and
    reduction nodes, 2 allocations, are one fused launch here)."""
    x = amc.morph_from_list([float(v) for v in range(16)], (16,))
    branches = [amc.morph_slice(x, [mm], [16], 4) for mm in range(4)]
    dec = amc.morph_slice(branches[0], [0], [4], 2)
    ctx = amc.make_morphism_context()
    for b in branches + [dec]:
        amc.realize_ctx(ctx, b)
    assert stats(amc, ctx)["allocations"] == 0
    filt = amc.morph_reduce("sum", amc.morph_mul(branches[0], amc.morph_from_list([0.25] * 4, (4,))))
    ctx2 = amc.make_morphism_context()
    r = amc.realize_ctx(ctx2, filt)
    assert stats(amc, ctx2)["allocations"] == 1 and float(r.values()) == 6.0


def test_blas_in_context(amc):
    """test-batch-ops.scm:387-445: matmul, a batched matmul with a shared
    weight and matvec traced and replayed in a context, equal to realize."""
    A = ml(amc, [[1, 2], [3, 4]], [2, 2])
    B = ml(amc, [[5, 6], [7, 8]], [2, 2])
    A3 = amc.stack_into_batch([ml(amc, [[1, 2], [3, 4]], [2, 2]), ml(amc, [[5, 6], [7, 8]], [2, 2])])
    for tree in (amc.morph_matmul(A, B), amc.morph_batch_matmul(A3, ml(amc, [[1, 0], [0, 1]], [2, 2])),
                 amc.morph_matvec(ml(amc, [[1, 2, 3], [4, 5, 6]], [2, 3]), ml(amc, [1, 2, 3], [3]))):
        ctx = amc.make_morphism_context()
        trace = np.asarray(amc.realize_ctx(ctx, tree).values())
        assert np.array_equal(trace, np.asarray(oracle.values(tree)))
        amc.finalize_context(ctx)
        amc.reset_context(ctx)
        assert np.array_equal(np.asarray(amc.realize_ctx(ctx, tree).values()), trace)
