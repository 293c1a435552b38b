"""Device parity of the context arena, the BLAS record entries and the
workload entry points (filter bank, linear regression, attention, conv)."""
import ctypes as C

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def _same(a, b):
    a, b = np.asarray(a), np.asarray(b)
    assert a.shape == b.shape
    a, b = a.reshape(-1), b.reshape(-1).astype(a.dtype) if b.dtype != a.dtype else b.reshape(-1)
    assert np.array_equal(a.view(np.uint8), b.view(np.uint8)), np.max(np.abs(a.astype(np.float64) - b))


# ---------------------------------------------------------------------------- context
def test_context_trace_finalize_replay(amc):
    """Reference example-06 (per-sample RMS): replay reproduces the traced
    values, allocates nothing, and colouring gives fewer buffers."""
    a = amc.morph_from_list([3.0, 4.0, 0.0, 1.0], (4,))
    b = amc.morph_from_list([4.0, 3.0, 5.0, 2.0], (4,))
    half = amc.morph_from_list([0.5] * 4, (4,))
    rms = amc.morph_sqrt(amc.morph_mul(amc.morph_add(amc.morph_mul(a, a), amc.morph_mul(b, b)), half))
    ctx = amc.make_morphism_context()
    r0 = amc.realize_ctx(ctx, rms).values()
    st = amc.context_stats(ctx)
    assert st["mode"] == "trace" and st["allocations"] >= 1
    amc.finalize_context(ctx)
    st = amc.context_stats(ctx)
    assert st["mode"] == "replay" and st["buffers"] <= st["allocations"]
    exp = np.sqrt(0.5 * (np.array([3, 4, 0, 1.0]) ** 2 + np.array([4, 3, 5, 2.0]) ** 2))
    np.testing.assert_allclose(r0, exp, rtol=1e-15)
    for _ in range(4):
        amc.reset_context(ctx)
        _same(amc.realize_ctx(ctx, rms).values(), r0)


def test_context_zero_copy_records_nothing(amc):
    ctx = amc.make_morphism_context()
    a = amc.morph_from_list([1.0, 2.0, 3.0, 4.0, 5.0, 6.0], (6,))
    amc.realize_ctx(ctx, amc.morph_transpose(amc.morph_reshape(a, (2, 3))))
    assert amc.context_stats(ctx)["allocations"] == 0
    amc.realize_ctx(ctx, amc.morph_add(amc.morph_reshape(a, (2, 3)), amc.morph_reshape(a, (2, 3))))
    assert amc.context_stats(ctx)["allocations"] == 1


def test_context_replay_of_multi_kernel_program(amc):
    """A program with several materialised nodes: the arena is smaller than
    the sum of the traced buffers and replay is bit-identical."""
    rng = np.random.default_rng(1)
    x = amc.morph_from_numpy(rng.standard_normal((64, 48)))
    w = amc.morph_from_numpy(rng.standard_normal((48, 32)))
    h1 = amc.morph_relu(amc.morph_matmul(x, w))
    h2 = amc.morph_matmul(amc.morph_transpose(h1), h1)
    out = amc.morph_reduce("sum", amc.morph_pad(h2, [(1, 1), (1, 1)], "edge"), (0,))
    ctx = amc.make_morphism_context()
    r0 = amc.realize_ctx(ctx, out, pin_output=True).values()
    _same(r0, oracle.realize(out).values())
    amc.finalize_context(ctx)
    for _ in range(3):
        amc.reset_context(ctx)
        _same(amc.realize_ctx(ctx, out).values(), r0)


def test_context_replay_with_gemm_epilogues_and_scan(amc):
    """Two GEMMs with folded epilogues feeding a SCAN node, traced, coloured
    and replayed: the epilogue outputs are written while their GEMM reads A
    and B, so colouring must keep those live; replay is bit-identical."""
    from test_batch_ops import _oracle_dag
    rng = np.random.default_rng(4)
    x = amc.morph_from_numpy(rng.standard_normal((64, 48)))
    w1 = amc.morph_from_numpy(rng.standard_normal((48, 32)))
    b1 = amc.morph_from_numpy(rng.standard_normal((32,)))
    w2 = amc.morph_from_numpy(rng.standard_normal((32, 16)))
    h = amc.morph_relu(amc.morph_add(amc.morph_matmul(x, w1), b1))
    y = amc.morph_map(lambda t: t * 0.5 - t * t * 0.01, amc.morph_matmul(h, w2))
    out = amc.batch_scan(amc.morph_add, amc.morph_from_numpy(np.zeros(16)), y)
    assert "scan" in out.meta and amc.Plan(out).stats()["launches"] == 3
    ctx = amc.make_morphism_context()
    r0 = amc.realize_ctx(ctx, out, pin_output=True).values()
    _same(r0, oracle.values(_oracle_dag(out, {})))
    amc.finalize_context(ctx)
    for _ in range(3):
        amc.reset_context(ctx)
        _same(amc.realize_ctx(ctx, out).values(), r0)


def test_context_replay_state_errors(amc):
    ctx = amc.make_morphism_context()
    with pytest.raises(amc.AmcError):
        amc.reset_context(ctx)   # not in replay mode
    a = amc.morph_from_list([1.0, 2.0], (2,))
    amc.realize_ctx(ctx, amc.morph_add(a, a))
    amc.finalize_context(ctx)
    with pytest.raises(amc.AmcError):
        amc.finalize_context(ctx)  # already finalized
    amc.reset_context(ctx)
    with pytest.raises(amc.AmcError):  # a bigger program than the trace
        amc.realize_ctx(ctx, amc.morph_mul(amc.morph_add(a, a), amc.morph_reduce("sum", a)))


def test_plan_graph_capture_replays(amc):
    from amcuda import workloads as W
    xm, ym = W.c1_inputs_morph("f64")
    p = amc.Plan(W.c1_tree(xm, ym))
    p.execute()
    r0 = p.result().values()
    p.capture_graph()
    p.execute()
    _same(p.result().values(), r0)


# ---------------------------------------------------------------------------- BLAS record
def _p(a, t):
    return a.ctypes.data_as(C.POINTER(t))


def test_blas_record_entries_match_oracle(amc):
    from amcuda import _abi as A
    lib = A.load()
    rng = np.random.default_rng(2)
    for dt, ct, pre in ((np.float64, C.c_double, "d"), (np.float32, C.c_float, "s")):
        M, N, K = 33, 29, 47
        Am = rng.standard_normal((M, K)).astype(dt)
        Bm = rng.standard_normal((K, N)).astype(dt)
        Cm = rng.standard_normal((M, N)).astype(dt)
        out = Cm.copy()
        A.check(getattr(lib, f"amc_blas_{pre}gemm")(M, N, K, ct(1.0), _p(Am, ct), _p(Bm, ct), ct(0.0), _p(out, ct)))
        ref = oracle.values(__import__("amcuda").morph_matmul(amc.morph_from_numpy(Am), amc.morph_from_numpy(Bm)))
        _same(out, ref)
        # alpha/beta form against double arithmetic
        out = Cm.copy()
        A.check(getattr(lib, f"amc_blas_{pre}gemm")(M, N, K, ct(0.5), _p(Am, ct), _p(Bm, ct), ct(2.0), _p(out, ct)))
        np.testing.assert_allclose(out, 0.5 * (Am.astype(np.float64) @ Bm) + 2.0 * Cm, rtol=1e-5 if pre == "s" else 1e-12,
                                   atol=1e-5 if pre == "s" else 1e-12)
        # strided: C = A^T B^T with A stored (K, M), B stored (N, K)
        At, Bt = np.ascontiguousarray(Am.T), np.ascontiguousarray(Bm.T)
        out = np.zeros((M, N), dt)
        A.check(getattr(lib, f"amc_blas_{pre}gemm_strided")(M, N, K, ct(1.0), _p(At, ct), M, 1, _p(Bt, ct), K, 1, ct(0.0),
                                                            _p(out, ct)))
        _same(out, ref)
        x = rng.standard_normal(K).astype(dt)
        y = np.zeros(M, dt)
        A.check(getattr(lib, f"amc_blas_{pre}gemv")(M, K, ct(1.0), _p(Am, ct), _p(x, ct), ct(0.0), _p(y, ct)))
        _same(y, oracle.values(amc.morph_matvec(amc.morph_from_numpy(Am), amc.morph_from_numpy(x))))
        r = np.zeros(1, dt)
        A.check(getattr(lib, f"amc_blas_{pre}dot")(K, _p(x, ct), _p(x, ct), _p(r, ct)))
        _same(r[0], oracle.values(amc.morph_dot(amc.morph_from_numpy(x), amc.morph_from_numpy(x))))
        yy = rng.standard_normal(K).astype(dt)
        exp = (np.float64(0.25) * x.astype(np.float64) + yy).astype(dt)
        A.check(getattr(lib, f"amc_blas_{pre}axpy")(K, ct(0.25), _p(x, ct), _p(yy, ct)))
        _same(yy, exp)


# ---------------------------------------------------------------------------- workloads on device tensors
def test_window_fir_entry_point(amc):
    import torch
    from amcuda import workloads as W
    L = 1 << 15
    x = np.stack([W.c2_signal(s, L) for s in range(3)])
    h = W.c2_prototype()
    F = W.c2_frames(L)
    xt, ht = torch.from_numpy(x).cuda(), torch.from_numpy(h).cuda()
    out = torch.empty((3, F, 64), dtype=torch.float32, device="cuda")
    W.window_fir(xt, ht, out)
    torch.cuda.synchronize()
    ref = oracle.realize(W.c2_tree(amc.morph_from_numpy(x), amc.morph_from_numpy(h))).values()
    _same(out.cpu().numpy(), ref)


def test_device_signal_generator_matches_host(amc):
    import torch
    from amcuda import workloads as W
    # identical SplitMix64 bits; the transcendental transform (torch vs numpy
    # libm) may differ in the last place
    dev = W.normal_torch(W.seed_of(5, 0), 4096).cpu().numpy()
    np.testing.assert_allclose(dev, W.normal(W.seed_of(5, 0), 4096), rtol=4e-15, atol=4e-15)
    u = W.uniform_torch(W.seed_of(5, 3), 4096).cpu().numpy()
    _same(u, W.uniform(W.seed_of(5, 3), 4096))
    sig = W.c2_signals_torch(2, 8192).cpu().numpy()
    np.testing.assert_allclose(sig, np.stack([W.c2_signal(s, 8192) for s in range(2)]), rtol=0, atol=2e-6)


@pytest.mark.parametrize("d", [256, 100])
def test_linreg_steps_match_oracle(amc, d):
    import torch
    from amcuda import workloads as W
    n, steps, lr = 4096 + 37, 6, 0.1
    X, y, _ = W.c5_inputs(n, d) if d == 256 else (np.random.default_rng(0).standard_normal((n, d)),
                                                   np.random.default_rng(1).standard_normal(n), None)
    w_ref, losses_ref = oracle.linreg(X, y, np.zeros(d), steps, lr)
    Xt, yt = torch.from_numpy(np.ascontiguousarray(X)).cuda(), torch.from_numpy(np.ascontiguousarray(y)).cuda()
    w = torch.zeros(d, dtype=torch.float64, device="cuda")
    npart = W.linreg_partials_count(n, d)
    part = torch.empty(npart * (d + 1), dtype=torch.float64, device="cuda")
    gl = torch.empty(d + 1, dtype=torch.float64, device="cuda")
    loss = torch.empty(1, dtype=torch.float64, device="cuda")
    losses = []
    for _ in range(steps):
        W.linreg_partials(Xt, yt, w, part, n)
        W.linreg_reduce(part, npart, d, gl)
        W.linreg_update(w, gl, n, lr, loss)
        losses.append(loss.item())
    np.testing.assert_allclose(w.cpu().numpy(), w_ref, rtol=1e-12, atol=1e-14)
    np.testing.assert_allclose(losses, losses_ref, rtol=1e-12)


def _attn_ref(q, k, v, scale):
    s = np.einsum("...id,...jd->...ij", q.astype(np.float64), k.astype(np.float64)) * scale
    p = np.exp(s - s.max(-1, keepdims=True))
    p /= p.sum(-1, keepdims=True)
    return p @ v.astype(np.float64)


@pytest.mark.parametrize("shape", [(2, 3, 128, 64), (1, 2, 96, 64), (2, 1, 256, 32), (1, 2, 384, 64),
                                   (1, 2, 512, 64), (1, 2, 2048, 64)])
def test_attention_entry_points(amc, shape):
    """Forward against the oracle's 3-pass kernel; backward against the
    double-precision VJP.  Tolerance 2e-3 of the output scale (TF32 tensor
    cores where used)."""
    import torch
    from amcuda import workloads as W
    rng = np.random.default_rng(4)
    q, k, v, do = (rng.standard_normal(shape).astype(np.float32) for _ in range(4))
    scale = 1.0 / np.sqrt(shape[-1])
    qt, kt, vt, dot = (torch.from_numpy(a).cuda() for a in (q, k, v, do))
    o = torch.empty_like(qt)
    lse = torch.empty(shape[:-1], dtype=torch.float32, device="cuda")
    W.attention_fwd(qt, kt, vt, o, lse, scale)
    ref = oracle.values(amc.attention_morphism(amc.morph_from_numpy(q), amc.morph_from_numpy(k),
                                               amc.morph_from_numpy(v), scale))
    err = np.max(np.abs(o.cpu().numpy() - ref)) / np.max(np.abs(ref))
    assert err <= 2e-3, err
    dq, dk, dv = torch.empty_like(qt), torch.empty_like(kt), torch.empty_like(vt)
    W.attention_bwd(qt, kt, vt, o, dot, lse, dq, dk, dv, scale)
    rq, rk, rv = oracle.attention_bwd(q, k, v, do, scale)
    for got, r in ((dq, rq), (dk, rk), (dv, rv)):
        e = np.max(np.abs(got.cpu().numpy() - r)) / np.max(np.abs(r))
        assert e <= 2e-3, e
    # no atomics anywhere: a second run gives the same bits
    dq2, dk2, dv2 = torch.empty_like(qt), torch.empty_like(kt), torch.empty_like(vt)
    W.attention_bwd(qt, kt, vt, o, dot, lse, dq2, dk2, dv2, scale)
    for a, b in ((dq, dq2), (dk, dk2), (dv, dv2)):
        assert torch.equal(a, b)


@pytest.mark.parametrize("N,Cc,H,Wd,K", [(2, 4, 9, 7, 5), (3, 64, 14, 14, 64), (2, 64, 56, 56, 64), (1, 64, 8, 60, 64), (1, 64, 6, 64, 64)])
def test_conv_entry_points(amc, N, Cc, H, Wd, K):
    import torch
    from amcuda import workloads as W
    rng = np.random.default_rng(6)
    x = rng.standard_normal((N, Cc, H, Wd)).astype(np.float32)
    w = (rng.standard_normal((K, Cc, 3, 3)) * np.sqrt(2.0 / (Cc * 9))).astype(np.float32)
    dy = rng.standard_normal((N, K, H, Wd)).astype(np.float32)
    xt, wt, dyt = (torch.from_numpy(a).cuda() for a in (x, w, dy))
    y = torch.empty((N, K, H, Wd), dtype=torch.float32, device="cuda")
    W.conv2d_fwd(xt, wt, y)
    ref = oracle.conv2d_fwd(x, w)
    e = np.max(np.abs(y.cpu().numpy() - ref)) / np.max(np.abs(ref))
    assert e <= 2e-3, e
    dx = torch.empty_like(xt)
    W.conv2d_dgrad(dyt, wt, dx)
    rdx = oracle.conv2d_dgrad(dy, w, x.shape)
    e = np.max(np.abs(dx.cpu().numpy() - rdx)) / np.max(np.abs(rdx))
    assert e <= 2e-3, e
    dw = torch.empty_like(wt)
    W.conv2d_wgrad(xt, dyt, dw)
    rdw = oracle.conv2d_wgrad(x, dy, w.shape)
    e = np.max(np.abs(dw.cpu().numpy() - rdw)) / np.max(np.abs(rdw))
    assert e <= 2e-3, e


def test_tc_peak_probe(amc):
    """The tcgen05 TF32 throughput probe returns a plausible dense rate (the
    nominal dense TF32 figure of a B200 is about 1.1 PFLOP/s)."""
    from amcuda import workloads as W
    v = W.tc_peak_tf32(2000)
    assert 300.0 < v < 3000.0, v
    # the same products with A read from tensor memory
    v = W.tc_peak_tf32(2000, 64, 2, a_tmem=True)
    assert 300.0 < v < 3000.0, v
