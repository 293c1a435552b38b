"""Large matrix-vector products: the row-pass kernels (amc_rowpass.cu).

At these sizes the planner and the BLAS record leave k_gemm's sequential
order (one CTA per 64x64 output tile would run a GEMV on a handful of CTAs)
for warp-per-row passes with a fixed parallel order: the forward GEMV over a
row-major matrix, the transposed GEMV X^T v, the dot product, and the GEMV
pair of a linear model's SSA program (X w and X^T e(X w) in one read of X).
The reference accumulates each output sequentially in double
(blas-exec.scm:405-458); these results agree with that order to the stated
tolerance: f64 within 1e-12 and f32 within 1e-6 of the largest output
(norm-wise: an individual output may cancel to near zero)."""
import ctypes as C

import numpy as np
import pytest

import amcuda as am
from amcuda import ssa as S
import oracle

pytestmark = pytest.mark.gpu

TOL = {"f64": 1e-12, "f32": 1e-6}


def _close(got, ref, dt):
    got, ref = np.asarray(got, dtype=np.float64), np.asarray(ref, dtype=np.float64)
    assert got.shape == ref.shape
    scale = max(np.max(np.abs(ref)), 1e-300)
    err = np.max(np.abs(got - ref)) / scale
    assert err <= TOL[dt], f"max error {err:.3e} of the output scale (tolerance {TOL[dt]})"


def _rng_mat(seed, shape, dt):
    a = np.random.default_rng(seed).standard_normal(shape)
    return a.astype(np.float32) if dt == "f32" else a


@pytest.mark.parametrize("dt", ["f64", "f32"])
@pytest.mark.parametrize("rows,d", [(1 << 14, 256), (1 << 15, 64), (1 << 14, 100), (1 << 13, 1000)])
def test_gemv_forward_rows(amc, dt, rows, d):
    X, v = _rng_mat(1, (rows, d), dt), _rng_mat(2, (d,), dt)
    got = am.realize(am.morph_matvec(am.morph_from_numpy(X, dt), am.morph_from_numpy(v, dt))).values()
    _close(got, X.astype(np.float64) @ v.astype(np.float64), dt)
    got = am.realize(am.morph_matmul(am.morph_from_numpy(X, dt), am.morph_from_numpy(v.reshape(d, 1), dt))).values()
    _close(got, (X.astype(np.float64) @ v.astype(np.float64)).reshape(rows, 1), dt)


@pytest.mark.parametrize("dt", ["f64", "f32"])
@pytest.mark.parametrize("rows,d", [(1 << 16, 256), (1 << 15, 32), (1 << 14, 1000), (100_003, 7)])
def test_gemv_transposed(amc, dt, rows, d):
    X, g = _rng_mat(3, (rows, d), dt), _rng_mat(4, (rows,), dt)
    Xm = am.morph_from_numpy(X, dt)
    ref = X.astype(np.float64).T @ g.astype(np.float64)
    got = am.realize(am.morph_matvec(am.morph_transpose(Xm, (1, 0)), am.morph_from_numpy(g, dt))).values()
    _close(got, ref, dt)
    got = am.realize(am.morph_matmul(am.morph_transpose(Xm, (1, 0)), am.morph_from_numpy(g.reshape(rows, 1), dt))).values()
    _close(got, ref.reshape(d, 1), dt)


@pytest.mark.parametrize("dt", ["f64", "f32"])
@pytest.mark.parametrize("n", [1 << 16, 1 << 20, 3_000_017])
def test_dot_long(amc, dt, n):
    x, y = _rng_mat(5, (n,), dt), _rng_mat(6, (n,), dt)
    got = am.realize(am.morph_dot(am.morph_from_numpy(x, dt), am.morph_from_numpy(y, dt))).values()
    xy = x.astype(np.float64) * y.astype(np.float64)
    # a dot product can cancel: the bound is relative to the sum of |x_k y_k|
    assert abs(float(got) - float(np.sum(xy))) <= TOL[dt] * float(np.sum(np.abs(xy)))


def test_dot_strided_views(amc):
    """A dot of two strided views (every other element, a reversed slice
    is not constructible, so a column of a matrix)."""
    M = _rng_mat(7, (1 << 18, 4), "f64")
    Mm = am.morph_from_numpy(M)
    a = am.morph_reshape(am.morph_slice(Mm, (0, 1), (1 << 18, 2), (1, 1)), (1 << 18,))
    b = am.morph_reshape(am.morph_slice(Mm, (0, 3), (1 << 18, 4), (1, 1)), (1 << 18,))
    got = float(am.realize(am.morph_dot(a, b)).values())
    ref = float(np.dot(M[:, 1], M[:, 3]))
    assert abs(got - ref) <= 1e-12 * np.sum(np.abs(M[:, 1] * M[:, 3]))


def test_blas_record_large_gemv_and_dot(amc):
    """The BLAS record entries (make-blas-backend slots, blas-exec.scm:16-46)
    at large sizes, with alpha and beta."""
    from amcuda import _abi as A
    lib = A.load()
    M, N = 1 << 14, 256
    Am = _rng_mat(8, (M, N), "f64")
    x, y0 = _rng_mat(9, (N,), "f64"), _rng_mat(10, (M,), "f64")
    y = y0.copy()
    P = lambda a: a.ctypes.data_as(C.POINTER(C.c_double))
    A.check(lib.amc_blas_dgemv(M, N, 0.5, P(Am), P(x), -2.0, P(y)))
    _close(y, 0.5 * (Am @ x) - 2.0 * y0, "f64")
    n = 1 << 20
    u, v = _rng_mat(11, (n,), "f64"), _rng_mat(12, (n,), "f64")
    out = np.zeros(1)
    A.check(lib.amc_blas_ddot(n, P(u), P(v), P(out)))
    assert abs(out[0] - np.dot(u, v)) <= 1e-12 * np.sum(np.abs(u * v))
    # transposed GEMM with N = 1 through the strided entry: C = A^T b
    K = 1 << 16
    Xs, b = _rng_mat(13, (K, 64), "f64"), _rng_mat(14, (K, 1), "f64")
    Cm = np.zeros((64, 1))
    A.check(lib.amc_blas_dgemm_strided(64, 1, K, 1.0, P(Xs), 64, 1, P(b), 1, 0, 0.0, P(Cm)))
    _close(Cm, Xs.T @ b, "f64")


def test_small_products_keep_the_reference_order(amc):
    """Below the row-pass sizes the products stay on k_gemm and equal the
    oracle's sequential order bit for bit."""
    X, v = _rng_mat(15, (512, 64), "f64"), _rng_mat(16, (64,), "f64")
    t = am.morph_matvec(am.morph_from_numpy(X), am.morph_from_numpy(v))
    np.testing.assert_array_equal(am.realize(t).values(), oracle.values(t))
    t = am.morph_matvec(am.morph_transpose(am.morph_from_numpy(X), (1, 0)), am.morph_from_numpy(X[:, 0].copy()))
    np.testing.assert_array_equal(am.realize(t).values(), oracle.values(t))


# ------------------------------------------------------------------ the GEMV pair (one read of X)

def _joint(loss, params):
    fwd = S.morphism_to_ssa(loss)
    pv = [S.ssa_constant_id(fwd, am.var_value(p)) for p in params]
    return S.ssa_vjp(fwd, pv, S.ssa_loss_binding_val(fwd))


def _plan_launches(joint):
    from amcuda.realize import Plan
    trees = [t for t in S._output_trees(joint) if not isinstance(t, am.Concrete)]
    return Plan(trees).stats()["launches"]


@pytest.mark.parametrize("d", [256, 128, 100])
def test_mse_program_runs_as_one_pass(amc, d):
    """The linear-regression MSE program's loss and gradient on the device
    (the forward and gradient GEMVs fused into one pass over X) against the
    same program realized by the oracle, f64 within 1e-12."""
    from amcuda import workloads as W
    rows = 1 << 15
    X, y, _ = W.c5_inputs(rows, d)
    w = np.random.default_rng(17).standard_normal((d, 1)) * 0.1
    Xv, yv = am.make_var(am.morph_from_numpy(X)), am.make_var(am.morph_from_numpy(y.reshape(rows, 1)))
    wv = am.make_var(am.morph_from_numpy(w), True)
    r = am.var_sub(am.var_matmul(Xv, wv), yv)
    joint = _joint(am.var_mean(am.var_mul(r, r)), [wv])
    got = S.ssa_realize(joint)
    ref = S.ssa_realize(joint, oracle.realize)
    for g, rr in zip(got, ref):
        _close(g.values(), rr.values(), "f64")
    # d a multiple of 32 up to 256 (the TMA-fed pair): 5 launches.  The pair
    # (row pass + partial sum) computes X w, the gradient and the loss's sum
    # of squared residuals in one read of X; then the loss's sum of the
    # per-CTA partials, the 1/N constant and the add of 0.  Other d: the
    # generic pair leaves the loss to its own two-level reduction (6).
    # Unfused, X w, the row program's map, X^T e and the loss's reduction
    # would take 5 to 6 launches in place of the pair's 2 and 1.
    assert _plan_launches(joint) == (5 if d in (32, 64, 128, 256) else 6)


def test_gemv_pair_with_a_nonlinear_row_program(amc):
    """A row program beyond the MSE's: loss = mean(tanh(X w) * y), whose
    gradient is X^T (g * y * (1 - tanh^2)) computed in the same pass."""
    rows, d = 1 << 15, 64
    rng = np.random.default_rng(18)
    X, y = rng.standard_normal((rows, d)), rng.standard_normal((rows, 1))
    wv = am.make_var(am.morph_from_numpy(rng.standard_normal((d, 1)) * 0.05), True)
    t = am.var_tanh(am.var_matmul(am.make_var(am.morph_from_numpy(X)), wv))
    joint = _joint(am.var_mean(am.var_mul(t, am.make_var(am.morph_from_numpy(y)))), [wv])
    for g, rr in zip(S.ssa_realize(joint), S.ssa_realize(joint, oracle.realize)):
        _close(g.values(), rr.values(), "f64")
