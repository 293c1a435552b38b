"""amc_linreg_step_noalloc: the linear-regression step for callers that
cannot allocate device memory (their device memory belongs to another
allocator, or cudaMalloc may not run in their timed loop).  Its scratch is a
static device array inside the library.  Checked through the C ABI against
the allocating entry point, amc_linreg_step, on two consecutive steps.

Collected last on purpose: a failure here leaves every other test already run.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

TOL = 1e-12  # f64 parity tolerance used by the linear-regression tests


def _p(t):
    return C.c_void_p(t.data_ptr())


def test_noalloc_linreg_step_matches_allocating_step(amc):
    import torch
    from amcuda import _abi as A
    from amcuda import workloads as W
    lib = A.load()
    n, d, lr = 50_000, 256, 0.1
    X, y, _ = W.c5_inputs(n, d)
    Xt = torch.from_numpy(np.ascontiguousarray(X)).cuda()
    yt = torch.from_numpy(np.ascontiguousarray(y)).cuda()
    w_ref = torch.zeros(d, dtype=torch.float64, device="cuda")
    w_na = torch.zeros(d, dtype=torch.float64, device="cuda")
    npart = W.linreg_partials_count(n, d)
    part = torch.empty(npart * (d + 1), dtype=torch.float64, device="cuda")
    gl = torch.empty(d + 1, dtype=torch.float64, device="cuda")
    loss_ref = torch.empty(1, dtype=torch.float64, device="cuda")
    loss_na = torch.empty(1, dtype=torch.float64, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for step in range(2):
        A.check(lib.amc_linreg_step(_p(Xt), _p(yt), _p(w_ref), n, d, C.c_double(lr), _p(part), _p(gl), _p(loss_ref),
                                    stream))
        A.check(lib.amc_linreg_step_noalloc(_p(Xt), _p(yt), _p(w_na), n, d, C.c_double(lr), _p(loss_na), stream))
        torch.cuda.synchronize()
        np.testing.assert_allclose(w_na.cpu().numpy(), w_ref.cpu().numpy(), rtol=TOL, atol=TOL)
        np.testing.assert_allclose(loss_na.item(), loss_ref.item(), rtol=TOL)


def test_noalloc_rejects_sizes_beyond_its_scratch(amc):
    import torch
    from amcuda import _abi as A
    lib = A.load()
    d = 1024  # (partials + 1) * 1025 doubles exceeds the static 262144
    X = torch.zeros((1 << 16, d), dtype=torch.float64, device="cuda")
    y = torch.zeros(1 << 16, dtype=torch.float64, device="cuda")
    w = torch.zeros(d, dtype=torch.float64, device="cuda")
    rc = lib.amc_linreg_step_noalloc(_p(X), _p(y), _p(w), 1 << 16, d, C.c_double(0.1), None, None)
    assert rc == 1  # AMC_ERR_INVALID
    assert "static scratch" in A.last_error()
