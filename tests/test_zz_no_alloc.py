"""amc_linreg_step_noalloc: the linear-regression step for callers that
cannot allocate device memory (their device memory belongs to another
allocator, or cudaMalloc may not run in their timed loop).  Its scratch is a
static device array inside the library.  Checked through the C ABI against
the allocating entry point, amc_linreg_step, on two consecutive steps: the
two run the same kernels in the same order, so the results are identical
bit for bit.  The cases cover the templated d = 256 kernel, the generic
kernel at other widths, a width that brings the scratch need to just below
the static array's 262144 doubles, and a width whose generic kernel needs
more than 48 KiB of dynamic shared memory.

Collected last on purpose: a failure here leaves every other test already run.
"""
import ctypes as C

import numpy as np
import pytest

pytestmark = pytest.mark.gpu

SCRATCH_DOUBLES = 262144   # the static scratch: (partials + 1) * (d + 1) must fit


def _p(t):
    return C.c_void_p(t.data_ptr())


def _widest(rows):
    """The largest d whose scratch need fits the static array at `rows`."""
    from amcuda import workloads as W
    return SCRATCH_DOUBLES // (W.linreg_partials_count(rows, 1) + 1) - 1


@pytest.mark.parametrize("rows,d", [(50_000, 256), (30_000, 100), (1 << 16, None), (10_000, 800)])
def test_noalloc_linreg_step_matches_allocating_step(amc, rows, d):
    import torch
    from amcuda import _abi as A
    from amcuda import workloads as W
    lib = A.load()
    d = d or _widest(rows)
    npart = W.linreg_partials_count(rows, d)
    assert (npart + 1) * (d + 1) <= SCRATCH_DOUBLES
    lr = 0.1
    X, y, _ = W.c5_inputs(rows, d)
    Xt = torch.from_numpy(np.ascontiguousarray(X)).cuda()
    yt = torch.from_numpy(np.ascontiguousarray(y)).cuda()
    w_ref = torch.zeros(d, dtype=torch.float64, device="cuda")
    w_na = torch.zeros(d, dtype=torch.float64, device="cuda")
    part = torch.empty(npart * (d + 1), dtype=torch.float64, device="cuda")
    gl = torch.empty(d + 1, dtype=torch.float64, device="cuda")
    loss_ref = torch.empty(1, dtype=torch.float64, device="cuda")
    loss_na = torch.empty(1, dtype=torch.float64, device="cuda")
    stream = C.c_void_p(torch.cuda.current_stream().cuda_stream)
    for step in range(2):
        A.check(lib.amc_linreg_step(_p(Xt), _p(yt), _p(w_ref), rows, d, C.c_double(lr), _p(part), _p(gl),
                                    _p(loss_ref), stream))
        A.check(lib.amc_linreg_step_noalloc(_p(Xt), _p(yt), _p(w_na), rows, d, C.c_double(lr), _p(loss_na), stream))
        torch.cuda.synchronize()
        np.testing.assert_array_equal(w_na.cpu().numpy(), w_ref.cpu().numpy())
        assert loss_na.item() == loss_ref.item()
        assert np.isfinite(loss_na.item()) and np.any(w_na.cpu().numpy() != 0.0)


def test_noalloc_rejects_sizes_beyond_its_scratch(amc):
    import torch
    from amcuda import _abi as A
    lib = A.load()
    rows = 1 << 16
    d = _widest(rows) + 1   # one column past the static scratch
    X = torch.zeros((rows, d), dtype=torch.float64, device="cuda")
    y = torch.zeros(rows, dtype=torch.float64, device="cuda")
    w = torch.zeros(d, dtype=torch.float64, device="cuda")
    rc = lib.amc_linreg_step_noalloc(_p(X), _p(y), _p(w), rows, d, C.c_double(0.1), None, None)
    assert rc == 1  # AMC_ERR_INVALID
    assert "static scratch" in A.last_error()
