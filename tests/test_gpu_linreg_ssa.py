"""Config 5 through the public SSA path on the device.

The linear-regression MSE program built from variables (grad.scm's var-*),
compiled by morphism_to_ssa / ssa_vjp, trained by ssa_realize_ctx with
buffer reuse (trace, finalize, compiled replay) and an in-place gradient
step per replay (workloads.LinregSSA).  The planner runs the program's
forward and gradient GEMVs as one pass over X.  Checked against the
oracle's restatement of the same steps (oracle.linreg: the GEMV, residual,
mean and strided GEMM of the SSA replay in the reference's sequential
order): weights and the loss of every step to 1e-12.  Replays allocate no
device memory."""
import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("rows,d,steps", [(1 << 16, 256, 6), (50_000, 100, 5)])
def test_linreg_ssa_replay_matches_the_oracle(amc, rows, d, steps):
    import torch
    from amcuda import workloads as W
    lr = 0.1
    X, y, _ = W.c5_inputs(rows, d)
    w0 = np.zeros(d)
    t = W.LinregSSA(X, y, w0, lr)
    t.trace()
    assert t.trace_stats["mode"] == "trace" and t.trace_stats["allocations"] > 0
    t.step()                       # first replay: compiles the plan, plans the update
    torch.cuda.synchronize()
    free0 = torch.cuda.mem_get_info()[0]
    for _ in range(steps - 2):
        t.step()
    torch.cuda.synchronize()
    assert torch.cuda.mem_get_info()[0] == free0, "a replayed step allocated device memory"
    w_ref, losses_ref = oracle.linreg(X, y, w0, steps, lr)
    np.testing.assert_allclose(t.weights(), w_ref, rtol=1e-12, atol=1e-15)
    np.testing.assert_allclose(t.losses(), losses_ref, rtol=1e-12)
    assert t.losses()[-1] < t.losses()[0]


def test_linreg_ssa_small_keeps_the_reference_order(amc):
    """Below the row-pass sizes the same program runs on k_gemm, in the
    reference's order: weights and losses equal the oracle bit for bit."""
    from amcuda import workloads as W
    rows, d, steps, lr = 256, 8, 4, 0.1
    X, y, _ = W.c5_inputs(rows, d)
    t = W.LinregSSA(X, y, np.zeros(d), lr)
    t.trace()
    for _ in range(steps - 1):
        t.step()
    w_ref, losses_ref = oracle.linreg(X, y, np.zeros(d), steps, lr)
    np.testing.assert_allclose(t.weights(), w_ref, rtol=1e-13, atol=1e-16)
    np.testing.assert_allclose(t.losses(), losses_ref, rtol=1e-13)
