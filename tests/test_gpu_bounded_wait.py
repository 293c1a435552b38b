"""The bounded device wait's failure path, made to run out on purpose.

Every TMA/tensor-core kernel waits on mbarriers with a poll limit and, on
expiry, records AMC_ERR_TIMEOUT and returns instead of spinning.  Here the
same wait runs alone on a one-thread launch whose barrier nothing arrives
on (amc_probe_bounded_wait with arrive = 0): the launch must return, the
entry must report the timeout, and the next calls on the same stream must
succeed.  No fault, trap or hang is involved: the wait gives up after a
short, fixed number of polls."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_the_context_stays_usable(amc):
    from amcuda import _abi as A
    lib = A.load()
    assert lib.amc_probe_bounded_wait(1000, 1, None) == 0          # completes: one arrival
    rc = lib.amc_probe_bounded_wait(1000, 0, None)                # nothing arrives
    assert rc == 7, A.last_error()                                 # AMC_ERR_TIMEOUT
    assert "gave up" in A.last_error()
    assert lib.amc_probe_bounded_wait(1, 0, None) == 7             # the smallest limit as well
    assert lib.amc_probe_bounded_wait(1000, 1, None) == 0          # flag cleared, stream usable
    # an ordinary realize on the same context afterwards
    x = np.arange(12, dtype=np.float64).reshape(3, 4)
    got = amc.realize(amc.morph_add(amc.morph_from_numpy(x), amc.morph_from_numpy(x))).values()
    np.testing.assert_array_equal(got, 2 * x)
    assert lib.amc_synchronize() == 0


def test_bounded_wait_rejects_bad_arguments(amc):
    from amcuda import _abi as A
    lib = A.load()
    assert lib.amc_probe_bounded_wait(0, 1, None) == 1
    assert lib.amc_probe_bounded_wait(1 << 23, 1, None) == 1
    assert lib.amc_probe_bounded_wait(10, 2, None) == 1
