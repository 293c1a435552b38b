"""The oracle against the known answers transcribed from the reference's
own tests (tests/golden/known_answers.json); CPU only."""
import json
from pathlib import Path

import numpy as np
import pytest

import oracle
from golden_dsl import build

CASES = json.loads((Path(__file__).parent / "golden" / "known_answers.json").read_text())["cases"]


def check(res, c):
    if c["shape"] is not None:
        assert list(res.shape) == c["shape"], c["name"]
    if c["dtype"] is not None:
        assert res.dtype == c["dtype"], c["name"]
    if c["values"] is not None:
        got = np.asarray(res.values(), dtype=np.float64).reshape(-1)
        exp = np.asarray(c["values"], dtype=np.float64).reshape(-1)
        assert got.shape == exp.shape, c["name"]
        np.testing.assert_allclose(got, exp, rtol=0, atol=c["tol"] if c["tol"] else 0, err_msg=c["name"])


@pytest.mark.parametrize("c", CASES, ids=[c["name"] for c in CASES])
def test_oracle_known_answer(c):
    check(oracle.realize(build(c["expr"])), c)


def test_colour_reference_examples():
    # example-06-buffer-reuse.scm: a2, b2, a2+b2, *half, sqrt -> 5 allocations, 3 buffers
    asg, nb = oracle.colour([1] * 5, [4] * 5, [[], [], [0, 1], [2], [3]])
    assert nb == 3 and asg == [0, 1, 2, 0, 2]
    # test-context.scm:207-220: linear chain of 4 ops -> at most 2 buffers
    _, nb = oracle.colour([1] * 4, [8] * 4, [[], [0], [1], [2]])
    assert nb == 2
    # test-context.scm:420-435: pinning alloc 0 of a 2-chain -> 2 buffers
    _, nb = oracle.colour([1] * 2, [8] * 2, [[], []], pinned=[1, 0])
    assert nb == 2
    _, nb = oracle.colour([1] * 2, [8] * 2, [[], []])
    assert nb == 1
