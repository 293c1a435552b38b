"""C-ABI checks that need no GPU: the library loads, exports every entry
point include/amc.h declares, its context colouring matches the oracle, and
host-side fault injection fails before touching the device."""
import ctypes as C
import os
import random
import re
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
HEADER = ROOT / "include" / "amc.h"


def declared():
    src = HEADER.read_text()
    return sorted(set(re.findall(r"^int\s+(amc_\w+)\s*\(", src, flags=re.M)))


def test_library_exports_every_declared_symbol():
    from amcuda import _abi
    lib = _abi.load()
    names = declared()
    assert len(names) >= 40
    missing = [n for n in names if not hasattr(lib, n)]
    assert not missing, missing
    # and the ctypes binding covers them all
    assert set(names) <= set(_abi.SIGNATURES), set(names) - set(_abi.SIGNATURES)


def test_colour_matches_oracle_on_random_traces():
    import oracle
    from amcuda.context import colour
    rng = random.Random(7)
    for trial in range(200):
        n = rng.randint(0, 24)
        dtypes = [rng.choice([0, 1, 2]) for _ in range(n)]
        sizes = [rng.choice([4, 8, 16, 32, 64]) for _ in range(n)]
        inputs = [sorted(rng.sample(range(i), rng.randint(0, min(i, 3)))) if i else [] for i in range(n)]
        pinned = [1 if rng.random() < 0.1 else 0 for _ in range(n)]
        assert colour(dtypes, sizes, inputs, pinned) == oracle.colour(dtypes, sizes, inputs, pinned), trial


def test_colour_reference_example_06():
    from amcuda.context import colour
    asg, nb = colour([1] * 5, [4] * 5, [[], [], [0, 1], [2], [3]])
    assert nb == 3 and asg == [0, 1, 2, 0, 2]


def test_injected_allocation_failure_is_reported_before_device_work():
    code = r"""
import sys, ctypes as C
sys.path.insert(0, %r)
from amcuda import _abi as A
h = C.c_uint64()
rc = A.load().amc_buf_create(1, 16, C.byref(h))
print(rc, A.last_error())
""" % str(ROOT / "array-morphisms_b200")
    env = dict(os.environ, AMC_FAULT="alloc")
    out = subprocess.run([sys.executable, "-c", code], env=env, capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    rc, msg = out.stdout.strip().split(" ", 1)
    assert int(rc) == 6 and "AMC_FAULT=alloc" in msg


def test_invalid_arguments_rejected_without_device():
    from amcuda import _abi as A
    lib = A.load()
    h = C.c_uint64()
    assert lib.amc_buf_create(99, 4, C.byref(h)) == 1  # invalid dtype
    assert lib.amc_plan_execute(123456, None) == 1     # unknown plan
    assert lib.amc_ctx_finalize(98765) == 1            # unknown context
    assert "unknown" in A.last_error()
