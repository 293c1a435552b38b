"""bench.py's reference arm runs on the host alone (the oracle port of the
reference's CPU path on every core): its JSON line carries the contract's
keys for the default and a non-default workload.  CPU only."""
import json
import subprocess
import sys
from pathlib import Path

import pytest

ROOT = Path(__file__).resolve().parents[1]
KEYS = {"impl", "metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step", "higher_is_better", "scaling",
        "vs_baseline", "dtype", "data", "config", "cpu_baseline", "e2e"}


@pytest.mark.parametrize("workload", ["fused", "linreg"])
def test_reference_arm_line(workload):
    out = subprocess.run([sys.executable, "bench.py", "--impl", "reference", "--workload", workload, "--steps", "1",
                          "--warmup", "1", "--ref-procs", "2"], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    line = json.loads(out.stdout.strip().splitlines()[-1])
    assert KEYS <= set(line) and line["impl"] == "reference" and line["value"] > 0
    assert line["cpu_baseline"]["kind"] == "port" and line["cpu_baseline"]["cores"] == 2
    assert line["e2e"]["h2d_bytes_per_step"] == 0 and line["e2e"]["value"] == line["value"]
    assert line["unit"] == "GB/s" and line["config"]["workload"].startswith("config")


@pytest.mark.parametrize("job", ["filterbank", "fused", "linreg"])
def test_reference_arm_processes_map_no_product_library(job):
    """The reference arm's processes build the workload trees and run the
    oracle: no library of the product (libamcuda.so) may be mapped in them,
    only the oracle's."""
    call = ("bench._oracle_filterbank_sample((0, 1 << 14))" if job == "filterbank"
            else f"bench._oracle_other_sample(({job!r}, 'f64'))")
    code = ("import sys; sys.path.insert(0, '.'); import bench; " + call + "; "
            "maps = open('/proc/self/maps').read(); "
            "print('amcuda' if 'libamcuda' in maps else 'clean', 'oracle' if 'liboracle' in maps else 'no-oracle')")
    out = subprocess.run([sys.executable, "-c", code], cwd=ROOT, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    assert out.stdout.split() == ["clean", "oracle"]
