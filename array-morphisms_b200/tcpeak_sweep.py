"""Print the tcgen05 kind::tf32 issue-rate table of this GPU.

    python array-morphisms_b200/tcpeak_sweep.py

A measurement script beside the package, not part of it: bench.py takes its
TF32 denominator from the same probe entry point directly.

Each row: M=128 x N x K=8 products issued back to back by 1, 2 or 4 threads
per SM (amc_tc_peak_tf32), B read from shared memory and A from shared memory
("smem") or tensor memory ("tmem").  The N=256 row is the dense TF32 peak.
The last column is the shared-memory operand bytes per product over the
clocks it took: at about 128 B/clock the product is bound by the
shared-memory read port, not by the pipe."""
from __future__ import annotations

import sys
from pathlib import Path

sys.path.insert(0, str(Path(__file__).resolve().parent))


def main() -> None:
    import amcuda as am
    from amcuda import workloads as W
    am.init(0)
    clk_ghz = None
    try:
        import pynvml
        pynvml.nvmlInit()
        h = pynvml.nvmlDeviceGetHandleByIndex(0)
        clk_ghz = pynvml.nvmlDeviceGetClockInfo(h, pynvml.NVML_CLOCK_SM) / 1000.0
    except Exception:
        pass
    import torch
    sms = torch.cuda.get_device_properties(0).multi_processor_count
    print("| A from | N | issuing threads/SM | TFLOP/s | SM clocks per MMA | shared-memory B/clock |")
    print("|---|---|---|---|---|---|")
    for a_tmem in (False, True):
        for n in (32, 64, 128, 256):
            for w in (1, 2, 4):
                if n * w > (480 if a_tmem else 512):
                    continue
                tf = W.tc_peak_tf32(4000, n, w, a_tmem)
                per = bw = ""
                if clk_ghz:
                    clocks = 2 * 128 * n * 8 * sms * clk_ghz * 1e9 / (tf * 1e12)
                    smem_bytes = n * 32 + (0 if a_tmem else 128 * 32)
                    per, bw = f"{clocks:.1f}", f"{smem_bytes / clocks:.0f}"
                print(f"| {'tmem' if a_tmem else 'smem'} | {n} | {w} | {tf:.1f} | {per} | {bw} |")
    if clk_ghz:
        print(f"\nSM clock sampled after the sweep: {clk_ghz * 1000:.0f} MHz, {sms} SMs")


if __name__ == "__main__":
    main()
