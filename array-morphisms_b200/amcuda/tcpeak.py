"""Print the tcgen05 kind::tf32 issue-rate table of this GPU.

    python -m amcuda.tcpeak        (with array-morphisms_b200 on sys.path)

Each row: M=128 x N x K=8 products issued back to back from shared-memory
operands by 1, 2 or 4 threads per SM (amc_tc_peak_tf32).  The N=256 row is
the dense TF32 peak; the smaller N rows show the per-instruction issue floor
that the attention and convolution tiles (N=64) run against."""
from __future__ import annotations


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
    print("| N | issuing threads/SM | TFLOP/s | SM clocks per MMA |")
    print("|---|---|---|---|")
    for n in (32, 64, 128, 256):
        for w in (1, 2, 4):
            if n * w > 512:
                continue
            tf = W.tc_peak_tf32(4000, n, w)
            per = ""
            if clk_ghz:
                per = f"{2 * 128 * n * 8 * sms * clk_ghz * 1e9 / (tf * 1e12):.1f}"
            print(f"| {n} | {w} | {tf:.1f} | {per} |")
    if clk_ghz:
        print(f"\nSM clock sampled after the sweep: {clk_ghz * 1000:.0f} MHz, {sms} SMs")


if __name__ == "__main__":
    main()
