"""Benchmark of the realize hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl amcuda|reference]
                    [--workload all|filterbank|fused|linreg|attention|conv]

Default (`all`): ONE JSON line whose headline is the polyphase filter bank
(config 2 of the five) realized through the public API: 64 signals of 2^24
f32 samples per GPU, 64 branches x 16 taps, the im2col -> reshape ->
transpose -> product -> tap-sum tree; one step = one realize of that tree on
device-resident inputs.  `value` is algorithmic HBM GB/s of the whole job;
`e2e` is the same metric with the host->device upload of every step's
signals from pinned memory and the device->host read of its result inside
the timed region.

The same line carries `per_config`: the other configs, each with its own
value, step time, roofline, CPU baseline, e2e and clocks:
  fused_f64, fused_s32  config 1 (view + map + reduce tree, realize)
  conv                  config 3 (Y, dX, dW through the conv entry points)
  attention             config 4 (O, dQ, dK, dV through the attention entries)
  linreg                config 5 (the MSE program through morphism-to-ssa,
                        ssa-vjp and ssa-realize/ctx replay, 2^22 x 256 f64)
`--workload X` prints the line of config X alone.

Multi-GPU runs one process per GPU (torchrun); per-GPU work is fixed (weak
scaling): signals, conv images, attention batch entries and regression rows
are sharded, config 1 runs as replicas.  The conv weight gradient and the
regression gradient cross the shards and are summed over ranks in a fixed
order.  Time is the max over ranks of CUDA-event time.
"""
from __future__ import annotations

import argparse
import gc
import json
import math
import multiprocessing as mp
import os
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "array-morphisms_b200"))

HBM_FALLBACK = 6650.0

# DRAM bytes per launch of the dominant kernel from one ncu capture
# (dram__bytes_read.sum + dram__bytes_write.sum, one pass, the full-size
# workload of the named bench command), with what was captured.  Absent
# where no capture of the current kernel exists.
_NCU = "ncu --metrics dram__bytes_read.sum,dram__bytes_write.sum --clock-control none -k regex:{k} -s {s} -c 1 "
_BENCH = "python bench.py --workload {w} --no-e2e --no-cpu --steps 2 --warmup 3"
NCU_TRAFFIC: dict = {
    "filterbank": {"bytes_per_launch": 4.54e9 + 4.23e9,
                   "source": _NCU.format(k="k_fir_tma", s=3) + _BENCH.format(w="filterbank") + " --no-per-config"
                             + ": k_fir_tma, 64 x 2^24 samples, read 4.54 GB + write 4.23 GB"},
    "fused_f64": {"bytes_per_launch": 8.424e6,
                  "source": "ncu --set full --clock-control none -k regex:k_colfold -s 3 -c 1 python bench.py "
                            "--workload fused --dtype f64 --no-e2e --no-cpu --no-cold --steps 20 --warmup 3: "
                            "k_colfold, read 8.42 MB + write 0 (the 8 KB result stays in L2)"},
    "conv": {"bytes_per_launch": 51.61e6 + 4.77e6,
             "source": _NCU.format(k="k_conv3x3_tc", s=4) + _BENCH.format(w="conv")
                       + ": k_conv3x3_tc (forward), read 51.61 MB + write 4.77 MB (most of Y stays in L2)"},
    "attention": {"bytes_per_launch": 541.16e6 + 238.75e6,
                  "source": _NCU.format(k="k_attn_bwd_dkv_tc", s=3) + _BENCH.format(w="attention")
                            + ": k_attn_bwd_dkv_tc (the largest share of the step), read 541.16 MB + write 238.75 MB"},
    "linreg": {"bytes_per_launch": 8.66e9 + 13.95e6,
               "source": _NCU.format(k="k_gemv_pair_tma", s=3) + _BENCH.format(w="linreg")
                         + ": k_gemv_pair_tma, X 2^22 x 256 f64, read 8.66 GB + write 13.95 MB"},
}


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d.get("hbm_gbs", HBM_FALLBACK)), float(d.get("bf16_tflops", 1590.0)), "measured"
    return HBM_FALLBACK, 1590.0, "fallback"


def traffic_of(name: str):
    t = NCU_TRAFFIC.get(name)
    return (t["bytes_per_launch"], t["source"]) if t else (None, None)


# ---------------------------------------------------------------------------- distributed plumbing
def dist_setup(args):
    ws = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if ws > 1 and args.impl != "reference":
        import datetime
        import torch
        import torch.distributed as dist
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=torch.device("cuda", local))
    return ws, rank, local


def barrier(ws):
    if ws > 1:
        import torch.distributed as dist
        dist.barrier()


def max_over_ranks(ws, v: float) -> float:
    if ws == 1:
        return v
    import torch
    import torch.distributed as dist
    t = torch.tensor([v], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


class Clocks:
    """SM clock and clock-event (throttle) reasons sampled while the GPU
    runs the measured work: NVML on a thread (as fast as NVML answers), or
    nvidia-smi -lms 200 when NVML is unavailable.  Only reads settings."""

    REASONS = (("hw_slowdown", 0x8), ("sw_power_cap", 0x4), ("sw_thermal_slowdown", 0x20),
               ("hw_thermal_slowdown", 0x40))

    def __init__(self, gpu: int):
        self.samples, self.mask, self.mx, self.p, self.h = [], 0, None, None, None
        try:
            import threading
            import pynvml
            import torch
            pynvml.nvmlInit()
            self.nv = pynvml
            try:   # the physical GPU behind CUDA device `gpu`
                self.h = pynvml.nvmlDeviceGetHandleByUUID("GPU-" + str(torch.cuda.get_device_properties(gpu).uuid))
            except Exception:
                self.h = pynvml.nvmlDeviceGetHandleByIndex(gpu)
            self.mx = float(pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM))
            self.run = True
            self._old_si = sys.getswitchinterval()
            sys.setswitchinterval(0.0002)   # let the sampler in while the main thread works
            self.t = threading.Thread(target=self._loop, daemon=True)
            self.t.start()
        except Exception:
            self.h = None
            self._start_smi(gpu)

    def _loop(self):
        nv = self.nv
        while self.run:
            try:
                self.samples.append(float(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM)))
                self.mask |= int(nv.nvmlDeviceGetCurrentClocksEventReasons(self.h))
            except Exception:
                pass
            time.sleep(0.0005)

    def mark(self):
        """Number of samples so far (to count those inside the timed region)."""
        return len(self.samples)

    def _start_smi(self, gpu):
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
             "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
             "clocks_event_reasons.sw_power_cap")
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={q}", "--format=csv,noheader,nounits", "-lms", "200",
                                       "-i", str(gpu)], stdout=self.f, stderr=subprocess.DEVNULL)
        except Exception:
            self.p = None

    def stop(self, timed_span=None):
        if self.h is not None:
            self.run = False
            self.t.join(timeout=2)
            sys.setswitchinterval(self._old_si)
            sm = sorted(self.samples)
            reasons = sorted(n for n, bit in self.REASONS if self.mask & bit)
            out = {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": self.mx, "reasons": reasons,
                   "samples": len(sm), "source": "nvml"}
            if timed_span is not None:
                out["samples_in_timed_region"] = timed_span[1] - timed_span[0]
            return out
        if self.p is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        time.sleep(0.25)
        self.p.terminate()
        try:
            self.p.wait(timeout=5)
        except Exception:
            self.p.kill()
        self.f.seek(0)
        rows = [r.split(",") for r in self.f.read().strip().splitlines() if r.strip()]
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for r in rows:
            try:
                sm.append(float(r[1]))
                mx = float(r[2])
                for n, v in zip(names, r[5:9]):
                    if "Active" in v and "Not" not in v:
                        reasons.add(n)
            except (ValueError, IndexError):
                continue
        sm.sort()
        return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm), "source": "nvidia-smi"}


# ---------------------------------------------------------------------------- reference arm / CPU baseline
# Host-only: these build the workload trees (amcuda.morph / amcuda.workloads
# need no library) and run the oracle port of the reference's CPU path.
def _oracle_filterbank_sample(args):
    """One oracle realize of the filter-bank tree on a signal sample; returns
    (seconds, algorithmic bytes)."""
    sig, length = args
    sys.path.insert(0, str(ROOT / "oracle"))
    import oracle
    from amcuda import morph as M
    from amcuda import workloads as W
    x = W.c2_signal(sig, length)[None, :]
    h = W.c2_prototype()
    tree = W.c2_tree(M.morph_from_numpy(x), M.morph_from_numpy(h))
    oracle.lib()
    t0 = time.perf_counter()
    oracle.realize(tree)
    dt = time.perf_counter() - t0
    F = W.c2_frames(length)
    return dt, length * 4 + F * 64 * 4 + 4096


def cpu_filterbank(length: int):
    """The oracle on one signal sample, one thread: (GB/s, seconds)."""
    dt, by = _oracle_filterbank_sample((0, length))
    return by / dt / 1e9, dt


def _timed(fn, min_s: float = 1.0):
    """Mean seconds of fn() over repeats totalling at least min_s (at least one)."""
    fn()   # first call builds / warms the oracle
    n, t0 = 0, time.perf_counter()
    while True:
        fn()
        n += 1
        dt = time.perf_counter() - t0
        if dt >= min_s:
            return dt / n


def _oracle_unit(wl: str, dtype: str):
    """One bounded unit of a workload for the oracle port of the reference's
    CPU path: (run, work in the GPU arm's unit, unit, scale, sample text)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np
    import oracle
    from amcuda import morph as M
    from amcuda import workloads as W
    oracle.lib()
    if wl == "fused":
        xm, ym = W.c1_inputs_morph(dtype)
        tree = W.c1_tree(xm, ym)
        esz = 8 if dtype == "f64" else 4
        return ((lambda: oracle.realize(tree)), (2 * (1 << 19) + 1024) * esz, "GB/s", 1e9,
                f"the whole config-1 tree ({dtype}), per-node realize with materialised map and add nodes")
    if wl == "linreg":
        rows, d = 1 << 15, 256
        X, y, _ = W.c5_inputs(rows, d)
        return ((lambda: oracle.linreg(X, y, np.zeros(d), 1, 0.1)), rows * (d + 1) * 8, "GB/s", 1e9,
                f"{rows} of the 2^22 rows, one step of the SSA replay (GEMV, residual, mean, strided GEMM)")
    if wl == "attention":
        n, dh = 2048, 64
        q, k, v, do = (W.normal(W.seed_of(4, j), n * dh).astype(np.float32).reshape(1, n, dh) for j in range(4))
        tree = M.attention_morphism(M.morph_from_numpy(q), M.morph_from_numpy(k), M.morph_from_numpy(v), 0.125)

        def run():
            oracle.realize(tree)
            oracle.attention_bwd(q, k, v, do, 0.125)
        return (run, 12.0 * n * n * dh, "TFLOP/s", 1e12,
                "1 of the 256 (batch, head) blocks: the %attn-2d! restatement forward and a double-precision VJP")
    x = W.normal(W.seed_of(3, 0), 64 * 56 * 56).astype(np.float32).reshape(1, 64, 56, 56)
    w = (W.normal(W.seed_of(3, 1), 64 * 64 * 9) * np.sqrt(2 / 576)).astype(np.float32).reshape(64, 64, 3, 3)
    dy = W.normal(W.seed_of(3, 2), 64 * 56 * 56).astype(np.float32).reshape(1, 64, 56, 56)

    def run():
        oracle.conv2d_fwd(x, w)
        oracle.conv2d_dgrad(dy, w, x.shape)
        oracle.conv2d_wgrad(x, dy, w.shape)
    return (run, 3 * 2.0 * 64 * 64 * 9 * 56 * 56, "TFLOP/s", 1e12,
            "1 of the 64 images: im2col + double-accumulating GEMM forward, col2im data gradient, weight gradient")


def cpu_other(wl: str, dtype: str) -> dict:
    """The oracle port timed on a bounded sample of the workload, 1 thread."""
    run, work, unit, scale, what = _oracle_unit(wl, dtype)
    t = _timed(run)
    return {"value": work / t / scale, "unit": unit, "cores": 1, "kind": "port", "sample": what + ", 1 thread"}


def _oracle_other_sample(job):
    """One bounded unit (see _oracle_unit) timed once: (seconds, work)."""
    wl, dtype = job
    run, work, _, _, _ = _oracle_unit(wl, dtype)
    t0 = time.perf_counter()
    run()
    return time.perf_counter() - t0, work


_OTHER_ARM = {
    "fused": ("GB/s", 1e9, "the whole config-1 tree ({dtype}) per process per step"),
    "linreg": ("GB/s", 1e9, "2^15 of the 2^22 rows of one step per process per step"),
    "attention": ("TFLOP/s", 1e12, "1 of the 256 (batch, head) blocks, forward and backward, per process per step"),
    "conv": ("TFLOP/s", 1e12, "1 of the 64 images, three passes, per process per step"),
}
_METRIC = {
    "fused": "fused view+map+reduce realize GB/s ({dtype})",
    "linreg": "linear-regression SSA training step GB/s (ssa-realize/ctx replay, one pass over X)",
    "attention": "attention forward + backward TFLOP/s",
    "conv": "conv2d forward + data gradient + weight gradient TFLOP/s",
}


def other_config(wl: str, args, dtype: str | None = None) -> dict:
    """The `config` of a non-headline workload (both arms)."""
    dtype = dtype or args.dtype
    if wl == "fused":
        return {"workload": f"config 1: x,y 2^20 {dtype}, reshape 1024x1024, transpose, slice step 2, "
                            f"sum(x^2+y) over axis 1", "l2": "256 MB flush between steps", "parallelism": "replicas"}
    if wl == "linreg":
        return {"workload": f"config 5: X {args.rows} x 256 f64 per GPU, loss mean((X w - y)^2), gradient by "
                            f"reverse-mode SSA, plain gradient step lr 0.1, ssa-realize/ctx replay",
                "l2": "X (8 GiB) larger than L2", "parallelism": "rows sharded, gradient summed over ranks"}
    if wl == "attention":
        return {"workload": f"config 4: Q,K,V,dO ({args.batch or 16},16,2048,64) f32, scale 1/8; O, dQ, dK, dV per step",
                "flops": "algorithmic 12*B*H*S^2*D (6 GEMMs; the backward recomputes S and dP twice more)",
                "l2": "operands (0.54 GB) larger than L2", "parallelism": "batch sharded"}
    return {"workload": f"config 3: x ({args.batch or 64},64,56,56) f32, w (64,64,3,3), stride 1 pad 1; "
                        f"Y, dX and dW per step", "l2": "x, dY, Y, dX (205 MB) larger than L2",
            "parallelism": "batch sharded, dW summed over ranks"}


def _ref_pool_steps(pool, jobs, args, steps=None):
    times, vals = [], []
    steps = args.steps if steps is None else steps
    for i in range(args.warmup + steps):
        res = pool.map(_oracle_other_sample, jobs)
        # the processes run their units side by side: the step takes the
        # longest one (input generation and process start-up excluded)
        dt = max(r[0] for r in res)
        if i >= args.warmup:
            times.append(dt)
            vals.append(sum(r[1] for r in res) / dt)
    return times, vals


def reference_line_other(args, cores, wl, dtype, pool, steps=None) -> dict:
    """The reference arm of a non-headline workload: the oracle port on every
    host core (one spawned process per core, each running one bounded unit),
    whole-job work over the wall time of each step."""
    unit, scale, what = _OTHER_ARM[wl]
    times, vals = _ref_pool_steps(pool, [(wl, dtype)] * cores, args, steps)
    value = sum(vals) / len(vals) / scale
    sample = (what.format(dtype=dtype) + f", {cores} spawned processes running side by side, step time = the "
              f"longest process, oracle port of the reference's CPU path")
    return {"impl": "reference", "metric": _METRIC[wl].format(dtype=dtype), "value": value, "unit": unit,
            "n_gpus": args.gpus, "steps": len(times), "warmup": args.warmup,
            "ms_per_step": 1000 * sum(times) / len(times), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": dtype if wl in ("fused", "linreg") else "f32", "data": "synthetic",
            "config": dict(other_config(wl, args, dtype), sample=sample),
            "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}


PER_CONFIG = [("fused_f64", "fused", "f64"), ("fused_s32", "fused", "s32"), ("conv", "conv", "f32"),
              ("attention", "attention", "f32"), ("linreg", "linreg", "f64")]


def reference_arm(args, ws, rank):
    if rank != 0:
        return
    cores = args.ref_procs or os.cpu_count() or 1
    with mp.get_context("spawn").Pool(cores) as pool:
        if args.workload not in ("all", "filterbank"):
            print(json.dumps(reference_line_other(args, cores, args.workload, args.dtype, pool)))
            return
        length = 1 << 20
        pool.map(_oracle_filterbank_sample, [(s, 1 << 14) for s in range(cores)])  # spawn + oracle build
        times, vals = [], []
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            res = pool.map(_oracle_filterbank_sample, [(s, length) for s in range(cores)])
            dt = time.perf_counter() - t0
            if i >= args.warmup:
                times.append(dt)
                vals.append(sum(r[1] for r in res) / dt / 1e9)
        value = sum(vals) / len(vals)
        sample = (f"{cores} signals x 2^20 samples per step (of the 64 x 2^24 workload), oracle port of the "
                  f"reference's per-node realize, one spawned process per host core")
        out = {
            "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * sum(times) / len(times),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "config": dict(CONFIG_FB, sample=sample),
            "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
            "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        }
        if args.workload == "all" and not args.no_per_config:
            # one timed step of each (a few seconds of host work apiece)
            out["per_config"] = {name: reference_line_other(args, cores, wl, dt, pool, steps=1)
                                 for name, wl, dt in PER_CONFIG}
        print(json.dumps(out))


METRIC = "fused realize() HBM GB/s (polyphase filter bank)"
CONFIG_FB = {"workload": "polyphase filter bank: 64 signals x 2^24 f32 per GPU, 64 branches x 16 taps, "
                         "1024-tap Hamming sinc prototype (cutoff 1/64), frames 262129",
             "signals_per_gpu": 64, "samples": 1 << 24, "branches": 64, "taps": 16,
             "l2": "inputs (4 GiB per GPU) larger than L2; no flush needed", "parallelism": "batch-sharded, weak"}


# ---------------------------------------------------------------------------- device helpers
def _cudart():
    import ctypes as C
    import torch  # noqa: F401  (loads the CUDA runtime)
    for name in ("libcudart.so.12", "libcudart.so"):
        try:
            return C.CDLL(name)
        except OSError:
            continue
    import glob
    for p in glob.glob(os.path.join(os.path.dirname(__import__("torch").__file__), "lib", "libcudart*.so*")):
        return C.CDLL(p)
    raise RuntimeError("libcudart not found")


def cudart_copy(dst: int, src: int, nbytes: int, kind: int = 3):
    """cudaMemcpy (kind 3: device to device, 2: device to host)."""
    import ctypes as C
    rt = _cudart()
    rt.cudaMemcpy.restype = C.c_int
    rc = rt.cudaMemcpy(C.c_void_p(dst), C.c_void_p(src), C.c_size_t(nbytes), kind)
    if rc:
        raise RuntimeError(f"cudaMemcpy failed {rc}")


def device_buffer_from(t, dtype: str):
    """A library buffer holding a copy of the torch CUDA tensor t."""
    import amcuda as am
    b = am.DeviceBuffer.create(dtype, t.numel())
    cudart_copy(b.devptr(), t.data_ptr(), t.numel() * t.element_size())
    return b


class CudaView:
    """A device pointer presented to torch (__cuda_array_interface__)."""

    def __init__(self, ptr: int, n: int, typestr: str = "<f8"):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": typestr, "data": (ptr, False), "version": 3}


def _release():
    import torch
    gc.collect()
    torch.cuda.synchronize()
    torch.cuda.empty_cache()


def time_steps(run, steps, warmup, stream, local, ws, pre=None, min_region_s: float = 0.0, max_steps: int = 20000):
    """Warm up, then time `steps` steps (more when one step is so short that
    the region would be under min_region_s) with CUDA events on `stream`,
    each step bracketed by its own events; clocks sampled meanwhile.
    Returns (per-step ms list, steps, clocks)."""
    import torch
    for _ in range(warmup):
        if pre:
            pre()
        run()
    torch.cuda.synchronize()
    if min_region_s > 0:
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        run()
        b.record(stream)
        torch.cuda.synchronize()
        est = max(a.elapsed_time(b) / 1e3, 1e-6)
        steps = max(steps, min(max_steps, int(math.ceil(min_region_s / est))))
        # every rank runs the same number of steps (collectives pair up)
        steps = int(max_over_ranks(ws, float(steps)))
    barrier(ws)
    clk = Clocks(local)
    time.sleep(0.01)
    evs = []
    m0 = clk.mark()
    for _ in range(steps):
        if pre:
            pre()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        run()
        b.record(stream)
        evs.append((a, b))
    torch.cuda.synchronize()
    m1 = clk.mark()
    clocks = clk.stop((m0, m1))
    return [a.elapsed_time(b) for a, b in evs], steps, clocks


def time_e2e(step, steps, stream):
    """Wall of `steps` end-to-end steps on `stream` by CUDA events (ms)."""
    import torch
    step()
    torch.cuda.synchronize()
    a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    a.record(stream)
    for _ in range(steps):
        step()
    b.record(stream)
    torch.cuda.synchronize()
    return a.elapsed_time(b)


def make_rank_sum(ws: int, n: int):
    """The in-place rank-order sum of an n-element device vector over the
    ranks: the library's peer-memory kernels (amcuda.dist.PeerSum) when the
    GPUs reach each other, else allreduce_fixed_order over NCCL."""
    if ws == 1:
        return None
    from amcuda.dist import PeerSum, allreduce_fixed_order
    try:
        ps = PeerSum(n)
    except Exception as e:   # no peer access between these GPUs
        print(f"bench: peer-memory rank sum unavailable ({e}); using allreduce_fixed_order", file=sys.stderr)
        return allreduce_fixed_order

    def run(t, stream=None):
        return ps.sum_(t, stream)
    run.peer = ps
    return run


def close_rank_sum(fn):
    if fn is not None and hasattr(fn, "peer"):
        fn.peer.close()


_TC_PEAK = {}


def tf32_peak():
    if "v" not in _TC_PEAK:
        from amcuda import workloads as W
        _TC_PEAK["v"] = W.tc_peak_tf32(4000)
    return _TC_PEAK["v"]


def entry(metric, value, unit, ms, steps, dtype, cfg, roofline, cpu, e2e, launches, clocks, **extra):
    d = {"metric": metric, "value": value, "unit": unit, "ms_per_step": ms, "steps": steps, "dtype": dtype,
         "config": cfg, "roofline": roofline, "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": launches,
         "clocks": clocks}
    d.update(extra)
    return d


# ---------------------------------------------------------------------------- GPU arm: filter bank (headline)
def bench_filterbank(args, ws, rank, local):
    import ctypes as C
    import torch
    import amcuda as am
    from amcuda import _abi as A
    from amcuda import workloads as W
    am.init(local)
    torch.cuda.set_device(local)
    B, L = args.signals, args.samples
    F = W.c2_frames(L)
    x_t = W.c2_signals_torch(B, L, device="cuda", first=rank * B)
    h_t = torch.from_numpy(W.c2_prototype()).cuda()
    xb = device_buffer_from(x_t, "f32")
    hb = device_buffer_from(h_t, "f32")
    del x_t
    _release()
    xm = am.Concrete(None, (B, L), dtype="f32", dev=xb)
    hm = am.Concrete(None, (W.PROTO,), dtype="f32", dev=hb)
    plan = am.Plan(W.c2_tree(xm, hm))
    st = plan.stats()
    stream = torch.cuda.Stream()  # an explicit stream: events and launches share it
    torch.cuda.set_stream(stream)
    sptr = stream.cuda_stream
    step_ms, steps, clocks = time_steps(lambda: plan.execute(sptr), args.steps, args.warmup, stream, local, ws)
    total_ms = max_over_ranks(ws, sum(step_ms))
    bytes_step = B * L * 4 + B * F * 64 * 4 + 4 * W.PROTO
    value = ws * bytes_step * steps / (total_ms / 1e3) / 1e9
    hbm, _, kind = peaks()
    achieved = bytes_step / (sum(step_ms) / len(step_ms) / 1e3) / 1e9
    traffic, tsrc = traffic_of("filterbank")

    # ---- end to end: pinned host signals -> device -> realize -> host result.
    # Two buffer sets (two plans of the same public tree) and three streams:
    # step k's upload, step k-1's realize and step k-2's download run at once,
    # so the two PCIe directions overlap each other and the kernel.  Every step
    # still moves its whole input in and its whole result out.
    e2e = None
    if not args.no_e2e:
        x_host = torch.empty((B, L), dtype=torch.float32, pin_memory=True)
        out_host = torch.empty((B, F, 64), dtype=torch.float32, pin_memory=True)
        cudart_copy(x_host.data_ptr(), xb.devptr(), 4 * B * L, 2)
        xb2 = am.DeviceBuffer.create("f32", B * L)
        plan2 = am.Plan(W.c2_tree(am.Concrete(None, (B, L), dtype="f32", dev=xb2), hm))
        sets = [(xb, plan, plan.result()._dev), (xb2, plan2, plan2.result()._dev)]
        s_in, s_run, s_out = torch.cuda.Stream(), torch.cuda.Stream(), torch.cuda.Stream()
        e_steps = max(4, min(args.steps, 6))
        ev = lambda: torch.cuda.Event(enable_timing=False)

        def pipeline(n, t0=None, t1=None):
            up_done, run_done, down_done = [None] * n, [None] * n, [None] * n
            if t0 is not None:
                t0.record(s_in)
            for k in range(n):
                xbk, pk, outk = sets[k % 2]
                # input buffer free once step k-2's realize finished; output once its download did
                if k >= 2:
                    s_in.wait_event(run_done[k - 2])
                A.call("amc_buf_upload_async", xbk.handle, C.c_void_p(x_host.data_ptr()), 4 * B * L, 0,
                       C.c_void_p(s_in.cuda_stream))
                up_done[k] = ev(); up_done[k].record(s_in)
                s_run.wait_event(up_done[k])
                if k >= 2:
                    s_run.wait_event(down_done[k - 2])
                pk.execute(s_run.cuda_stream)
                run_done[k] = ev(); run_done[k].record(s_run)
                s_out.wait_event(run_done[k])
                A.call("amc_buf_download_async", outk.handle, C.c_void_p(out_host.data_ptr()), 4 * B * F * 64, 0,
                       C.c_void_p(s_out.cuda_stream))
                down_done[k] = ev(); down_done[k].record(s_out)
            if t1 is not None:
                t1.record(s_out)

        pipeline(2)
        torch.cuda.synchronize()
        barrier(ws)
        s0, s1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        pipeline(e_steps, s0, s1)
        torch.cuda.synchronize()
        e_ms = max_over_ranks(ws, s0.elapsed_time(s1))
        e2e = {"value": ws * bytes_step * e_steps / (e_ms / 1e3) / 1e9, "unit": "GB/s",
               "h2d_bytes_per_step": 4 * B * L, "d2h_bytes_per_step": 4 * B * F * 64, "steps": e_steps,
               "path": "two Plans of the public realize tree over two device buffer sets; per step "
                       "amc_buf_upload_async of the signals from pinned memory, execute, amc_buf_download_async of "
                       "the (B,F,64) result, on three streams so consecutive steps' copies and realize overlap"}
        del plan2, xb2, sets, x_host, out_host

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        v, wall = cpu_filterbank(1 << 22)
        cpu = {"value": v, "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": f"1 signal x 2^22 samples through the oracle port of the reference's per-node realize "
                         f"(im2col, product and tap reduction materialised), 1 thread, {wall:.1f} s"}
    out = {
        "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": ws, "steps": steps,
        "warmup": args.warmup, "ms_per_step": total_ms / steps, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": CONFIG_FB,
        "roofline": {"bound": "hbm", "kernel": "k_fir_tma (+ k_fir_tail)", "achieved": achieved, "peak": hbm,
                     "unit": "GB/s", "frac": achieved / hbm, "traffic": traffic, "traffic_source": tsrc,
                     "peak_source": f"{kind} (MEASURED_PEAKS.json hbm_gbs)" if kind == "measured" else kind,
                     "algorithmic_bytes_per_launch": bytes_step},
        "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": st["launches"] * steps, "clocks": clocks,
    }
    del plan, xm, hm, xb, hb
    _release()
    return out


# ---------------------------------------------------------------------------- GPU arm: the other configs
def pc_fused(args, ws, rank, local, dtype):
    """Config 1 through realize: the view + map + reduce tree on device leaves."""
    import ctypes as C
    import torch
    import amcuda as am
    from amcuda import _abi as A
    from amcuda import workloads as W
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    x, y = W.c1_inputs(dtype)
    xm, ym = am.morph_from_numpy(x, dtype), am.morph_from_numpy(y, dtype)
    plan = am.Plan(W.c1_tree(xm, ym))
    esz = 8 if dtype == "f64" else 4
    work = 2 * (1 << 19) * esz + 1024 * esz
    flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
    ms, steps, clocks = time_steps(lambda: plan.execute(sptr), args.steps, args.warmup, stream, local, ws,
                                   pre=lambda: flush.fill_(1), min_region_s=0.3, max_steps=4000)
    t = max_over_ranks(ws, sum(ms))
    hbm, _, kind = peaks()
    per = work / (sum(ms) / len(ms) / 1e3) / 1e9
    e2e = None
    if not args.no_e2e:
        from amcuda.realize import device_buffer_of
        xh = torch.from_numpy(x).pin_memory()
        yh = torch.from_numpy(y).pin_memory()
        out_dev = plan.result()._dev
        oh = torch.empty(1024 * esz, dtype=torch.uint8, pin_memory=True)
        xbuf, ybuf = device_buffer_of(xm), device_buffer_of(ym)
        sp = C.c_void_p(sptr)

        def step():
            A.call("amc_buf_upload_async", xbuf.handle, C.c_void_p(xh.data_ptr()), x.nbytes, 0, sp)
            A.call("amc_buf_upload_async", ybuf.handle, C.c_void_p(yh.data_ptr()), y.nbytes, 0, sp)
            plan.execute(sptr)
            A.call("amc_buf_download_async", out_dev.handle, C.c_void_p(oh.data_ptr()), 1024 * esz, 0, sp)
        n_e = 50
        e_ms = max_over_ranks(ws, time_e2e(step, n_e, stream))
        e2e = {"value": ws * work * n_e / (e_ms / 1e3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": x.nbytes + y.nbytes,
               "d2h_bytes_per_step": 1024 * esz, "steps": n_e,
               "path": "amc_buf_upload_async of x and y from pinned memory into the plan's leaves, the realize "
                       "plan, amc_buf_download_async of the 1024 sums, one stream"}
    # the same step on inputs larger than L2 instead of a flush: 16 copies of
    # x and y (16 plans) realized in turn, back to back, so every step reads
    # its leaves from HBM without the write-back of a 256 MB flush before it
    cold = None
    if not args.no_cold:
        copies = [am.Plan(W.c1_tree(am.morph_from_numpy(x, dtype), am.morph_from_numpy(y, dtype)))
                  for _ in range(16)]
        for q in copies:
            q.execute(sptr)
        torch.cuda.synchronize()
        barrier(ws)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        rounds = 64
        a.record(stream)
        for _ in range(rounds):
            for q in copies:
                q.execute(sptr)
        b.record(stream)
        torch.cuda.synchronize()
        c_ms = max_over_ranks(ws, a.elapsed_time(b)) / (rounds * len(copies))
        cold = {"ms_per_step": c_ms, "value": ws * work / (c_ms / 1e3) / 1e9, "unit": "GB/s",
                "steps": rounds * len(copies),
                "method": "16 input copies (%d MiB) realized in turn, back to back, one event pair around all steps"
                          % (16 * 2 * x.nbytes >> 20)}
        del copies
    cpu = cpu_other("fused", dtype) if rank == 0 and ws == 1 and not args.no_cpu else None
    traffic, tsrc = traffic_of(f"fused_{dtype}")
    launches = plan.stats()["launches"]
    return entry(_METRIC["fused"].format(dtype=dtype), ws * work * steps / (t / 1e3) / 1e9, "GB/s", t / steps, steps,
                 dtype, other_config("fused", args, dtype),
                 {"bound": "hbm", "kernel": "k_colfold", "achieved": per, "peak": hbm, "unit": "GB/s",
                  "frac": per / hbm, "traffic": traffic, "traffic_source": tsrc, "peak_source": kind + " hbm_gbs",
                  "algorithmic_bytes_per_launch": work},
                 cpu, e2e, launches * steps, clocks, scaling="replicas", cold_inputs=cold)


def pc_conv(args, ws, rank, local):
    """Config 3 through the conv entry points (the plugin seam of
    execute-conv2d-blas): Y, dX and dW per step."""
    import numpy as np
    import torch
    from amcuda import workloads as W
    stream = torch.cuda.current_stream()
    N = args.batch or 64
    gen = lambda j, n: W.normal(W.seed_of(3, j), n, start=rank * n if j != 1 else 0)
    x = torch.from_numpy(gen(0, N * 64 * 56 * 56).astype(np.float32)).cuda().view(N, 64, 56, 56)
    wt = torch.from_numpy((gen(1, 64 * 64 * 9) * math.sqrt(2 / 576)).astype(np.float32)).cuda().view(64, 64, 3, 3)
    dy = torch.from_numpy(gen(2, N * 64 * 56 * 56).astype(np.float32)).cuda().view(N, 64, 56, 56)
    yy, dx, dw = torch.empty_like(x), torch.empty_like(x), torch.empty_like(wt)
    rank_sum = make_rank_sum(ws, dw.numel())
    # dW first: its rank-order sum (peer-memory kernels of a few registers,
    # which fit beside the conv CTAs) runs on a side stream while the
    # forward and data-gradient passes run on the main one
    overlap = rank_sum is not None and hasattr(rank_sum, "peer")
    side = torch.cuda.Stream() if overlap else None
    w_done, s_done = torch.cuda.Event(), torch.cuda.Event()

    def run():
        W.conv2d_wgrad(x, dy, dw)
        if overlap:
            w_done.record(stream)
            side.wait_event(w_done)
            rank_sum(dw, side.cuda_stream)   # dW sums over the batch shards, in rank order
        W.conv2d_fwd(x, wt, yy)
        W.conv2d_dgrad(dy, wt, dx)
        if overlap:
            s_done.record(side)
            stream.wait_event(s_done)
        elif ws > 1:
            rank_sum(dw)
    work = 3 * 2.0 * N * 64 * 64 * 9 * 56 * 56
    ms, steps, clocks = time_steps(run, args.steps, args.warmup, stream, local, ws, min_region_s=0.3, max_steps=4000)
    t = max_over_ranks(ws, sum(ms))
    peak = tf32_peak()
    per = work / (sum(ms) / len(ms) / 1e3) / 1e12
    e2e = None
    if not args.no_e2e:
        xh, dyh = x.cpu().pin_memory(), dy.cpu().pin_memory()
        yh, dxh, dwh = (torch.empty(t_.shape, dtype=torch.float32, pin_memory=True) for t_ in (yy, dx, dw))

        def step():
            x.copy_(xh, non_blocking=True)
            dy.copy_(dyh, non_blocking=True)
            run()
            yh.copy_(yy, non_blocking=True)
            dxh.copy_(dx, non_blocking=True)
            dwh.copy_(dw, non_blocking=True)
        n_e = 10
        e_ms = max_over_ranks(ws, time_e2e(step, n_e, stream))
        e2e = {"value": ws * work * n_e / (e_ms / 1e3) / 1e12, "unit": "TFLOP/s",
               "h2d_bytes_per_step": 2 * x.numel() * 4, "d2h_bytes_per_step": 2 * x.numel() * 4 + dw.numel() * 4,
               "steps": n_e, "path": "x and dY copied from pinned memory, amc_conv2d_fwd/dgrad/wgrad_f32, Y, dX and "
                                     "dW copied back, one stream"}
    cpu = cpu_other("conv", "f32") if rank == 0 and ws == 1 and not args.no_cpu else None
    traffic, tsrc = traffic_of("conv")
    close_rank_sum(rank_sum)
    return entry(_METRIC["conv"], ws * work * steps / (t / 1e3) / 1e12, "TFLOP/s", t / steps, steps, "f32",
                 other_config("conv", args),
                 {"bound": "tensor", "kernel": "k_conv3x3_tc, k_conv_wgrad_tc", "achieved": per, "peak": peak,
                  "unit": "TFLOP/s", "frac": per / peak, "traffic": traffic, "traffic_source": tsrc,
                  "peak_source": "dense TF32 rate of a tcgen05 kind::tf32 M=128 N=256 issue loop on this GPU "
                                 "(amc_tc_peak_tf32), measured in this run",
                  "algorithmic_flops_per_step": work},
                 cpu, e2e, 6 * steps, clocks, scaling="weak")


def pc_attention(args, ws, rank, local):
    """Config 4 through the attention entry points: O, dQ, dK, dV per step."""
    import numpy as np
    import torch
    from amcuda import workloads as W
    stream = torch.cuda.current_stream()
    B, H, S, D = args.batch or 16, 16, 2048, 64
    n = B * H * S * D
    q, k, v, do = (torch.from_numpy(W.normal(W.seed_of(4, j), n, start=rank * n).astype(np.float32)).cuda()
                   .view(B, H, S, D) for j in range(4))
    o = torch.empty_like(q)
    lse = torch.empty((B, H, S), dtype=torch.float32, device="cuda")
    dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)

    def run():
        W.attention_fwd(q, k, v, o, lse, 1.0 / 8.0)
        W.attention_bwd(q, k, v, o, do, lse, dq, dk, dv, 1.0 / 8.0)
    work = 12.0 * B * H * S * S * D
    ms, steps, clocks = time_steps(run, args.steps, args.warmup, stream, local, ws, min_region_s=0.3, max_steps=2000)
    t = max_over_ranks(ws, sum(ms))
    peak = tf32_peak()
    per = work / (sum(ms) / len(ms) / 1e3) / 1e12
    e2e = None
    if not args.no_e2e:
        hs = [a.cpu().pin_memory() for a in (q, k, v, do)]
        outs = [torch.empty(a.shape, dtype=torch.float32, pin_memory=True) for a in (o, dq, dk, dv)]

        def step():
            for dev_t, h in zip((q, k, v, do), hs):
                dev_t.copy_(h, non_blocking=True)
            run()
            for h, dev_t in zip(outs, (o, dq, dk, dv)):
                h.copy_(dev_t, non_blocking=True)
        n_e = 6
        e_ms = max_over_ranks(ws, time_e2e(step, n_e, stream))
        e2e = {"value": ws * work * n_e / (e_ms / 1e3) / 1e12, "unit": "TFLOP/s", "h2d_bytes_per_step": 4 * n * 4,
               "d2h_bytes_per_step": 4 * n * 4, "steps": n_e,
               "path": "Q, K, V, dO copied from pinned memory, amc_attention_fwd_f32 + amc_attention_bwd_f32, O, dQ, "
                       "dK, dV copied back, one stream"}
    cpu = cpu_other("attention", "f32") if rank == 0 and ws == 1 and not args.no_cpu else None
    traffic, tsrc = traffic_of("attention")
    return entry(_METRIC["attention"], ws * work * steps / (t / 1e3) / 1e12, "TFLOP/s", t / steps, steps, "f32",
                 other_config("attention", args),
                 {"bound": "tensor", "kernel": "k_attn_fwd_tc3, k_attn_bwd_dkv_tc, k_attn_bwd_dq_tc", "achieved": per,
                  "peak": peak, "unit": "TFLOP/s", "frac": per / peak, "traffic": traffic, "traffic_source": tsrc,
                  "peak_source": "dense TF32 rate of a tcgen05 kind::tf32 M=128 N=256 issue loop on this GPU "
                                 "(amc_tc_peak_tf32), measured in this run",
                  "algorithmic_flops_per_step": work},
                 cpu, e2e, 6 * steps, clocks, scaling="weak")


def pc_linreg(args, ws, rank, local):
    """Config 5 through the public SSA path (workloads.LinregSSA): the MSE
    program compiled by morphism-to-ssa / ssa-vjp, one traced step, then
    ssa-realize/ctx replays with an in-place gradient step.  Rows are
    sharded; at N > 1 each replay's gradient is summed over the ranks in rank
    order before the step (lr / N: the mean over all rows)."""
    import ctypes as C
    import numpy as np
    import torch
    import amcuda as am
    from amcuda import _abi as A
    from amcuda import workloads as W
    stream = torch.cuda.current_stream()
    sptr = stream.cuda_stream
    n, d = args.rows, 256
    X_t, y_t = W.c5_shard_torch(n, d, rank)
    xb, yb = device_buffer_from(X_t, "f64"), device_buffer_from(y_t, "f64")
    del X_t, y_t
    _release()
    Xm = am.Concrete(None, (n, d), dtype="f64", dev=xb)
    ym = am.Concrete(None, (n, 1), dtype="f64", dev=yb)
    hook = None
    rank_sum = make_rank_sum(ws, d)
    if ws > 1:
        views = {}   # the replay's gradient lives at a fixed arena address: one torch view of it

        def hook(dw):
            # the gradient sums over the row shards, in rank order
            if dw._dev is None:   # the traced step's gradient comes back on the host
                arr = dw.data
                t_ = torch.from_numpy(arr[dw.offset:dw.offset + d].copy()).cuda()
                rank_sum(t_)
                arr[dw.offset:dw.offset + d] = t_.cpu().numpy()
            else:
                ptr = dw._dev.devptr() + 8 * dw.offset
                if ptr not in views:
                    views[ptr] = torch.as_tensor(CudaView(ptr, d), device="cuda")
                rank_sum(views[ptr])
    steps_total = args.warmup + max(args.steps, 64) + 64
    tr = W.LinregSSA(Xm, ym, np.zeros(d), 0.1 / ws, stream=sptr, max_steps=steps_total + 16, grad_hook=hook)
    tr.trace()
    tr.step()     # compiles the replay plan
    work = n * d * 8 + n * 8
    ms, steps, clocks = time_steps(tr.step, args.steps, args.warmup, stream, local, ws, min_region_s=0.08,
                                   max_steps=64)
    t = max_over_ranks(ws, sum(ms))
    hbm, _, kind = peaks()
    per = work / (sum(ms) / len(ms) / 1e3) / 1e9
    replay_launches = tr.replay_launches()
    # the hand-fused kernels of the same step on the same data (amc_linreg_step), for comparison
    direct = None
    if ws == 1:
        w_ = torch.zeros(d, dtype=torch.float64, device="cuda")
        npart = W.linreg_partials_count(n, d)
        part = torch.empty(npart * (d + 1), dtype=torch.float64, device="cuda")
        gl = torch.empty(d + 1, dtype=torch.float64, device="cuda")
        loss = torch.empty(1, dtype=torch.float64, device="cuda")
        lib = A.load()

        def direct_step():
            A.check(lib.amc_linreg_step(C.c_void_p(xb.devptr()), C.c_void_p(yb.devptr()), C.c_void_p(w_.data_ptr()),
                                        n, d, C.c_double(0.1), C.c_void_p(part.data_ptr()),
                                        C.c_void_p(gl.data_ptr()), C.c_void_p(loss.data_ptr()), C.c_void_p(sptr)))
        dms, dsteps, _ = time_steps(direct_step, args.steps, args.warmup, stream, local, 1)
        direct = {"value": work / (sum(dms) / len(dms) / 1e3) / 1e9, "unit": "GB/s",
                  "ms_per_step": sum(dms) / len(dms), "steps": dsteps,
                  "path": "amc_linreg_step: the hand-fused partials, reduce and update kernels on the same X, y"}
        del part
    e2e = None
    if not args.no_e2e:
        Xh = torch.empty(n * d, dtype=torch.float64, pin_memory=True)
        yh = torch.empty(n, dtype=torch.float64, pin_memory=True)
        cudart_copy(Xh.data_ptr(), xb.devptr(), 8 * n * d, 2)
        cudart_copy(yh.data_ptr(), yb.devptr(), 8 * n, 2)
        wh = torch.empty(d, dtype=torch.float64, pin_memory=True)
        lh = torch.empty(1, dtype=torch.float64, pin_memory=True)
        from amcuda.realize import device_buffer_of
        wbuf = device_buffer_of(tr.w)
        sp = C.c_void_p(sptr)

        def step():
            A.call("amc_buf_upload_async", xb.handle, C.c_void_p(Xh.data_ptr()), 8 * n * d, 0, sp)
            A.call("amc_buf_upload_async", yb.handle, C.c_void_p(yh.data_ptr()), 8 * n, 0, sp)
            tr.step()
            A.call("amc_buf_download_async", wbuf.handle, C.c_void_p(wh.data_ptr()), 8 * d, 0, sp)
            A.call("amc_buf_download_async", tr._losses.handle, C.c_void_p(lh.data_ptr()), 8, 8 * (tr.steps - 1), sp)
        n_e = 4
        e_ms = max_over_ranks(ws, time_e2e(step, n_e, stream))
        e2e = {"value": ws * work * n_e / (e_ms / 1e3) / 1e9, "unit": "GB/s", "h2d_bytes_per_step": 8 * n * d + 8 * n,
               "d2h_bytes_per_step": 8 * d + 8, "steps": n_e,
               "path": "X and y uploaded from pinned memory into the program's constants (amc_buf_upload_async), "
                       "one ssa-realize/ctx replay + gradient step, w and the loss read back, one stream"}
        del Xh, yh
    losses = tr.losses()
    cpu = cpu_other("linreg", "f64") if rank == 0 and ws == 1 and not args.no_cpu else None
    traffic, tsrc = traffic_of("linreg")
    out = entry(_METRIC["linreg"], ws * work * steps / (t / 1e3) / 1e9, "GB/s", t / steps, steps, "f64",
                other_config("linreg", args),
                {"bound": "hbm", "kernel": "k_gemv_pair_tma<double,8,3> (the GEMV pair with the loss folded in) + its partial sums",
                 "achieved": per, "peak": hbm, "unit": "GB/s", "frac": per / hbm, "traffic": traffic,
                 "traffic_source": tsrc, "peak_source": kind + " hbm_gbs (a copy: read + write)",
                 "algorithmic_bytes_per_step": work},
                cpu, e2e, replay_launches * steps, clocks, scaling="weak",
                direct_kernel=direct, loss_first=float(losses[0]), loss_last=float(losses[-1]),
                steps_trained=int(tr.steps), blas=blas_lines(args, Xm, n, d, stream, local, ws, hbm))
    close_rank_sum(rank_sum)
    del tr, Xm, ym, xb, yb
    _release()
    return out


def blas_lines(args, Xm, n, d, stream, local, ws, hbm):
    """morph-matvec X w, morph-matvec X^T r and morph-dot over the config-5 X
    (blas-exec.scm:260-310) through realize plans, each timed alone on the
    device-resident X (larger than L2).  GB/s of the algorithmic bytes: X
    once, plus the vectors."""
    import amcuda as am
    from amcuda import workloads as W
    sptr = stream.cuda_stream
    w = am.morph_from_numpy(W.normal(W.seed_of(6, 0), d), "f64")
    r = am.morph_from_numpy(W.normal(W.seed_of(6, 1), n), "f64")
    flat = am.morph_reshape(Xm, (n * d,))
    half = n * d // 2
    v1 = am.morph_slice(flat, (0,), (half,))
    v2 = am.morph_slice(flat, (half,), (2 * half,))
    cases = {
        "matvec": (am.morph_matvec(Xm, w), n * d * 8 + d * 8 + n * 8, f"X w, X {n} x {d} f64"),
        "matvec_t": (am.morph_matvec(am.morph_transpose(Xm), r), n * d * 8 + n * 8 + d * 8,
                     f"X^T r, X {n} x {d} f64 (a transposed view)"),
        "dot": (am.morph_dot(v1, v2), 2 * half * 8 + 8, f"dot of the two halves of X ({half} f64 each)"),
    }
    out = {}
    for name, (tree, work, what) in cases.items():
        plan = am.Plan(tree)
        ms, steps, _ = time_steps(lambda: plan.execute(sptr), args.steps, args.warmup, stream, local, ws)
        t = max_over_ranks(ws, sum(ms) / len(ms))
        value = work / (t / 1e3) / 1e9
        out[name] = {"what": what, "value": value, "unit": "GB/s", "ms_per_step": t, "steps": steps,
                     "frac_of_hbm": value / hbm, "launches_per_step": plan.stats()["launches"],
                     "algorithmic_bytes": work}
        del plan
    return out


PC_FUNCS = {"fused": pc_fused, "conv": pc_conv, "attention": pc_attention, "linreg": pc_linreg}


def bench_one(args, ws, rank, local, wl, dtype):
    import amcuda as am
    import torch
    am.init(local)
    torch.cuda.set_device(local)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    if wl == "fused":
        return pc_fused(args, ws, rank, local, dtype)
    return PC_FUNCS[wl](args, ws, rank, local)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="amcuda", choices=["amcuda", "reference"])
    ap.add_argument("--workload", default="all", choices=["all", "filterbank", "fused", "linreg", "attention", "conv"])
    ap.add_argument("--signals", type=int, default=64)
    ap.add_argument("--samples", type=int, default=1 << 24)
    ap.add_argument("--rows", type=int, default=1 << 22)
    ap.add_argument("--batch", type=int, default=None,
                    help="per-GPU batch: default 16 (attention, config 4) or 64 (conv, config 3)")
    ap.add_argument("--dtype", default="f64", help="config 1's dtype with --workload fused")
    ap.add_argument("--no-cold", action="store_true", help="skip config 1's cold-input (rotated copies) timing")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-per-config", action="store_true", help="the headline alone")
    ap.add_argument("--ref-procs", type=int, default=None,
                    help="processes of the reference arm (default: one per host core)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl != "reference" else args.warmup
    ws, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            reference_arm(args, ws, rank)
        elif args.workload in ("all", "filterbank"):
            out = bench_filterbank(args, ws, rank, local)
            if args.workload == "all" and not args.no_per_config:
                import torch
                stream = torch.cuda.Stream()
                torch.cuda.set_stream(stream)
                per = {}
                for name, wl, dt in PER_CONFIG:
                    per[name] = pc_fused(args, ws, rank, local, dt) if wl == "fused" else PC_FUNCS[wl](args, ws, rank,
                                                                                                     local)
                    _release()
                out["per_config"] = per
            if rank == 0:
                print(json.dumps(out))
        else:
            e = bench_one(args, ws, rank, local, args.workload, args.dtype)
            if rank == 0:
                e.update({"n_gpus": ws, "warmup": args.warmup, "higher_is_better": True, "vs_baseline": None,
                          "data": "synthetic"})
                print(json.dumps(e))
    finally:
        if ws > 1 and args.impl != "reference":
            import torch.distributed as dist
            if dist.is_initialized():
                dist.destroy_process_group()


if __name__ == "__main__":
    main()
