"""Benchmark of the realize hot path on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl amcuda|reference]
                    [--workload filterbank|fused|linreg|attention|conv]

Default workload: the polyphase filter bank (config 2 of the five) realized
through the public API: 64 signals of 2^24 f32 samples per GPU, 64 branches x
16 taps, the im2col -> reshape -> transpose -> product -> tap-sum tree.  One
step = one realize of that tree on device-resident inputs.  Multi-GPU runs one
process per GPU (torchrun); each rank realizes its own 64 signals (weak
scaling, no data-path collective); time is the max over ranks.

Prints ONE JSON line (rank 0).  `value` is algorithmic HBM GB/s of the whole
job; `e2e` is the same metric with the host->device upload of every step's
signals from pinned memory and the device->host read of its result inside
the timed region.
"""
from __future__ import annotations

import argparse
import json
import math
import multiprocessing as mp
import os
import re
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT / "array-morphisms_b200"))

HBM_FALLBACK = 6650.0
TF32_NOMINAL = 1125.0  # dense TF32 TFLOP/s (half the dense bf16 nominal), used when no measurement exists


def peaks():
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        d = json.loads(p.read_text())
        return float(d.get("hbm_gbs", HBM_FALLBACK)), float(d.get("bf16_tflops", 1590.0)), "measured"
    return HBM_FALLBACK, 1590.0, "fallback"


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
    """SM clock and clock-event (throttle) reasons sampled during the timed
    region: NVML every 2 ms on a thread (short regions get samples too), or
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
            time.sleep(0.002)

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

    def stop(self):
        if self.h is not None:
            self.run = False
            self.t.join(timeout=2)
            sm = sorted(self.samples)
            reasons = sorted(n for n, bit in self.REASONS if self.mask & bit)
            return {"sm_mhz": sm[len(sm) // 2] if sm else None, "sm_max_mhz": self.mx, "reasons": reasons,
                    "samples": len(sm), "source": "nvml"}
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
def _oracle_filterbank_sample(args):
    """One oracle realize of the filter-bank tree on a signal sample; returns
    (seconds, algorithmic bytes)."""
    sig, length = args
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np
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


def cpu_filterbank(n_procs: int, length: int, signals: int):
    """Oracle on `signals` signal samples over n_procs spawned processes."""
    jobs = [(s, length) for s in range(signals)]
    t0 = time.perf_counter()
    if n_procs == 1:
        res = [_oracle_filterbank_sample(j) for j in jobs]
    else:
        with mp.get_context("spawn").Pool(n_procs) as pool:
            res = pool.map(_oracle_filterbank_sample, jobs)
    wall = time.perf_counter() - t0
    by = sum(r[1] for r in res)
    return by / wall / 1e9, wall


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


def cpu_other(wl: str, dtype: str):
    """The oracle port of the reference's CPU path, timed on a bounded sample
    of the workload on one host thread: (value, unit, sample)."""
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np
    import oracle
    from amcuda import morph as M
    from amcuda import workloads as W
    if wl == "fused":
        xm, ym = W.c1_inputs_morph(dtype)
        tree = W.c1_tree(xm, ym)
        esz = 8 if dtype == "f64" else 4
        t = _timed(lambda: oracle.realize(tree))
        return ((2 * (1 << 19) + 1024) * esz / t / 1e9, "GB/s",
                f"the whole config-1 tree ({dtype}), per-node realize with materialised map and add nodes, 1 thread")
    if wl == "linreg":
        rows, d = 1 << 15, 256
        X, y, _ = W.c5_inputs(rows, d)
        t = _timed(lambda: oracle.linreg(X, y, np.zeros(d), 1, 0.1))
        return (rows * (d + 1) * 8 / t / 1e9, "GB/s",
                f"{rows} of the 2^22 rows, one step of the SSA replay (GEMV, residual, strided GEMM), 1 thread")
    if wl == "attention":
        n, dh = 2048, 64
        q, k, v, do = (W.normal(W.seed_of(4, j), n * dh).astype(np.float32).reshape(1, n, dh) for j in range(4))
        tree = M.attention_morphism(M.morph_from_numpy(q), M.morph_from_numpy(k), M.morph_from_numpy(v), 0.125)

        def run():
            oracle.realize(tree)
            oracle.attention_bwd(q, k, v, do, 0.125)
        t = _timed(run)
        return (12.0 * n * n * dh / t / 1e12, "TFLOP/s",
                "1 of the 256 (batch, head) blocks: the %attn-2d! restatement forward and a double-precision VJP, 1 thread")
    if wl == "conv":
        x = W.normal(W.seed_of(3, 0), 64 * 56 * 56).astype(np.float32).reshape(1, 64, 56, 56)
        w = (W.normal(W.seed_of(3, 1), 64 * 64 * 9) * np.sqrt(2 / 576)).astype(np.float32).reshape(64, 64, 3, 3)
        dy = W.normal(W.seed_of(3, 2), 64 * 56 * 56).astype(np.float32).reshape(1, 64, 56, 56)

        def run():
            oracle.conv2d_fwd(x, w)
            oracle.conv2d_dgrad(dy, w, x.shape)
            oracle.conv2d_wgrad(x, dy, w.shape)
        t = _timed(run)
        return (3 * 2.0 * 64 * 64 * 9 * 56 * 56 / t / 1e12, "TFLOP/s",
                "1 of the 64 images: im2col + double-accumulating GEMM forward, col2im data gradient, weight gradient, 1 thread")
    return None


def _oracle_other_sample(job):
    """One bounded unit of a non-default workload through the oracle port of
    the reference's CPU path: the whole config-1 tree, 2^15 rows of one
    linear-regression step, one (batch, head) attention block forward and
    backward, or one conv image's three passes.  Returns (seconds, work) with
    work in the GPU arm's unit (bytes or FLOPs)."""
    wl, dtype = job
    sys.path.insert(0, str(ROOT / "oracle"))
    import numpy as np
    import oracle
    from amcuda import morph as M
    from amcuda import workloads as W
    oracle.lib()
    if wl == "fused":
        xm, ym = W.c1_inputs_morph(dtype)
        tree = W.c1_tree(xm, ym)
        run, work = (lambda: oracle.realize(tree)), (2 * (1 << 19) + 1024) * (8 if dtype == "f64" else 4)
    elif wl == "linreg":
        rows, d = 1 << 15, 256
        X, y, _ = W.c5_inputs(rows, d)
        run, work = (lambda: oracle.linreg(X, y, np.zeros(d), 1, 0.1)), rows * (d + 1) * 8
    elif wl == "attention":
        n, dh = 2048, 64
        q, k, v, do = (W.normal(W.seed_of(4, j), n * dh).astype(np.float32).reshape(1, n, dh) for j in range(4))
        tree = M.attention_morphism(M.morph_from_numpy(q), M.morph_from_numpy(k), M.morph_from_numpy(v), 0.125)

        def run():
            oracle.realize(tree)
            oracle.attention_bwd(q, k, v, do, 0.125)
        work = 12.0 * n * n * dh
    else:
        x = W.normal(W.seed_of(3, 0), 64 * 56 * 56).astype(np.float32).reshape(1, 64, 56, 56)
        w = (W.normal(W.seed_of(3, 1), 64 * 64 * 9) * np.sqrt(2 / 576)).astype(np.float32).reshape(64, 64, 3, 3)
        dy = W.normal(W.seed_of(3, 2), 64 * 56 * 56).astype(np.float32).reshape(1, 64, 56, 56)

        def run():
            oracle.conv2d_fwd(x, w)
            oracle.conv2d_dgrad(dy, w, x.shape)
            oracle.conv2d_wgrad(x, dy, w.shape)
        work = 3 * 2.0 * 64 * 64 * 9 * 56 * 56
    t0 = time.perf_counter()
    run()
    return time.perf_counter() - t0, work


_OTHER_ARM = {
    "fused": ("GB/s", 1e9, "the whole config-1 tree ({dtype}) per process per step"),
    "linreg": ("GB/s", 1e9, "2^15 of the 2^22 rows of one step per process per step"),
    "attention": ("TFLOP/s", 1e12, "1 of the 256 (batch, head) blocks, forward and backward, per process per step"),
    "conv": ("TFLOP/s", 1e12, "1 of the 64 images, three passes, per process per step"),
}
_OTHER_METRIC = {
    "fused": "fused view+map+reduce realize GB/s ({dtype})",
    "linreg": "linear-regression step (fused pass over X) GB/s",
    "attention": "attention forward + backward TFLOP/s",
    "conv": "conv2d forward + data gradient + weight gradient TFLOP/s",
}


def other_config(wl: str, args) -> dict:
    """The `config` of a non-default workload's bench line (both arms)."""
    if wl == "fused":
        return {"workload": f"config 1: x,y 2^20 {args.dtype}, reshape 1024x1024, transpose, slice step 2, "
                            f"sum(x^2+y) over axis 1", "l2": "256 MB flush between steps"}
    if wl == "linreg":
        return {"workload": f"config 5: X {args.rows} x 256 f64 per GPU, MSE gradient step, lr 0.1",
                "l2": "X larger than L2"}
    if wl == "attention":
        return {"workload": f"config 4: Q,K,V,dO ({args.batch or 16},16,2048,64) f32, scale 1/8; O, dQ, dK, dV per step",
                "flops": "algorithmic 12*B*H*S^2*D (6 GEMMs; the backward recomputes S and dP twice more)"}
    return {"workload": f"config 3: x ({args.batch or 64},64,56,56) f32, w (64,64,3,3), stride 1 pad 1; "
                        f"Y, dX and dW per step"}


def reference_arm_other(args, cores):
    """The reference arm of the non-default workloads: the oracle port on
    every host core (one spawned process per core, each running the bounded
    unit above), whole-job work over the wall time of each step."""
    wl = args.workload
    unit, scale, what = _OTHER_ARM[wl]
    dtype = args.dtype if wl == "fused" else ("f64" if wl == "linreg" else "f32")
    jobs = [(wl, args.dtype)] * cores
    times, vals = [], []
    with mp.get_context("spawn").Pool(cores) as pool:
        for i in range(args.warmup + args.steps):
            res = pool.map(_oracle_other_sample, jobs)
            # the processes run their units side by side: the step takes the
            # longest one (input generation and process start-up excluded)
            dt = max(r[0] for r in res)
            if i >= args.warmup:
                times.append(dt)
                vals.append(sum(r[1] for r in res) / dt / scale)
    value = sum(vals) / len(vals)
    sample = (what.format(dtype=args.dtype) + f", {cores} spawned processes running side by side, step time = the "
              f"longest process, oracle port of the reference's CPU path")
    print(json.dumps({
        "impl": "reference", "metric": _OTHER_METRIC[wl].format(dtype=args.dtype), "value": value, "unit": unit,
        "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * sum(times) / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": dtype, "data": "synthetic",
        "config": dict(other_config(wl, args), sample=sample),
        "cpu_baseline": {"value": value, "unit": unit, "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": unit, "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


def reference_arm(args, ws, rank):
    if rank != 0:
        return
    cores = args.ref_procs or os.cpu_count() or 1
    if args.workload != "filterbank":
        reference_arm_other(args, cores)
        return
    length = 1 << 20
    signals = cores
    # warm-up (spawn + oracle build) then timed steps
    times, vals = [], []
    with mp.get_context("spawn").Pool(cores) as pool:
        pool.map(_oracle_filterbank_sample, [(s, 1 << 14) for s in range(cores)])
        for i in range(args.warmup + args.steps):
            t0 = time.perf_counter()
            res = pool.map(_oracle_filterbank_sample, [(s, length) for s in range(signals)])
            dt = time.perf_counter() - t0
            if i >= args.warmup:
                times.append(dt)
                vals.append(sum(r[1] for r in res) / dt / 1e9)
    value = sum(vals) / len(vals)
    sample = (f"{signals} signals x 2^20 samples per step (of the 64 x 2^24 workload), oracle port of the "
              f"reference's per-node realize, one spawned process per host core")
    print(json.dumps({
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000 * sum(times) / len(times),
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": dict(CONFIG_FB, sample=sample),
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }))


METRIC = "fused realize() HBM GB/s (polyphase filter bank)"
CONFIG_FB = {"workload": "polyphase filter bank: 64 signals x 2^24 f32 per GPU, 64 branches x 16 taps, "
                         "1024-tap Hamming sinc prototype (cutoff 1/64), frames 262129",
             "signals_per_gpu": 64, "samples": 1 << 24, "branches": 64, "taps": 16,
             "l2": "inputs (4 GiB per GPU) larger than L2; no flush needed", "parallelism": "batch-sharded, weak"}


# ---------------------------------------------------------------------------- GPU arm: filter bank
def bench_filterbank(args, ws, rank, local):
    import numpy as np
    import torch
    import amcuda as am
    from amcuda import workloads as W
    from amcuda.dist import allreduce_fixed_order
    am.init(local)
    torch.cuda.set_device(local)
    B, L = args.signals, args.samples
    F = W.c2_frames(L)
    x_t = W.c2_signals_torch(B, L, device="cuda", first=rank * B)
    h_t = torch.from_numpy(W.c2_prototype()).cuda()
    # leaves wrap the device tensors (no copy); the tree is the public API's
    xb = am.DeviceBuffer.create("f32", B * L)
    hb = am.DeviceBuffer.create("f32", h_t.numel())
    torch.cuda.synchronize()
    import ctypes as C
    from amcuda import _abi as A
    A.call("amc_buf_upload", hb.handle, C.c_void_p(h_t.cpu().numpy().ctypes.data), 4 * h_t.numel(), 0)
    # copy the generated signals into the library's buffer (device to device)
    xptr = xb.devptr()
    cudart_copy(xptr, x_t.data_ptr(), 4 * B * L)
    del x_t
    torch.cuda.empty_cache()
    xm = am.Concrete(None, (B, L), dtype="f32", dev=xb)
    hm = am.Concrete(None, (W.PROTO,), dtype="f32", dev=hb)
    plan = am.Plan(W.c2_tree(xm, hm))
    st = plan.stats()
    torch.cuda.synchronize()
    stream = torch.cuda.Stream()  # an explicit stream: events and launches share it
    torch.cuda.set_stream(stream)
    sptr = stream.cuda_stream
    for _ in range(args.warmup):
        plan.execute(sptr)
    torch.cuda.synchronize()
    barrier(ws)
    clk = Clocks(local)
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    per = []
    torch.cuda.synchronize()
    t_all0 = torch.cuda.Event(enable_timing=True)
    t_all1 = torch.cuda.Event(enable_timing=True)
    t_all0.record(stream)
    for _ in range(args.steps):
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        plan.execute(sptr)
        b.record(stream)
        per.append((a, b))
    t_all1.record(stream)
    torch.cuda.synchronize()
    clocks = clk.stop()
    barrier(ws)
    total_ms = t_all0.elapsed_time(t_all1)
    step_ms = [a.elapsed_time(b) for a, b in per]
    total_ms = max_over_ranks(ws, total_ms)
    bytes_step = B * L * 4 + B * F * 64 * 4 + 4 * W.PROTO
    value = ws * bytes_step * args.steps / (total_ms / 1e3) / 1e9
    hbm, _, kind = peaks()
    mean_step = sum(step_ms) / len(step_ms)
    achieved = bytes_step / (mean_step / 1e3) / 1e9
    traffic = None

    # ---- end to end: pinned host signals -> device -> realize -> host result.
    # Two buffer sets (two plans of the same public tree) and three streams:
    # step k's upload, step k-1's realize and step k-2's download run at once,
    # so the two PCIe directions overlap each other and the kernel.  Every step
    # still moves its whole input in and its whole result out.
    e2e = None
    if not args.no_e2e:
        x_host = torch.empty((B, L), dtype=torch.float32, pin_memory=True)
        out_host = torch.empty((B, F, 64), dtype=torch.float32, pin_memory=True)
        cudart_copy_d2h(x_host.data_ptr(), xptr, 4 * B * L)
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
        del plan2, xb2

    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        v, wall = cpu_filterbank(1, 1 << 22, 1)
        cpu = {"value": v, "unit": "GB/s", "cores": 1, "kind": "port",
               "sample": f"1 signal x 2^22 samples through the oracle port of the reference's per-node realize "
                         f"(im2col, product and tap reduction materialised), 1 thread, {wall:.1f} s"}
    if rank == 0:
        out = {
            "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": ws, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": total_ms / args.steps, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f32", "data": "synthetic", "config": CONFIG_FB,
            "roofline": {"bound": "hbm", "kernel": "k_fir_tma (+ k_fir_tail)", "achieved": achieved, "peak": hbm,
                         "unit": "GB/s", "frac": achieved / hbm, "traffic": traffic,
                         "peak_source": f"{kind} (MEASURED_PEAKS.json hbm_gbs)" if kind == "measured" else kind,
                         "algorithmic_bytes_per_launch": bytes_step},
            "cpu_baseline": cpu, "e2e": e2e, "gpu_launches": st["launches"] * args.steps, "clocks": clocks,
        }
        print(json.dumps(out))


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


def cudart_copy(dst: int, src: int, nbytes: int):
    import ctypes as C
    rt = _cudart()
    rt.cudaMemcpy.restype = C.c_int
    rc = rt.cudaMemcpy(C.c_void_p(dst), C.c_void_p(src), C.c_size_t(nbytes), 3)  # device to device
    if rc:
        raise RuntimeError(f"cudaMemcpy failed {rc}")


def cudart_copy_d2h(dst: int, src: int, nbytes: int):
    import ctypes as C
    rt = _cudart()
    rt.cudaMemcpy.restype = C.c_int
    rc = rt.cudaMemcpy(C.c_void_p(dst), C.c_void_p(src), C.c_size_t(nbytes), 2)
    if rc:
        raise RuntimeError(f"cudaMemcpy failed {rc}")


# ---------------------------------------------------------------------------- other workloads (per-config measurement)
def bench_other(args, ws, rank, local):
    import numpy as np
    import torch
    import amcuda as am
    from amcuda import workloads as W
    from amcuda.dist import allreduce_fixed_order
    am.init(local)
    torch.cuda.set_device(local)
    stream = torch.cuda.Stream()
    torch.cuda.set_stream(stream)
    sptr = stream.cuda_stream
    hbm, bf16, kind = peaks()
    wl = args.workload
    if wl == "fused":
        xm, ym = W.c1_inputs_morph(args.dtype)
        plan = am.Plan(W.c1_tree(xm, ym))
        run = lambda: plan.execute(sptr)
        esz = 8 if args.dtype == "f64" else 4
        work = 2 * (1 << 19) * esz + 1024 * esz
        unit, bound, metric = "GB/s", "hbm", f"fused view+map+reduce realize GB/s ({args.dtype})"
        flush = torch.empty(256 << 20, dtype=torch.uint8, device="cuda")
        pre = lambda: flush.fill_(1)
        cfg = other_config(wl, args)
        launches = plan.stats()["launches"]
    elif wl == "linreg":
        n, d = args.rows, 256
        X, y, _ = W.c5_inputs_torch(n, d)
        w = torch.zeros(d, dtype=torch.float64, device="cuda")
        npart = W.linreg_partials_count(n, d)
        part = torch.empty(npart * (d + 1), dtype=torch.float64, device="cuda")
        gl = torch.empty(d + 1, dtype=torch.float64, device="cuda")
        loss = torch.empty(1, dtype=torch.float64, device="cuda")
        N_total = n * ws

        def run():
            W.linreg_partials(X, y, w, part, N_total)
            W.linreg_reduce(part, npart, d, gl)
            if ws > 1:
                # the grad+loss row crosses the row shards: rank-ordered all-reduce
                allreduce_fixed_order(gl)
            W.linreg_update(w, gl, N_total, 0.1, loss)
        work = n * d * 8 + n * 8
        unit, bound, metric = "GB/s", "hbm", "linear-regression step (fused pass over X) GB/s"
        pre = lambda: None
        cfg = other_config(wl, args)
        launches = 3
    elif wl == "attention":
        B, H, S, D = args.batch or 16, 16, 2048, 64
        q, k, v = (torch.from_numpy(W.normal(W.seed_of(4, j), B * H * S * D).astype(np.float32)).cuda().view(B, H, S, D)
                   for j in range(3))
        do = torch.from_numpy(W.normal(W.seed_of(4, 3), B * H * S * D).astype(np.float32)).cuda().view(B, H, S, D)
        o = torch.empty_like(q)
        lse = torch.empty((B, H, S), dtype=torch.float32, device="cuda")
        dq, dk, dv = torch.empty_like(q), torch.empty_like(k), torch.empty_like(v)

        def run():
            W.attention_fwd(q, k, v, o, lse, 1.0 / 8.0)
            W.attention_bwd(q, k, v, o, do, lse, dq, dk, dv, 1.0 / 8.0)
        # algorithmic: forward 2 GEMMs (Q K^T, P V), backward 4 (dV, dP, dQ, dK)
        work = 12.0 * B * H * S * S * D
        unit, bound, metric = "TFLOP/s", "tensor", "attention forward + backward TFLOP/s"
        pre = lambda: None
        cfg = other_config(wl, args)
        launches = 6   # forward: V^T, K rounding, kernel; backward: pre-pass, dK/dV, dQ
    elif wl == "conv":
        N = args.batch or 64
        x = torch.from_numpy(W.normal(W.seed_of(3, 0), N * 64 * 56 * 56).astype(np.float32)).cuda().view(N, 64, 56, 56)
        wt = torch.from_numpy((W.normal(W.seed_of(3, 1), 64 * 64 * 9) * math.sqrt(2 / 576)).astype(np.float32)).cuda().view(64, 64, 3, 3)
        dy = torch.from_numpy(W.normal(W.seed_of(3, 2), N * 64 * 56 * 56).astype(np.float32)).cuda().view(N, 64, 56, 56)
        yy, dx, dw = torch.empty_like(x), torch.empty_like(x), torch.empty_like(wt)

        def run():
            W.conv2d_fwd(x, wt, yy)
            W.conv2d_dgrad(dy, wt, dx)
            W.conv2d_wgrad(x, dy, dw)
            if ws > 1:
                # dW sums over the batch shards: fixed-order all-reduce.  It is
                # not overlapped with the next pass: NCCL's kernel would hold SMs
                # that the one-CTA-per-SM conv kernels wait for (measured slower).
                allreduce_fixed_order(dw)
        work = 3 * 2.0 * N * 64 * 64 * 9 * 56 * 56
        unit, bound, metric = "TFLOP/s", "tensor", "conv2d forward + data gradient + weight gradient TFLOP/s"
        pre = lambda: None
        cfg = other_config(wl, args)
        launches = 6   # 2 x (weights, kernel) + weight-gradient kernel + reduce
    else:
        raise SystemExit(f"unknown workload {wl}")
    for _ in range(args.warmup):
        pre()
        run()
    torch.cuda.synchronize()
    barrier(ws)
    clk = Clocks(local)
    # Steps are enqueued back to back; each step's events bracket its own work
    # on the stream.  The L2 flush (where there is one) runs between them, so
    # the host's launch latency overlaps device work instead of being timed.
    evs = []
    for _ in range(args.steps):
        pre()
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record(stream)
        run()
        b.record(stream)
        evs.append((a, b))
    torch.cuda.synchronize()
    ms = [a.elapsed_time(b) for a, b in evs]
    clocks = clk.stop()
    t = max_over_ranks(ws, sum(ms))
    per = work / (sum(ms) / len(ms) / 1e3)
    cpu = None
    if rank == 0 and ws == 1 and not args.no_cpu:
        r = cpu_other(wl, args.dtype)
        if r:
            cpu = {"value": r[0], "unit": r[1], "cores": 1, "kind": "port", "sample": r[2]}
    scale = 1e9 if unit == "GB/s" else 1e12
    if bound == "hbm":
        peak, peak_source = hbm, kind + " hbm_gbs"
    else:
        # TF32 denominator measured now, on this GPU, by the library's tcgen05 probe
        peak = W.tc_peak_tf32(4000)
        peak_source = (f"tcgen05 kind::tf32 M=128 N=256 issue loop on this GPU (amc_tc_peak_tf32); "
                       f"{kind} bf16/2 = {bf16 / 2.0:.1f} for context")
    if rank == 0:
        print(json.dumps({
            "metric": metric, "value": ws * work * args.steps / (t / 1e3) / scale, "unit": unit, "n_gpus": ws,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": t / args.steps, "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": args.dtype if wl == "fused" else ("f64" if wl == "linreg" else "f32"),
            "data": "synthetic", "config": cfg,
            "roofline": {"bound": bound, "achieved": per / scale, "peak": peak, "unit": unit, "frac": per / scale / peak,
                         "traffic": None,
                         "peak_source": peak_source},
            "cpu_baseline": cpu, "gpu_launches": launches * args.steps, "clocks": clocks}))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=20)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", default="amcuda", choices=["amcuda", "reference"])
    ap.add_argument("--workload", default="filterbank", choices=["filterbank", "fused", "linreg", "attention", "conv"])
    ap.add_argument("--signals", type=int, default=64)
    ap.add_argument("--samples", type=int, default=1 << 24)
    ap.add_argument("--rows", type=int, default=1 << 22)
    ap.add_argument("--batch", type=int, default=None,
                    help="per-GPU batch: default 16 (attention, config 4) or 64 (conv, config 3)")
    ap.add_argument("--dtype", default="f64")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--ref-procs", type=int, default=None,
                    help="processes of the reference arm (default: one per host core)")
    args = ap.parse_args()
    args.warmup = max(args.warmup, 3) if args.impl != "reference" else args.warmup
    ws, rank, local = dist_setup(args)
    try:
        if args.impl == "reference":
            reference_arm(args, ws, rank)
        elif args.workload == "filterbank":
            bench_filterbank(args, ws, rank, local)
        else:
            bench_other(args, ws, rank, local)
    finally:
        if ws > 1 and args.impl != "reference":
            import torch.distributed as dist
            if dist.is_initialized():
                dist.destroy_process_group()


if __name__ == "__main__":
    main()
