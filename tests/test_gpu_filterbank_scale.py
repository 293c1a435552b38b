"""The filter-bank kernel (k_fir_tma, the bench kernel) pinned to the oracle
at the scales it runs: several 256-frame chunks per signal, and the full
config-2 workload, 64 signals x 2^24 samples, through the public plan.

At full size the oracle cannot realize the whole tree in test time, so
sampled (signal, frame) rows are checked: a frame depends only on its own
1024-sample window, so the oracle realizes the same tree on that window
alone (one frame) and the device's row must equal it bit for bit.  The
samples include the first and last frames and both sides of chunk
boundaries."""
import ctypes as C

import numpy as np
import pytest

import oracle

pytestmark = pytest.mark.gpu


def test_fir_tma_multichunk_matches_oracle(amc):
    """2 signals x 2^18 samples: 4081 frames, 16 chunks per signal, realized
    by the planner's filter-bank lowering; bit-exact against the oracle."""
    from amcuda import workloads as W
    L = 1 << 18
    x = np.stack([W.c2_signal(s, L) for s in range(2)])
    h = W.c2_prototype()
    plan = amc.Plan(W.c2_tree(amc.morph_from_numpy(x), amc.morph_from_numpy(h)))
    plan.execute()
    got = plan.result().values()
    ref = oracle.realize(W.c2_tree(amc.morph_from_numpy(x), amc.morph_from_numpy(h))).values()
    assert got.shape == ref.shape == (2, W.c2_frames(L), 64)
    np.testing.assert_array_equal(got.view(np.uint32), ref.view(np.uint32))


def test_fir_full_size_sampled_rows_match_oracle(amc):
    import torch
    from amcuda import _abi as A
    from amcuda import workloads as W
    B, L = 64, 1 << 24
    F = W.c2_frames(L)
    x_t = W.c2_signals_torch(B, L, device="cuda")
    xb = amc.DeviceBuffer.create("f32", B * L)
    torch.cuda.synchronize()
    src = torch.as_tensor(_CudaView(xb.devptr(), B * L), device="cuda")
    src.copy_(x_t.view(-1))
    torch.cuda.synchronize()
    del x_t
    torch.cuda.empty_cache()
    h = W.c2_prototype()
    xm = amc.Concrete(None, (B, L), dtype="f32", dev=xb)
    plan = amc.Plan(W.c2_tree(xm, amc.morph_from_numpy(h)))
    plan.execute()
    out = plan.result()._dev
    rng = np.random.default_rng(2024)
    frames = [0, 1, 255, 256, 257, 511, 512, F - 257, F - 256, F - 2, F - 1]
    samples = [(int(rng.integers(B)), f) for f in frames] + [(int(rng.integers(B)), int(rng.integers(F)))
                                                             for _ in range(120)]
    row = np.empty(64, dtype=np.float32)
    win = np.empty(1024, dtype=np.float32)
    for s, f in samples:
        A.check(A.load().amc_buf_download(out.handle, row.ctypes.data_as(C.c_void_p), 256, 4 * (s * F + f) * 64))
        A.check(A.load().amc_buf_download(xb.handle, win.ctypes.data_as(C.c_void_p), 4096, 4 * (s * L + 64 * f)))
        ref = oracle.realize(W.c2_tree(amc.morph_from_numpy(win[None, :].copy()), amc.morph_from_numpy(h))).values()
        assert ref.shape == (1, 1, 64)
        np.testing.assert_array_equal(row.view(np.uint32), ref[0, 0].view(np.uint32), err_msg=f"signal {s} frame {f}")


class _CudaView:
    def __init__(self, ptr, n):
        self.__cuda_array_interface__ = {"shape": (n,), "typestr": "<f4", "data": (ptr, False), "version": 3}
