"""Multi-rank host logic on CPU: world_size 2 gloo ranks shard rows of the
linear-regression problem and combine with the fixed-order all-reduce; the
result must match the unsharded oracle.  Also checks shard_range."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

ROOT = Path(__file__).resolve().parents[1]


def test_shard_range_partitions():
    from amcuda.dist import shard_range
    for n in (0, 1, 7, 64, 1000):
        for world in (1, 2, 3, 8):
            spans = [shard_range(n, world, r) for r in range(world)]
            assert spans[0][0] == 0 and spans[-1][1] == n
            assert all(a[1] == b[0] for a, b in zip(spans, spans[1:]))
            assert max(s[1] - s[0] for s in spans) - min(s[1] - s[0] for s in spans) <= 1


def _free_port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _worker(rank, world, port, n, d, steps, lr, q):
    sys.path.insert(0, str(ROOT / "array-morphisms_b200"))
    import torch
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from amcuda import workloads as W
        from amcuda.dist import ShardedLinearRegression, shard_range
        X, y, _ = W.c5_inputs(n, d)
        a, b = shard_range(n, world, rank)
        Xl, yl = torch.from_numpy(X[a:b].copy()), torch.from_numpy(y[a:b].copy())

        def partials(X, y, w, n_total, out):  # host math of the device kernel's row fold
            r = X @ w - y
            dr = 2.0 * ((1.0 / n_total) * r)
            out[:-1] = X.T @ dr
            out[-1] = (r * r).sum()

        def update(w, gl, n_total, lr, loss):
            w -= lr * gl[:-1]
            loss[0] = gl[-1] / n_total

        m = ShardedLinearRegression(Xl, yl, n, lr, partials, update)
        losses = []
        for _ in range(steps):
            m.step()
            losses.append(float(m.loss[0]))
        q.put((rank, m.w.numpy().copy(), losses))
    finally:
        dist.destroy_process_group()


def test_sharded_linreg_matches_oracle_two_gloo_ranks():
    import multiprocessing as mp
    import oracle
    from amcuda import workloads as W
    n, d, steps, lr = 3001, 256, 5, 0.1
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, n, d, steps, lr, q)) for r in range(2)]
    for p in ps:
        p.start()
    res = [q.get(timeout=180) for _ in ps]
    for p in ps:
        p.join(timeout=60)
        assert p.exitcode == 0
    X, y, _ = W.c5_inputs(n, d)
    w_ref, l_ref = oracle.linreg(X, y, np.zeros(d), steps, lr)
    for rank, w, losses in res:
        np.testing.assert_allclose(w, w_ref, rtol=1e-12, atol=1e-14)
        np.testing.assert_allclose(losses, l_ref, rtol=1e-12)
    np.testing.assert_array_equal(res[0][1], res[1][1])  # replicas stay identical


def _async_worker(rank, world, port, out):
    import torch
    import torch.distributed as dist
    from amcuda.dist import allreduce_fixed_order
    dist.init_process_group("gloo", init_method=f"tcp://127.0.0.1:{port}", rank=rank, world_size=world)
    try:
        t = torch.arange(6, dtype=torch.float64) * (rank + 1)
        p = allreduce_fixed_order(t, async_op=True)
        p.wait()
        out[rank] = t.tolist()
    finally:
        dist.destroy_process_group()


def test_allreduce_async_matches_sum():
    """The started-then-waited form gives the same sum on every rank."""
    import multiprocessing as mp
    ctx = mp.get_context("spawn")
    port = _free_port()
    mgr = ctx.Manager()
    out = mgr.dict()
    ps = [ctx.Process(target=_async_worker, args=(r, 2, port, out)) for r in range(2)]
    for p in ps:
        p.start()
    for p in ps:
        p.join(60)
        assert p.exitcode == 0
    expect = [float(i * 3) for i in range(6)]
    assert out[0] == expect and out[1] == expect
