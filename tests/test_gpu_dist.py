"""The fixed-order sum over GPUs through peer memory (amc_peer_sum), on 2
GPUs of one node as two processes.  Skipped when fewer than 2 GPUs are
visible.  Each rank's vectors come from a seeded generator, so every rank
knows the expected result: the rank-order sum accumulated in double, stored
in the vector's dtype, bit for bit and identical on both ranks.  A second
case makes one rank skip a sum: the other's bounded wait runs out and the
library reports AMC_ERR_TIMEOUT, with no fault and the context still
usable."""
import os
import socket
import sys
from pathlib import Path

import numpy as np
import pytest

pytestmark = pytest.mark.gpu
ROOT = Path(__file__).resolve().parents[1]


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _vec(rank, n, dt, k):
    return np.random.default_rng(1000 * k + rank).standard_normal(n).astype(dt)


def _worker(rank, world, port, mode, q):
    sys.path.insert(0, str(ROOT / "array-morphisms_b200"))
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
    import datetime
    import torch
    import torch.distributed as dist
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", rank=rank, world_size=world, timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    try:
        import amcuda as am
        from amcuda import _abi as A
        from amcuda.dist import PeerSum
        am.init(rank)
        ps = PeerSum(1 << 16)
        results = []
        if mode == "sum":
            cases = [(36864, np.float32), (257, np.float64), (1, np.float64), (65536, np.float32), (65536, np.float64)]
            for k, (n, dt) in enumerate(cases * 2):
                t = torch.from_numpy(_vec(rank, n, dt, k)).cuda()
                ps.sum_(t)
                torch.cuda.synchronize()
                A.check(A.load().amc_synchronize())
                ref = np.zeros(n)
                for r in range(world):
                    ref = ref + _vec(r, n, dt, k).astype(np.float64)
                results.append(bool(np.array_equal(t.cpu().numpy(), ref.astype(dt))))
        else:
            # rank 1 skips this sum: rank 0's wait must give up and report it
            t = torch.ones(1024, dtype=torch.float64, device="cuda")
            rc = 0
            if rank == 0:
                ps.sum_(t)
                torch.cuda.synchronize()
                rc = A.load().amc_synchronize()
            results.append(rc)
            # the context still works afterwards
            x = torch.arange(8, dtype=torch.float64, device="cuda")
            results.append(float(x.sum().item()))
        ps.close()
        q.put((rank, results))
    finally:
        dist.destroy_process_group()


def _run(mode):
    import torch
    import torch.multiprocessing as mp
    if torch.cuda.device_count() < 2:
        pytest.skip("needs 2 GPUs")
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _port()
    ps = [ctx.Process(target=_worker, args=(r, 2, port, mode, q)) for r in range(2)]
    for p in ps:
        p.start()
    out = dict(q.get(timeout=300) for _ in ps)
    for p in ps:
        p.join(timeout=120)
        assert p.exitcode == 0
    return out


def test_peer_sum_is_the_rank_order_sum_on_every_rank():
    out = _run("sum")
    assert all(out[0]) and all(out[1]), out


def test_peer_sum_wait_gives_up_when_a_rank_never_arrives():
    out = _run("timeout")
    assert out[0][0] == 7, out      # AMC_ERR_TIMEOUT on the waiting rank
    assert out[0][1] == 28.0 and out[1][1] == 28.0
