"""Batch-axis sharding across the GPUs of one node (one process per GPU).

The reference has one notion of parallelism, the batch axis of a morphism
(core.scm:247-269, batch-ops.scm:217-239).  Here batched work is partitioned
across ranks:
  - independent items (filter-bank signals, attention batch entries, conv
    images for Y and dX) need no exchange;
  - a reduction that crosses the batch axis (the linear-regression gradient,
    the conv weight gradient) is combined with a deterministic sum in rank
    order, so results do not depend on a collective's internal reduction
    order: PeerSum does it through NVLink peer memory in the library's own
    kernels; allreduce_fixed_order is the same sum over torch.distributed
    (an all-gather, then the rank-axis sum), for any backend.
"""
from __future__ import annotations

from typing import Callable


def shard_range(n: int, world: int, rank: int) -> tuple[int, int]:
    """Contiguous [start, stop) of n items for `rank` of `world` (sizes differ by at most 1)."""
    if world <= 0 or not 0 <= rank < world:
        raise ValueError("bad world/rank")
    base, extra = divmod(n, world)
    start = rank * base + min(rank, extra)
    return start, start + base + (1 if rank < extra else 0)


class PendingReduce:
    """An all-reduce started with async_op=True: wait() finishes it."""

    def __init__(self, t, buf, work):
        self.t, self.buf, self.work = t, buf, work

    def wait(self):
        if self.work is not None:
            self.work.wait()   # orders the current stream after the collective
            self.work = None
        self.t.copy_(self.buf.sum(dim=0).view_as(self.t))
        return self.t


def allreduce_fixed_order(t, group=None, async_op: bool = False):
    """In-place sum of `t` over ranks in a fixed order: one all-gather of every
    rank's copy into a (world, n) buffer, then one sum over the rank axis.
    The result does not depend on the collective's internal reduction order
    and is the same on every rank and every run.  With async_op=True the
    all-gather is only started and a PendingReduce is returned; its wait()
    orders the current stream after it and forms the sum, so independent work
    can run in between."""
    import torch
    import torch.distributed as dist
    world = dist.get_world_size(group)
    if world == 1:
        return PendingReduce(t, t.view(1, -1), None) if async_op else t
    flat = t.contiguous().view(-1)
    buf = torch.empty((world, flat.numel()), dtype=t.dtype, device=t.device)
    try:
        work = dist.all_gather_into_tensor(buf, flat, group=group, async_op=async_op)
    except (RuntimeError, NotImplementedError, AttributeError):
        work = dist.all_gather(list(buf.unbind(0)), flat, group=group, async_op=async_op)
    pending = PendingReduce(t, buf, work if async_op else None)
    return pending if async_op else pending.wait()


class PeerSum:
    """The fixed-order sum over the ranks of one node through NVLink peer
    memory (amc_peer_sum): each rank pushes its vector into every rank's
    memory and sums all ranks' copies in rank order on its own GPU, in one
    pair of launches and no NCCL call.  Ranks are added in rank order,
    accumulated in double, so the result is bit-identical on every rank and
    every run.  Needs one process per GPU
    on the same node with peer access between the GPUs; `max_elems` bounds
    the vectors (8-byte elements).  close() is collective."""

    def __init__(self, max_elems: int, group=None):
        import ctypes as C
        import torch.distributed as dist
        from . import _abi as A
        from .realize import _ensure_init
        _ensure_init()
        self.group = group
        self.rank, self.world = dist.get_rank(group), dist.get_world_size(group)
        h = C.c_uint64(0)
        handle = (C.c_char * 64)()
        A.call("amc_peer_group_create", self.rank, self.world, int(max_elems), C.byref(h), handle)
        self.handle = h.value
        handles = [None] * self.world
        dist.all_gather_object(handles, bytes(handle), group=group)
        blob = b"".join(handles)
        A.call("amc_peer_group_open", self.handle, C.c_char_p(blob))

    def sum_(self, t, stream=None):
        """In place: t <- sum over ranks, in rank order (f32 / f64 CUDA tensor)."""
        import ctypes as C
        import torch
        from . import _abi as A
        if not t.is_contiguous():
            raise ValueError("PeerSum: a contiguous tensor")
        dt = {torch.float32: A.F32, torch.float64: A.F64}[t.dtype]
        s = stream if stream is not None else torch.cuda.current_stream().cuda_stream
        A.call("amc_peer_sum", self.handle, C.c_void_p(t.data_ptr()), t.numel(), dt, C.c_void_p(t.data_ptr()),
               C.c_void_p(s))
        return t

    def close(self):
        import torch
        import torch.distributed as dist
        from . import _abi as A
        if self.handle:
            torch.cuda.synchronize()
            dist.barrier(group=self.group)   # no rank still pushes into a buffer about to be freed
            A.call("amc_peer_group_destroy", self.handle)
            self.handle = 0


class ShardedLinearRegression:
    """Gradient descent on rows sharded across ranks.

    Each step: every rank forms the (d+1) row of gradient sums and squared
    residual sum over its rows (partials_fn), the rows are all-reduced in rank
    order, and every rank applies the same update, so w stays replicated.
    partials_fn(X, y, w, n_total, out) fills `out` (d+1); update_fn(w, gl,
    n_total, lr, loss) applies w -= lr * gl[:d] and writes gl[d] / n_total to
    loss.  The defaults run the device kernels of libamcuda."""

    def __init__(self, X, y, n_total: int, lr: float, partials_fn: Callable | None = None,
                 update_fn: Callable | None = None, group=None):
        import torch
        self.X, self.y, self.n_total, self.lr, self.group = X, y, n_total, lr, group
        d = X.shape[1]
        self.w = torch.zeros(d, dtype=torch.float64, device=X.device)
        self.gl = torch.empty(d + 1, dtype=torch.float64, device=X.device)
        self.loss = torch.empty(1, dtype=torch.float64, device=X.device)
        if partials_fn is None:
            from . import workloads as W
            npart = W.linreg_partials_count(X.shape[0], d)
            part = torch.empty(npart * (d + 1), dtype=torch.float64, device=X.device)

            def partials_fn(X, y, w, n_total, out):
                W.linreg_partials(X, y, w, part, n_total)
                W.linreg_reduce(part, npart, d, out)
        if update_fn is None:
            from . import workloads as W

            def update_fn(w, gl, n_total, lr, loss):
                W.linreg_update(w, gl, n_total, lr, loss)
        self.partials_fn, self.update_fn = partials_fn, update_fn

    def step(self) -> None:
        self.partials_fn(self.X, self.y, self.w, self.n_total, self.gl)
        allreduce_fixed_order(self.gl, self.group)
        self.update_fn(self.w, self.gl, self.n_total, self.lr, self.loss)
