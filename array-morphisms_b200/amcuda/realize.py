"""realize / realize_ctx: serialize a morphism tree and run it on the device.

The reference's realize (realization.scm:92-115) walks the tree and runs
per-element loops on the host.  Here the walk only serializes the tree into
amc_node records (operands first, root last) and libamcuda lowers and runs
it; the result comes back as a Concrete whose device buffer is kept so that
later realizes reuse it without another upload.
"""
from __future__ import annotations

import ctypes as C
import threading

import numpy as np

from . import _abi as A
from .morph import DTYPES, NP_DTYPES, Concrete, Expr, Morphism, compute_strides, shape_size

_init_lock = threading.Lock()
_initialized: set[int] = set()


def init(device: int | None = None) -> int:
    """amc_init on `device` (default: torch's current device if torch has
    initialized CUDA, else 0)."""
    if device is None:
        device = 0
        try:
            import torch
            if torch.cuda.is_available() and torch.cuda.is_initialized():
                device = torch.cuda.current_device()
        except Exception:
            pass
    with _init_lock:
        A.call("amc_init", device)
        _initialized.add(device)
    return device


def _ensure_init() -> None:
    if not _initialized:
        init()


class DeviceBuffer:
    """One reference to a libamcuda buffer handle."""

    def __init__(self, handle: int, dtype: str, nelem: int):
        self.handle = handle
        self.dtype = dtype
        self.nelem = nelem

    @classmethod
    def create(cls, dtype: str, nelem: int) -> "DeviceBuffer":
        _ensure_init()
        h = C.c_uint64(0)
        A.call("amc_buf_create", DTYPES[dtype], int(nelem), C.byref(h))
        return cls(h.value, dtype, nelem)

    @classmethod
    def from_host(cls, arr: np.ndarray, dtype: str) -> "DeviceBuffer":
        a = np.ascontiguousarray(arr, dtype=NP_DTYPES[dtype])
        b = cls.create(dtype, a.size)
        if a.size:
            A.call("amc_buf_upload", b.handle, a.ctypes.data_as(C.c_void_p), a.nbytes, 0)
        return b

    def download(self) -> np.ndarray:
        out = np.empty(self.nelem, dtype=NP_DTYPES[self.dtype])
        if out.size:
            A.call("amc_buf_download", self.handle, out.ctypes.data_as(C.c_void_p), out.nbytes, 0)
        return out

    def devptr(self) -> int:
        p = C.c_void_p()
        A.call("amc_buf_devptr", self.handle, C.byref(p))
        return p.value or 0

    def __del__(self):
        try:
            if self.handle and A._lib is not None:
                A._lib.amc_buf_free(self.handle)
        except Exception:
            pass
        self.handle = 0


def device_buffer_of(m: Concrete) -> DeviceBuffer:
    """The device copy of a concrete array's typed vector (uploaded once)."""
    if m._dev is None:
        m._dev = DeviceBuffer.from_host(m.data, m.dtype)
    return m._dev


def _view(buf: DeviceBuffer, dtype, shape, strides, offset) -> A.View:
    v = A.View()
    v.buf = buf.handle
    v.dtype = DTYPES[dtype]
    v.rank = len(shape)
    for i, (s, st) in enumerate(zip(shape, strides)):
        v.shape[i] = s
        v.strides[i] = st
    v.offset = offset
    return v


def _fill_shape(nd: A.Node, shape) -> None:
    nd.rank = len(shape)
    if nd.rank > A.MAX_RANK:
        raise ValueError(f"rank {nd.rank} exceeds {A.MAX_RANK}")
    for i, s in enumerate(shape):
        nd.shape[i] = s


class Serialized:
    """amc_node records of one tree plus the ctypes objects they point to."""

    def __init__(self):
        self.nodes: list[A.Node] = []
        self.keep: list = []
        self.leaf_owner: dict[int, Concrete] = {}   # buffer handle -> leaf
        self.index: dict[int, int] = {}

    def array(self):
        arr = (A.Node * len(self.nodes))(*self.nodes)
        self.keep.append(arr)
        return arr


_MAP_OPS = {"add", "sub", "mul", "div", "pow", "gt", "lt", "eq", "ge", "le", "map", "sqrt", "exp", "log", "sin",
            "cos", "tan", "negate", "abs", "floor", "ceiling", "relu", "sigmoid", "tanh"}


def serialize(root) -> Serialized:
    """amc_node records of one tree, or of several roots (a list) realized
    together: then a final OUTPUTS node lists the roots, and a node shared
    between them is serialized, planned and computed once."""
    S = Serialized()

    def visit(m: Morphism) -> int:
        key = id(m)
        if key in S.index:
            return S.index[key]
        nd = A.Node()
        if isinstance(m, Concrete):
            buf = device_buffer_of(m)
            nd.kind = A.NODE["LEAF"]
            nd.dtype = DTYPES[m.dtype]
            _fill_shape(nd, m.shape)
            nd.leaf = _view(buf, m.dtype, m.shape, m.strides, m.offset)
            S.leaf_owner[buf.handle] = m
        elif "scan" in m.meta:
            # batch-fold / batch-scan of an element-wise step: one SCAN node
            # over (init, x) in place of the tree of per-element map nodes
            init, x, prog, keep = m.meta["scan"]
            ins = [visit(init), visit(x)]
            nd.kind = A.NODE["SCAN"]
            nd.dtype = DTYPES[m.dtype]
            _fill_shape(nd, m.shape)
            nd.n_in = 2
            nd.in_[0], nd.in_[1] = ins
            nd.iparam[0] = 1 if keep else 0
            arr = (A.Insn * len(prog))(*[A.Insn(o, a, imm) for (o, a, imm) in prog])
            S.keep.append(arr)
            nd.prog = C.cast(arr, C.POINTER(A.Insn))
            nd.prog_len = len(prog)
        else:
            assert isinstance(m, Expr)
            ins = [visit(o) for o in m.operands]
            nd.dtype = DTYPES[m.dtype]
            _fill_shape(nd, m.shape)
            nd.n_in = len(ins)
            if len(ins) <= A.NODE_MAX_IN:
                for k, i in enumerate(ins):
                    nd.in_[k] = i
            else:
                ext = (C.c_int32 * len(ins))(*ins)
                S.keep.append(ext)
                nd.in_ext = C.cast(ext, C.POINTER(C.c_int32))
            op, meta = m.op, m.meta
            if op in _MAP_OPS:
                nd.kind = A.NODE["MAP"]
                prog = meta["prog"]
                arr = (A.Insn * len(prog))(*[A.Insn(o, a, imm) for (o, a, imm) in prog])
                S.keep.append(arr)
                nd.prog = C.cast(arr, C.POINTER(A.Insn))
                nd.prog_len = len(prog)
            elif op == "reshape":
                nd.kind = A.NODE["RESHAPE"]
            elif op == "transpose":
                nd.kind = A.NODE["TRANSPOSE"]
                for i, p in enumerate(meta["permutation"]):
                    nd.iparam[i] = p
            elif op == "slice":
                nd.kind = A.NODE["SLICE"]
                for i, (s, st) in enumerate(zip(meta["start"], meta["step"])):
                    nd.iparam[i] = s
                    nd.iparam[8 + i] = st
            elif op == "reduce":
                nd.kind = A.NODE["REDUCE"]
                nd.iparam[0] = A.RED[meta["op"]]
                mask = 0
                for ax in meta["axes"]:
                    mask |= 1 << ax
                nd.iparam[1] = mask
                nd.iparam[2] = 1 if meta["keepdims"] else 0
            elif op == "pad":
                nd.kind = A.NODE["PAD"]
                nd.iparam[0] = A.PAD[meta["mode"]]
                for i, (b, a) in enumerate(meta["padding"]):
                    nd.iparam[1 + 2 * i] = b
                    nd.iparam[2 + 2 * i] = a
                nd.fparam[0] = meta["value"]
            elif op in ("im2col", "col2im"):
                nd.kind = A.NODE["IM2COL" if op == "im2col" else "COL2IM"]
                (kh, kw), (sh, sw), (ph, pw) = meta["kernel-size"], meta["stride"], meta["padding"]
                for i, v in enumerate((kh, kw, sh, sw, ph, pw)):
                    nd.iparam[i] = v
            elif op in ("stack", "concat"):
                nd.kind = A.NODE["STACK" if op == "stack" else "CONCAT"]
                nd.iparam[0] = meta["axis"]
            elif op in ("matmul", "matvec", "dot"):
                nd.kind = A.NODE[op.upper()]
            elif op == "attention":
                nd.kind = A.NODE["ATTENTION"]
                nd.fparam[0] = meta["scale"]
            else:
                raise ValueError(f"realize: no device lowering for op {op!r}")
        S.nodes.append(nd)
        idx = len(S.nodes) - 1
        S.index[key] = idx
        S.keep.append(m)  # keep the morphism (and its buffers) alive
        return idx

    if isinstance(root, (list, tuple)):
        idx = [visit(r) for r in root]
        nd = A.Node()
        nd.kind = A.NODE["OUTPUTS"]
        nd.n_in = len(idx)
        if len(idx) <= A.NODE_MAX_IN:
            for k, i in enumerate(idx):
                nd.in_[k] = i
        else:
            ext = (C.c_int32 * len(idx))(*idx)
            S.keep.append(ext)
            nd.in_ext = C.cast(ext, C.POINTER(C.c_int32))
        S.nodes.append(nd)
    else:
        visit(root)
    return S


class Plan:
    """A created device plan (amc_plan_*) for one tree, or for a list of
    roots realized together (their results in order: results())."""

    def __init__(self, root, ctx=None):
        _ensure_init()
        self.roots = list(root) if isinstance(root, (list, tuple)) else [root]
        self.root = self.roots[0]
        self.S = serialize(root)
        arr = self.S.array()
        h = C.c_uint64(0)
        if ctx is None:
            A.call("amc_plan_create", arr, len(self.S.nodes), C.byref(h))
        else:
            A.call("amc_plan_create_ctx", ctx.handle, arr, len(self.S.nodes), C.byref(h))
        self.handle = h.value
        self.ctx = ctx

    def execute(self, stream: int | None = None) -> None:
        A.call("amc_plan_execute", self.handle, C.c_void_p(stream or 0))

    def capture_graph(self, stream: int | None = None) -> None:
        A.call("amc_plan_capture_graph", self.handle, C.c_void_p(stream or 0))

    def stats(self) -> dict:
        l, b, by = C.c_int32(), C.c_int32(), C.c_int64()
        A.call("amc_plan_stats", self.handle, C.byref(l), C.byref(b), C.byref(by))
        return {"launches": l.value, "buffers": b.value, "bytes": by.value}

    def result(self, keep_device: bool = True, index: int = 0, arena: bool = False) -> Concrete:
        """Result `index` as a Concrete.  Its device buffer is kept (read on
        the host only when .data is first used) for plans outside a context;
        a context plan's result is downloaded now, since the next replay
        writes the same arena memory, unless `arena` asks for the arena
        buffer itself (valid until the context's next replay writes it, as
        the reference's pool vectors are)."""
        v = A.View()
        A.call("amc_plan_result_at", self.handle, index, C.byref(v))
        shape = tuple(v.shape[i] for i in range(v.rank))
        strides = tuple(v.strides[i] for i in range(v.rank))
        root = self.roots[index]
        dtype = root.dtype
        owner = self.S.leaf_owner.get(v.buf)
        ba = getattr(root, "batch_axis", -1)
        if owner is not None:
            # zero-copy view of a leaf (create-view): shares the leaf's vector
            A._lib.amc_buf_free(v.buf)
            out = Concrete(owner._data, shape, strides, v.offset, dtype, ba, dev=owner._dev)
            return out
        nel = C.c_int64()
        A.call("amc_buf_info", v.buf, None, C.byref(nel))
        buf = DeviceBuffer(v.buf, dtype, nel.value)
        if keep_device and (self.ctx is None or arena):
            return Concrete(None, shape, strides, v.offset, dtype, ba, dev=buf)
        data = buf.download()
        return Concrete(data, shape, strides, v.offset, dtype, ba)

    def results(self, keep_device: bool = True, arena: bool = False) -> list:
        return [self.result(keep_device, i, arena) for i in range(len(self.roots))]

    def __del__(self):
        try:
            if getattr(self, "handle", 0) and A._lib is not None:
                A._lib.amc_plan_destroy(self.handle)
        except Exception:
            pass
        self.handle = 0


def realize(m: Morphism) -> Concrete:
    """realize (realization.scm:92-115): concrete arrays are returned as-is."""
    if isinstance(m, Concrete):
        return m
    p = Plan(m)
    p.execute()
    return p.result()


def realize_many(ms: list) -> list:
    """The morphisms of `ms` realized together in one plan: a node shared
    between them is computed once (concrete arrays are returned as-is)."""
    lazy = [m for m in ms if not isinstance(m, Concrete)]
    if not lazy:
        return list(ms)
    p = Plan(lazy)
    p.execute()
    it = iter(p.results())
    return [m if isinstance(m, Concrete) else next(it) for m in ms]


def force_morphism(m: Morphism) -> Concrete:
    return realize(m)


realize_bang = realize


def morph_to_list(m: Morphism):
    """morph->list (core.scm:862-882): nested Python lists of the values."""
    r = realize(m)
    v = r.values()
    return v.tolist()


def to_numpy(m: Morphism) -> np.ndarray:
    return realize(m).values()
