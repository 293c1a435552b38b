"""CPU oracle: the reference's realize, restated (TEST INFRASTRUCTURE ONLY).

Only tests/, __graft_entry__.smoke() and bench.py's CPU baseline use this
module, as the checker; the product (libamcuda) never imports it.

`realize` below walks the same lazy tree the product realizes and follows the
reference's recursion (realization.scm:92-115, :398-468): every non-view node
is materialised into a fresh typed vector by the per-element loops in
amc_oracle.c; reshape/transpose/slice of a concrete array are zero-copy views
(can-use-zero-copy? / create-view, :649-717), and a reshape of a
non-contiguous array copies in logical row-major order (:849-862).  The conv
pattern reshape(matmul(W, im2col(X))) runs execute-conv2d-blas's per-image
im2col + GEMM (:136-252).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess
import sys
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent
sys.path.insert(0, str(ROOT / "array-morphisms_b200"))

from amcuda import _abi as A  # noqa: E402  (constants only)
from amcuda.morph import (DTYPES, NP_DTYPES, Concrete, Expr, Morphism, compute_strides,  # noqa: E402
                          shape_size)

LIB = HERE / "liboracle.so"
SRC = HERE / "amc_oracle.c"


def build() -> Path:
    if not LIB.exists() or LIB.stat().st_mtime < SRC.stat().st_mtime:
        subprocess.run(["gcc", "-O2", "-shared", "-fPIC", "-std=c11", str(SRC), "-o", str(LIB), "-lm"], check=True)
    return LIB


class OView(C.Structure):
    _fields_ = [("data", C.c_void_p), ("dtype", C.c_int32), ("rank", C.c_int32),
                ("shape", C.c_int64 * 8), ("strides", C.c_int64 * 8), ("offset", C.c_int64)]


_lib = None


def lib():
    global _lib
    if _lib is None:
        _lib = C.CDLL(str(build()))
        for f in ("orc_map", "orc_reduce", "orc_copy_logical", "orc_pad", "orc_im2col", "orc_col2im", "orc_route",
                  "orc_gemm", "orc_gemv", "orc_dot", "orc_conv2d", "orc_attention", "orc_attention_bwd",
                  "orc_linreg", "orc_colour"):
            getattr(_lib, f).restype = C.c_int
    return _lib


def _ov(m: Concrete) -> OView:
    v = OView()
    v.data = m.data.ctypes.data
    v.dtype = DTYPES[m.dtype]
    v.rank = len(m.shape)
    for i, (s, st) in enumerate(zip(m.shape, m.strides)):
        v.shape[i] = s
        v.strides[i] = st
    v.offset = m.offset
    return v


def _i64(xs):
    return (C.c_int64 * max(len(xs), 1))(*xs)


def _alloc(dtype: str, shape) -> Concrete:
    return Concrete(np.zeros(shape_size(shape), dtype=NP_DTYPES[dtype]), shape, dtype=dtype)


def _check(rc: int, what: str):
    if rc != 0:
        raise RuntimeError(f"oracle {what} failed ({rc})")


def _contiguous(m: Concrete) -> bool:
    """contiguous-array? (realization.scm:626-642): offset 0, row-major strides."""
    return m.offset == 0 and tuple(m.strides) == compute_strides(m.shape)


def _view(m: Concrete, shape, strides, offset) -> Concrete:
    return Concrete(m.data, shape, strides, offset, m.dtype)


_MAP = {"add", "sub", "mul", "div", "pow", "gt", "lt", "eq", "ge", "le", "map", "sqrt", "exp", "log", "sin", "cos",
        "tan", "negate", "abs", "floor", "ceiling", "relu", "sigmoid", "tanh"}


def realize(m: Morphism) -> Concrete:
    if isinstance(m, Concrete):
        return m
    assert isinstance(m, Expr)
    op = m.op
    L = lib()
    # conv pattern first, on the unrealized tree (realization.scm:425-430)
    if op == "reshape" and isinstance(m.operands[0], Expr) and m.operands[0].op == "matmul":
        mm = m.operands[0]
        if isinstance(mm.operands[1], Expr) and mm.operands[1].op == "im2col":
            ic = mm.operands[1]
            X = realize(ic.operands[0])
            Wm = realize(mm.operands[0])
            Wc = _contig(Wm)
            (kh, kw), (sh, sw), (ph, pw) = ic.meta["kernel-size"], ic.meta["stride"], ic.meta["padding"]
            out = _alloc(m.dtype, m.shape)
            _check(L.orc_conv2d(out.data.ctypes.data_as(C.c_void_p), DTYPES[m.dtype], C.byref(_ov(X)), C.byref(_ov(Wc)),
                                1 if len(X.shape) == 4 else 0, kh, kw, sh, sw, ph, pw), "conv2d")
            return out
    if op == "attention":
        Q, K, V = (realize(o) for o in m.operands)
        out = _alloc(m.dtype, m.shape)
        _check(L.orc_attention(out.data.ctypes.data_as(C.c_void_p), DTYPES[m.dtype], C.byref(_ov(Q)), C.byref(_ov(K)),
                               C.byref(_ov(V)), m.meta["n-leading"], C.c_double(m.meta["scale"])), "attention")
        return out
    ops = [realize(o) for o in m.operands]
    if op in ("matmul", "matvec", "dot"):
        out = _alloc(m.dtype, m.shape)
        f = {"matmul": L.orc_gemm, "matvec": L.orc_gemv, "dot": L.orc_dot}[op]
        _check(f(out.data.ctypes.data_as(C.c_void_p), DTYPES[m.dtype], C.byref(_ov(ops[0])), C.byref(_ov(ops[1]))), op)
        return out
    if op == "reshape":
        src = ops[0]
        if _contiguous(src):
            return _view(src, m.shape, compute_strides(m.shape), 0)
        out = _alloc(m.dtype, m.shape)
        _check(L.orc_copy_logical(out.data.ctypes.data_as(C.c_void_p), DTYPES[m.dtype], C.byref(_ov(src))), "copy")
        return out
    if op == "transpose":
        src = ops[0]
        perm = m.meta["permutation"]
        return _view(src, m.shape, [src.strides[p] for p in perm], src.offset)
    if op == "slice":
        src = ops[0]
        st, step = m.meta["start"], m.meta["step"]
        return _view(src, m.shape, [s * k for s, k in zip(src.strides, step)],
                     src.offset + sum(a * s for a, s in zip(st, src.strides)))
    if op in _MAP:
        out = _alloc(m.dtype, m.shape)
        prog = m.meta["prog"]
        P = (A.Insn * len(prog))(*[A.Insn(o, a, imm) for (o, a, imm) in prog])
        V = (OView * len(ops))(*[_ov(o) for o in ops])
        _check(L.orc_map(out.data.ctypes.data_as(C.c_void_p), DTYPES[m.dtype], len(m.shape), _i64(m.shape), len(ops), V,
                         P, len(prog)), f"map {op}")
        return out
    if op == "reduce":
        out = _alloc(m.dtype, m.shape)
        mask = 0
        for ax in m.meta["axes"]:
            mask |= 1 << ax
        rc = L.orc_reduce(out.data.ctypes.data_as(C.c_void_p), DTYPES[m.dtype], C.byref(_ov(ops[0])), C.c_int64(mask),
                          1 if m.meta["keepdims"] else 0, A.RED[m.meta["op"]])
        if rc == -4:
            raise ValueError("integer max/min reduction (the reference fails storing +-inf)")
        _check(rc, "reduce")
        return out
    if op == "pad":
        out = _alloc(m.dtype, m.shape)
        pads = [x for p in m.meta["padding"] for x in p]
        _check(L.orc_pad(out.data.ctypes.data_as(C.c_void_p), DTYPES[m.dtype], len(m.shape), _i64(m.shape),
                         C.byref(_ov(ops[0])), _i64(pads), A.PAD[m.meta["mode"]], C.c_double(m.meta["value"])), "pad")
        return out
    if op == "im2col":
        out = _alloc(m.dtype, m.shape)
        (kh, kw), (sh, sw), (ph, pw) = m.meta["kernel-size"], m.meta["stride"], m.meta["padding"]
        _check(L.orc_im2col(out.data.ctypes.data_as(C.c_void_p), DTYPES[m.dtype], C.byref(_ov(ops[0])),
                            1 if len(ops[0].shape) == 4 else 0, kh, kw, sh, sw, ph, pw), "im2col")
        return out
    if op == "col2im":
        col = _contig(ops[0])
        out = _alloc(m.dtype, m.shape)
        (kh, kw), (sh, sw), (ph, pw) = m.meta["kernel-size"], m.meta["stride"], m.meta["padding"]
        b = len(m.shape) == 4
        N, Cc, H, W = m.shape if b else (1,) + tuple(m.shape)
        _check(L.orc_col2im(out.data.ctypes.data_as(C.c_void_p), DTYPES[m.dtype], 1 if b else 0, C.c_int64(N), C.c_int64(Cc),
                            C.c_int64(H), C.c_int64(W), col.data.ctypes.data_as(C.c_void_p), DTYPES[col.dtype],
                            kh, kw, sh, sw, ph, pw), "col2im")
        return out
    if op in ("stack", "concat"):
        out = _alloc(m.dtype, m.shape)
        V = (OView * len(ops))(*[_ov(o) for o in ops])
        _check(L.orc_route(out.data.ctypes.data_as(C.c_void_p), DTYPES[m.dtype], len(m.shape), _i64(m.shape), len(ops), V,
                           m.meta["axis"], 1 if op == "stack" else 0), op)
        return out
    raise ValueError(f"oracle: unknown op {op}")


def _contig(m: Concrete) -> Concrete:
    if _contiguous(m):
        return m
    out = _alloc(m.dtype, m.shape)
    _check(lib().orc_copy_logical(out.data.ctypes.data_as(C.c_void_p), DTYPES[m.dtype], C.byref(_ov(m))), "copy")
    return out


def values(m: Morphism) -> np.ndarray:
    return realize(m).values()


# ---------------------------------------------------------------------------- direct restatements
def conv2d_fwd(X: np.ndarray, W: np.ndarray, stride=1, pad=1) -> np.ndarray:
    from amcuda.morph import morph_from_numpy
    Xm, Wm = morph_from_numpy(X), morph_from_numpy(W)
    N = X.shape[0]
    K, Cc, KH, KW = W.shape
    OH = 1 + (X.shape[2] + 2 * pad - KH) // stride
    OW = 1 + (X.shape[3] + 2 * pad - KW) // stride
    out = np.zeros((N, K, OH, OW), dtype=X.dtype)
    w2 = Concrete(Wm.data, (K, Cc * KH * KW), dtype=Wm.dtype)
    _check(lib().orc_conv2d(out.ctypes.data_as(C.c_void_p), DTYPES[Xm.dtype], C.byref(_ov(Xm)), C.byref(_ov(w2)), 1,
                            KH, KW, stride, stride, pad, pad), "conv2d")
    return out


def conv2d_dgrad(dY: np.ndarray, W: np.ndarray, x_shape, stride=1, pad=1) -> np.ndarray:
    """dX = col2im(W2d^T . dY_n) per sample, as the reference composes it
    (GEMM with double accumulation stored as dtype, then col2im's ordered sum)."""
    from amcuda.morph import col2im_morph, morph_from_numpy, morph_matmul, morph_reshape, morph_transpose
    N = dY.shape[0]
    K, Cc, KH, KW = W.shape
    out = np.zeros(x_shape, dtype=dY.dtype)
    Wm = morph_reshape(morph_from_numpy(W), (K, Cc * KH * KW))
    for n in range(N):
        g = morph_reshape(morph_from_numpy(dY[n]), (K, dY.shape[2] * dY.shape[3]))
        col = morph_matmul(morph_transpose(Wm), g)
        out[n] = values(col2im_morph(col, x_shape[1:], (KH, KW), stride, pad))
    return out


def conv2d_wgrad(X: np.ndarray, dY: np.ndarray, w_shape, stride=1, pad=1) -> np.ndarray:
    """dW = sum_n dY_n . im2col(X_n)^T (per-sample GEMMs summed in n order)."""
    from amcuda.morph import im2col_morph, morph_from_numpy, morph_matmul, morph_reshape, morph_transpose
    K, Cc, KH, KW = w_shape
    acc = np.zeros(K * Cc * KH * KW, dtype=X.dtype)
    for n in range(X.shape[0]):
        col = im2col_morph(morph_from_numpy(X[n]), (KH, KW), stride, pad)
        g = morph_reshape(morph_from_numpy(dY[n]), (K, dY.shape[2] * dY.shape[3]))
        part = values(morph_matmul(g, morph_transpose(col))).reshape(-1)
        acc = (acc.astype(np.float64) + part.astype(np.float64)).astype(X.dtype)
    return acc.reshape(w_shape)


def attention_bwd(Q, K, V, dO, scale):
    nb = int(np.prod(Q.shape[:-2]))
    n, dk, dv = Q.shape[-2], Q.shape[-1], V.shape[-1]
    dQ = np.zeros(Q.shape, np.float32)
    dK = np.zeros(K.shape, np.float32)
    dV = np.zeros(V.shape, np.float32)
    f = lambda a: np.ascontiguousarray(a, dtype=np.float32).ctypes.data_as(C.c_void_p)
    Qc, Kc, Vc, Gc = (np.ascontiguousarray(a, dtype=np.float32) for a in (Q, K, V, dO))
    _check(lib().orc_attention_bwd(Qc.ctypes.data_as(C.c_void_p), Kc.ctypes.data_as(C.c_void_p),
                                   Vc.ctypes.data_as(C.c_void_p), Gc.ctypes.data_as(C.c_void_p),
                                   dQ.ctypes.data_as(C.c_void_p), dK.ctypes.data_as(C.c_void_p),
                                   dV.ctypes.data_as(C.c_void_p), C.c_int64(nb), C.c_int64(n), C.c_int64(dk),
                                   C.c_int64(dv), C.c_double(scale)), "attention_bwd")
    return dQ, dK, dV


def linreg(X: np.ndarray, y: np.ndarray, w0: np.ndarray, steps: int, lr: float):
    X = np.ascontiguousarray(X, dtype=np.float64)
    y = np.ascontiguousarray(y, dtype=np.float64).reshape(-1)
    w = np.array(w0, dtype=np.float64).reshape(-1).copy()
    losses = np.zeros(steps, dtype=np.float64)
    _check(lib().orc_linreg(X.ctypes.data_as(C.c_void_p), y.ctypes.data_as(C.c_void_p), w.ctypes.data_as(C.c_void_p),
                            C.c_int64(X.shape[0]), C.c_int32(X.shape[1]), C.c_int32(steps), C.c_double(lr),
                            losses.ctypes.data_as(C.c_void_p)), "linreg")
    return w, losses


def colour(dtypes, sizes, inputs, pinned=None):
    n = len(dtypes)
    off = [0]
    flat = []
    for ins in inputs:
        flat.extend(ins)
        off.append(len(flat))
    DT = (C.c_int32 * max(n, 1))(*dtypes)
    SZ = (C.c_int64 * max(n, 1))(*sizes)
    OF = (C.c_int32 * (n + 1))(*off)
    IN = (C.c_int32 * max(len(flat), 1))(*flat)
    PN = (C.c_int32 * max(n, 1))(*(pinned or [0] * n))
    AS = (C.c_int32 * max(n, 1))()
    NB = C.c_int32()
    _check(lib().orc_colour(n, DT, SZ, OF, IN, PN, AS, C.byref(NB)), "colour")
    return list(AS)[:n], NB.value
