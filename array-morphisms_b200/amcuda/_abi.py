"""ctypes binding of include/amc.h (the C ABI of libamcuda.so).

This is the binding a host language wraps around the library: the Scheme
host would declare the same entry points with foreign-lambda.  Loading fails
loudly when the shared library is missing; there is no fallback.
"""
from __future__ import annotations

import ctypes as C
import os
from pathlib import Path

LIB_PATH = Path(__file__).resolve().parent / "libamcuda.so"

AMC_OK = 0
ERR_NAMES = {1: "INVALID", 2: "UNSUPPORTED", 3: "CUDA", 4: "OOM", 5: "STATE", 6: "INJECTED", 7: "TIMEOUT"}

F32, F64, S32, S64, U32, U64 = 0, 1, 2, 3, 4, 5
MAX_RANK = 8

OP = dict(LOAD=1, CONST=2, ICONST=3, CVT=4, NEG=10, ABS=11, FLOOR=12, CEIL=13, SQRT=14, EXP=15, LOG=16, SIN=17,
          COS=18, TAN=19, RELU=20, SIGMOID=21, TANH=22, ADD=40, SUB=41, MUL=42, DIV=43, POW=44, MAX=45, MIN=46,
          GT=50, LT=51, EQ=52, GE=53, LE=54)
RED = dict(sum=0, mean=1, prod=2, max=3, min=4)
PAD = dict(constant=0, edge=1, reflect=2)
NODE = dict(LEAF=1, RESHAPE=2, TRANSPOSE=3, SLICE=4, MAP=5, REDUCE=6, PAD=7, IM2COL=8, COL2IM=9, STACK=10,
            CONCAT=11, MATMUL=12, MATVEC=13, DOT=14, ATTENTION=15, SCAN=16, OUTPUTS=17)
PROG_MAX = 64
STACK_MAX = 16
NODE_MAX_IN = 4


class AmcError(RuntimeError):
    def __init__(self, code: int, msg: str):
        super().__init__(f"amc error {ERR_NAMES.get(code, code)}: {msg}")
        self.code = code


class View(C.Structure):
    _fields_ = [("buf", C.c_uint64), ("dtype", C.c_int32), ("rank", C.c_int32),
                ("shape", C.c_int64 * MAX_RANK), ("strides", C.c_int64 * MAX_RANK), ("offset", C.c_int64)]


class Insn(C.Structure):
    _fields_ = [("op", C.c_int32), ("a", C.c_int32), ("imm", C.c_double)]


class Node(C.Structure):
    _fields_ = [("kind", C.c_int32), ("dtype", C.c_int32), ("rank", C.c_int32), ("n_in", C.c_int32),
                ("shape", C.c_int64 * MAX_RANK), ("in_", C.c_int32 * NODE_MAX_IN), ("in_ext", C.POINTER(C.c_int32)),
                ("iparam", C.c_int64 * 24), ("fparam", C.c_double * 4), ("prog", C.POINTER(Insn)),
                ("prog_len", C.c_int32), ("_pad", C.c_int32), ("leaf", View)]


_P = C.c_void_p
_I32, _I64, _U64 = C.c_int32, C.c_int64, C.c_uint64
_PI32, _PI64, _PU64 = C.POINTER(C.c_int32), C.POINTER(C.c_int64), C.POINTER(C.c_uint64)
_D, _F = C.c_double, C.c_float
_PD, _PF = C.POINTER(C.c_double), C.POINTER(C.c_float)

# name -> argtypes (every entry point returns int)
SIGNATURES = {
    "amc_last_error": [C.c_char_p, C.c_size_t],
    "amc_version": [C.POINTER(C.c_int), C.POINTER(C.c_int)],
    "amc_device_count": [C.POINTER(C.c_int)],
    "amc_init": [C.c_int],
    "amc_shutdown": [],
    "amc_synchronize": [],
    "amc_buf_create": [_I32, _I64, _PU64],
    "amc_buf_wrap": [_P, _I32, _I64, _PU64],
    "amc_buf_upload": [_U64, _P, _I64, _I64],
    "amc_buf_download": [_U64, _P, _I64, _I64],
    "amc_buf_upload_async": [_U64, _P, _I64, _I64, _P],
    "amc_buf_download_async": [_U64, _P, _I64, _I64, _P],
    "amc_buf_copy_async": [_U64, _I64, _U64, _I64, _I64, _P],
    "amc_buf_devptr": [_U64, C.POINTER(_P)],
    "amc_buf_info": [_U64, _PI32, _PI64],
    "amc_buf_free": [_U64],
    "amc_plan_create": [C.POINTER(Node), _I32, _PU64],
    "amc_plan_execute": [_U64, _P],
    "amc_plan_result": [_U64, C.POINTER(View)],
    "amc_plan_result_count": [_U64, _PI32],
    "amc_plan_result_at": [_U64, _I32, C.POINTER(View)],
    "amc_plan_stats": [_U64, _PI32, _PI32, _PI64],
    "amc_plan_capture_graph": [_U64, _P],
    "amc_plan_destroy": [_U64],
    "amc_ctx_create": [_PU64],
    "amc_plan_create_ctx": [_U64, C.POINTER(Node), _I32, _PU64],
    "amc_ctx_pin_output": [_U64, _U64],
    "amc_ctx_finalize": [_U64],
    "amc_ctx_reset": [_U64],
    "amc_ctx_replay": [_U64, _U64, _P],
    "amc_ctx_stats": [_U64, _PI32, _PI32, _PI64, _PI32],
    "amc_ctx_destroy": [_U64],
    "amc_colour": [_I32, _PI32, _PI64, _PI32, _PI32, _PI32, _PI32, _PI32],
    "amc_blas_dgemm": [_I32, _I32, _I32, _D, _PD, _PD, _D, _PD],
    "amc_blas_sgemm": [_I32, _I32, _I32, _F, _PF, _PF, _F, _PF],
    "amc_blas_dgemm_strided": [_I32, _I32, _I32, _D, _PD, _I32, _I32, _PD, _I32, _I32, _D, _PD],
    "amc_blas_sgemm_strided": [_I32, _I32, _I32, _F, _PF, _I32, _I32, _PF, _I32, _I32, _F, _PF],
    "amc_blas_dgemv": [_I32, _I32, _D, _PD, _PD, _D, _PD],
    "amc_blas_sgemv": [_I32, _I32, _F, _PF, _PF, _F, _PF],
    "amc_blas_ddot": [_I32, _PD, _PD, _PD],
    "amc_blas_sdot": [_I32, _PF, _PF, _PF],
    "amc_blas_daxpy": [_I32, _D, _PD, _PD],
    "amc_blas_saxpy": [_I32, _F, _PF, _PF],
    "amc_window_fir_f32": [_P, _I64, _I64, _I64, _I64, _I32, _I32, _P, _P, _P],
    "amc_linreg_partials_count": [_I64, _I32, _PI32],
    "amc_linreg_partials": [_P, _P, _P, _I64, _I32, _I64, _P, _P],
    "amc_linreg_reduce": [_P, _I32, _I32, _P, _P],
    "amc_linreg_update": [_P, _P, _I32, _I64, _D, _P, _P],
    "amc_linreg_step": [_P, _P, _P, _I64, _I32, _D, _P, _P, _P, _P],
    "amc_linreg_step_noalloc": [_P, _P, _P, _I64, _I32, _D, _P, _P],
    "amc_attention_fwd_f32": [_P, _P, _P, _P, _P, _I64, _I32, _I32, _I32, _F, _P],
    "amc_attention_bwd_f32": [_P, _P, _P, _P, _P, _P, _P, _P, _P, _I64, _I32, _I32, _I32, _F, _P],
    "amc_conv2d_fwd_f32": [_P, _P, _P] + [_I32] * 11 + [_P],
    "amc_conv2d_dgrad_f32": [_P, _P, _P] + [_I32] * 11 + [_P],
    "amc_conv2d_wgrad_f32": [_P, _P, _P] + [_I32] * 11 + [_P],
    "amc_tc_peak_tf32": [_I32, _I32, _I32, _I32, _P, _P],
    "amc_peer_group_create": [_I32, _I32, _I64, _PU64, _P],
    "amc_peer_group_open": [_U64, _P],
    "amc_peer_sum": [_U64, _P, _I64, _I32, _P, _P],
    "amc_peer_group_destroy": [_U64],
    "amc_probe_bounded_wait": [_I32, _I32, _P],
    "amc_colfold_launch_count": [_P],
}

_lib = None


def load() -> C.CDLL:
    """Load libamcuda.so (no CUDA call is made by loading)."""
    global _lib
    if _lib is not None:
        return _lib
    if not LIB_PATH.exists():
        raise ImportError(f"libamcuda.so is not built ({LIB_PATH}); run array-morphisms_b200/build.py")
    lib = C.CDLL(str(LIB_PATH))
    for name, argtypes in SIGNATURES.items():
        fn = getattr(lib, name)
        fn.argtypes = argtypes
        fn.restype = C.c_int
    _lib = lib
    return lib


def last_error() -> str:
    buf = C.create_string_buffer(1024)
    load().amc_last_error(buf, 1024)
    return buf.value.decode(errors="replace")


def check(rc: int) -> None:
    if rc != AMC_OK:
        raise AmcError(rc, last_error())


def call(name: str, *args) -> None:
    check(getattr(load(), name)(*args))
