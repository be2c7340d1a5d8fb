"""ctypes binding of libcq_b200.so (the C ABI declared in include/cq_b200.h).

The library is the only implementation of the hot path: there is no CPU or eager fallback.  Loading fails
with an exception when the shared object is missing, and every entry point raises on a nonzero status.
"""
from __future__ import annotations

import ctypes
import os
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libcq_b200.so")

CQ_OK = 0
CQ_ERR_ARG = 1
CQ_ERR_SHAPE = 2
CQ_ERR_ALIGN = 3
CQ_ERR_CUDA = 4
CQ_ERR_TIMEOUT = 5
CQ_ERR_UNSUPPORTED = 6
CQ_ERR_CAPACITY = 7

CQ_ACT_INT8_ROW = 0
CQ_ACT_INT4_ROW = 1
CQ_ACT_INT4_GROUP = 2

CQ_W_INT4_ROW = 0
CQ_W_INT8_ROW = 1
CQ_W_AFFINE_INT4_GROUP = 2
CQ_W_INT4_GROUP_BF16UP = 3

CQ_Q_INT8_CODES = 1
CQ_Q_KPERM = 2

CQ_B_INT4_SIGNED = 0
CQ_B_INT8 = 1

CQ_GEMM_AUTO = 0
CQ_GEMM_ONE_SM = 1
CQ_GEMM_PAIR = 2

CQ_OUT_PLAIN = 0
CQ_OUT_GELU_TANH = 1
CQ_OUT_GATED_RESIDUAL = 2

_i64 = ctypes.c_int64
_int = ctypes.c_int
_vp = ctypes.c_void_p
_f32 = ctypes.c_float


class CQOutOp(ctypes.Structure):
    """cq_out_op: the output operation of the W4A8 affine GEMM's epilogue."""
    _fields_ = [("kind", ctypes.c_int), ("residual", ctypes.c_void_p), ("residual_ld", ctypes.c_int64),
                ("gate", ctypes.c_void_p)]


_opp = ctypes.POINTER(CQOutOp)

# name -> (restype, argtypes), one line per declaration of include/cq_b200.h
SIGNATURES = {
    "cq_version": (ctypes.c_char_p, []),
    "cq_status_string": (ctypes.c_char_p, [_int]),
    "cq_set_gemm_variant": (_int, [_int]),
    "cq_take_device_status": (_int, [ctypes.POINTER(_int), _vp]),
    "cq_selftest_bounded_wait": (_int, [_vp]),
    "cq_rotquant": (_int, [_vp, _i64, _i64, _int, _int, _int, _int, _i64, _int, _vp, _vp, _vp, _vp]),
    "cq_weight_rotquant": (_int, [_vp, _int, _i64, _i64, _int, _int, _int, _vp, _vp, _vp, _vp]),
    "cq_unpack_int4": (_int, [_vp, _i64, _i64, _vp, _vp]),
    "cq_gemm_rowcol": (_int, [_vp, _int, _vp, _vp, _int, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "cq_group_sum_cols": (_i64, [_i64]),
    "cq_prepare_affine_zeros": (_int, [_vp, _i64, _i64, _int, _vp, _vp]),
    "cq_gemm_groupwise": (_int, [_vp, _int, _vp, _i64, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp]),
    "cq_gemm_intratio": (_int, [_vp, _int, _vp, _vp, _vp, _vp, _int, _int, _vp, _vp, _i64, _i64, _i64, _vp]),
    "cq_gemm_affine": (_int, [_vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _int, _vp]),
    "cq_gemm_affine_op": (_int, [_vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _opp, _vp, _i64, _i64, _i64, _int, _vp]),
    "cq_linear_workspace_bytes": (_i64, [_i64, _i64]),
    "cq_linear_workspace_bytes_n": (_i64, [_i64, _i64, _i64]),
    "cq_linear_convrot_w4a4": (_int, [_vp, _i64, _i64, _i64, _int, _int, _int, _vp, _vp, _vp, _vp, _vp, _i64, _vp]),
    "cq_linear_w4a8_affine": (_int, [_vp, _i64, _i64, _i64, _int, _int, _vp, _vp, _vp, _int, _vp, _vp, _vp, _i64,
                                     _vp]),
    "cq_linear_w8a8": (_int, [_vp, _i64, _i64, _i64, _int, _int, _vp, _vp, _vp, _vp, _vp, _i64, _vp]),
    "cq_linear_convrot_w4a4_op": (_int, [_vp, _i64, _i64, _i64, _int, _int, _vp, _vp, _f32, _vp, _vp, _vp, _opp,
                                         _vp, _vp, _i64, _vp]),
    "cq_linear_w8a8_op": (_int, [_vp, _i64, _i64, _i64, _int, _vp, _vp, _f32, _vp, _vp, _vp, _opp, _vp, _vp, _i64,
                                 _vp]),
    "cq_linear_w4a8_affine_noalloc": (_int, [_vp, _i64, _i64, _i64, _int, _int, _vp, _vp, _vp, _int, _vp, _vp, _vp]),
    "cq_gemm_affine_peers": (_int, [_vp, _int, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _int, _i64, _i64, _i64, _i64, _i64,
                                    _int, _vp]),
    "cq_linear_w4a8_affine_peers": (_int, [_vp, _i64, _i64, _i64, _int, _int, _vp, _vp, _vp, _int, _vp, _vp, _int,
                                           _i64, _i64, _vp, _i64, _vp]),
    "cq_rotquant_lnmod": (_int, [_vp, _i64, _i64, _int, _vp, _vp, _f32, _i64, _int, _vp, _vp, _vp, _vp]),
    "cq_linear_w4a8_affine_lnmod": (_int, [_vp, _i64, _i64, _i64, _int, _vp, _vp, _f32, _vp, _vp, _vp, _int, _vp,
                                           _vp, _vp, _i64, _vp]),
    "cq_linear_w4a8_op": (_int, [_vp, _i64, _i64, _i64, _int, _vp, _vp, _f32, _vp, _vp, _vp, _int, _vp, _opp, _vp,
                                 _vp, _i64, _vp]),
    "cq_rotquant_absmax": (_int, [_vp, _i64, _i64, _int, _i64, _vp, _vp]),
    "cq_rotquant_scaled": (_int, [_vp, _i64, _i64, _int, _vp, _i64, _int, _vp, _vp, _vp, _vp]),
    "cq_qkv_rmsnorm_rope": (_int, [_vp, _i64, _int, _int, _vp, _vp, _f32, _vp, _vp, _vp, _vp, _i64, _i64, _vp]),
    "cq_rmsnorm_rope_rows": (_int, [_vp, _i64, _int, _vp, _f32, _vp, _int, _vp, _vp]),
    "cq_qkv_rmsnorm_rope_layout": (_int, [_vp, _i64, _int, _int, _vp, _vp, _f32, _vp, _vp, _vp, _vp, _i64, _i64, _int,
                                          _vp]),
    "cq_heads_to_rows": (_int, [_vp, _i64, _int, _int, _vp, _int, _i64, _i64, _vp]),
    "cq_gemm_rowcol_swiglu": (_int, [_vp, _vp, _vp, _vp, _vp, _vp, _i64, _i64, _i64, _vp]),
    "cq_linear_convrot_w4a4_swiglu": (_int, [_vp, _i64, _i64, _i64, _int, _int, _vp, _vp, _vp, _vp, _vp, _i64, _vp]),
}


class CQError(RuntimeError):
    """A nonzero cq_status from the native library."""

    def __init__(self, fn: str, status: int, message: str):
        super().__init__(f"{fn} failed: {message} (status {status})")
        self.status = status


class CQShapeError(CQError, ValueError):
    """Shape / argument rejected by the native library (mirrors the reference's ValueError / TORCH_CHECK)."""


_lock = threading.Lock()
_lib = None


def load() -> ctypes.CDLL:
    """Load (once) and type the shared library.  Raises if it is absent: there is no fallback path."""
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise ImportError(f"{LIB_PATH} is missing: build it with `python -m comfy_quant_bench_b200.build` "
                                  "(the quantized-linear path has no CPU fallback)")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def status_string(status: int) -> str:
    return load().cq_status_string(status).decode()


def check(fn: str, status: int) -> None:
    if status == CQ_OK:
        return
    msg = status_string(status)
    if status in (CQ_ERR_ARG, CQ_ERR_SHAPE, CQ_ERR_ALIGN):
        raise CQShapeError(fn, status, msg)
    raise CQError(fn, status, msg)


def call(name: str, *args) -> None:
    check(name, getattr(load(), name)(*args))


def exported_symbols() -> list[str]:
    return list(SIGNATURES)


def set_gemm_variant(variant: int) -> None:
    """Process-wide kernel form of the packed-int4-weight GEMMs (CQ_GEMM_AUTO, CQ_GEMM_ONE_SM, CQ_GEMM_PAIR)."""
    call("cq_set_gemm_variant", int(variant))


def take_device_status(stream=None) -> tuple[int, int]:
    st = (ctypes.c_int * 2)()
    call("cq_take_device_status", st, stream)
    return int(st[0]), int(st[1])
