"""ctypes view of the CPU parity oracle (oracle/liboracle.so).

TEST INFRASTRUCTURE ONLY: imported by tests/, by ``__graft_entry__.smoke()``
and by ``bench.py``'s CPU-baseline / reference legs, and only as the checker.
The product library ``tiler_b200/libtiler_cuda.so`` never calls it.

The C++ restatement it wraps follows moderately-ai/tiler's
``crates/tiler-reference`` (file:line cited per function in oracle.cpp).
"""
from __future__ import annotations

import ctypes as C
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "liboracle.so")

OK = 0
INVALID_APPLICATION = 1
GATHER_INDEX_OUT_OF_BOUNDS = 3
NAN_INPUT = 4
UNDECIDED = 5
SCALE_DOMAIN = 9


class OracleError(C.Structure):
    _fields_ = [("code", C.c_int32), ("position", C.c_uint64), ("value", C.c_int64),
                ("extent", C.c_uint64)]


def build() -> str:
    """Compile liboracle.so from oracle.cpp (make) if it is missing or stale."""
    src = os.path.join(_HERE, "oracle.cpp")
    if (not os.path.exists(_LIB_PATH)
            or os.path.getmtime(_LIB_PATH) < os.path.getmtime(src)):
        subprocess.run(["make", "-C", _HERE], check=True, capture_output=True)
    return _LIB_PATH


_lib = None


def lib() -> C.CDLL:
    global _lib
    if _lib is None:
        if not os.path.exists(_LIB_PATH):
            build()
        _lib = C.CDLL(_LIB_PATH)
        _declare(_lib)
    return _lib


def _declare(L: C.CDLL) -> None:
    p = C.c_void_p
    u64, i64, u32, i32 = C.c_uint64, C.c_int64, C.c_uint32, C.c_int32
    sig = {
        "oracle_canonicalize": (C.c_float, [C.c_float]),
        "oracle_maximum": (C.c_float, [C.c_float, C.c_float]),
        "oracle_exp": (C.c_float, [C.c_float, p]),
        "oracle_rsqrt": (C.c_float, [C.c_float, p]),
        "oracle_silu": (C.c_float, [C.c_float, p]),
        "oracle_f32_to_bf16": (C.c_uint16, [C.c_float]),
        "oracle_bf16_to_f32": (C.c_float, [C.c_uint16]),
        "oracle_strict_sum": (i32, [p, u64, u64, p]),
        "oracle_partitioned_sum": (i32, [p, u64, u64, u64, u64, p]),
        "oracle_cooperative_sum": (i32, [p, u64, u64, u64, u64, u64, i32, p]),
        "oracle_compose_fold": (i32, [p, u64, u32, u32, u32, i32, p]),
        "oracle_grid_fold": (i32, [p, u64, u64, u64, u32, u32, u32, u32, u32, u32, i32, i32, p]),
        "oracle_strict_max": (i32, [p, u64, u64, p]),
        "oracle_rms_norm_f32": (i32, [p, p, i64, u64, u64, u32, p, i32]),
        "oracle_rms_norm_bf16": (i32, [p, p, i64, u64, u64, u32, p, i32]),
        "oracle_softmax_f32": (i32, [p, u64, u64, u64, u64, p, i32]),
        "oracle_silu_f32": (i32, [p, u64, p]),
        "oracle_scale_bias_f32": (i32, [p, u64, p, i32, p, i32, p]),
        "oracle_gather_rows": (i32, [p, u64, u64, p, i32, u64, p, p]),
        "oracle_quantize_i8_rows": (i32, [p, u64, u64, p, p, p, i32]),
        "oracle_dequantize_i8_rows": (i32, [p, p, u64, u64, p, i32]),
        "oracle_quantize_affine_u8": (i32, [p, u64, C.c_float, u32, u32, p, p]),
        "oracle_dequantize_affine_u8": (i32, [p, u64, C.c_float, u32, p]),
        "oracle_contract_f32": (i32, [p, p, u64, u64, u64, p, i32]),
        "oracle_gemm_bf16_silu": (i32, [p, p, u64, u64, u64, u64, u64, i32, p, i32]),
    }
    for name, (res, args) in sig.items():
        fn = getattr(L, name)
        fn.restype = res
        fn.argtypes = args


def _ptr(a: np.ndarray) -> int:
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data


def f32(bits) -> np.ndarray:
    return np.asarray(bits, dtype=np.uint32).view(np.float32)


def bits(a) -> np.ndarray:
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


# ---- scalar primitives ------------------------------------------------------

def _undecided_call(name, x):
    flag = C.c_int32(0)
    v = getattr(lib(), name)(float(np.float32(x)), C.byref(flag))
    return np.float32(v), bool(flag.value)


def exp(x):
    return _undecided_call("oracle_exp", x)[0]


def rsqrt(x):
    return _undecided_call("oracle_rsqrt", x)[0]


def silu(x):
    return _undecided_call("oracle_silu", x)[0]


def maximum(a, b):
    return np.float32(lib().oracle_maximum(float(np.float32(a)), float(np.float32(b))))


def f32_to_bf16(x: np.ndarray) -> np.ndarray:
    """Vectorised RNE rounding to bf16 bits (canonical NaN 0x7fc0)."""
    b = bits(x).astype(np.uint64)
    r = ((b + 0x7FFF + ((b >> 16) & 1)) >> 16).astype(np.uint16)
    r[np.isnan(np.asarray(x, dtype=np.float32))] = 0x7FC0
    return r


def bf16_to_f32(b: np.ndarray) -> np.ndarray:
    return (np.asarray(b, dtype=np.uint16).astype(np.uint32) << 16).view(np.float32)


# ---- reductions -------------------------------------------------------------

def _rows_call(name, x, *args):
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, count = (1, x.size) if x.ndim == 1 else x.shape
    out = np.zeros(rows, dtype=np.float32)
    st = getattr(lib(), name)(_ptr(x), rows, count, *args, _ptr(out))
    return st, out


def strict_sum(x):
    return _rows_call("oracle_strict_sum", x)


def partitioned_sum(x, partitions, per):
    return _rows_call("oracle_partitioned_sum", x, partitions, per)


def cooperative_sum(x, participants, per, rounds, participant_major=False):
    return _rows_call("oracle_cooperative_sum", x, participants, per, rounds,
                      1 if participant_major else 0)


def strict_max(x):
    return _rows_call("oracle_strict_max", x)


def compose_fold(seq, threads, k, rounds, op=0):
    seq = np.ascontiguousarray(seq, dtype=np.float32)
    out = np.zeros(1, dtype=np.float32)
    st = lib().oracle_compose_fold(_ptr(seq), seq.size, threads, k, rounds, op, _ptr(out))
    return st, out[0]


def grid_fold(x, grouping, op=0, nthreads=1):
    """Evaluate the backend's declared grid grouping (dict or object with
    partitions/threads/k/rounds/combine_threads/combine_k/combine_rounds)."""
    g = grouping if isinstance(grouping, dict) else grouping.__dict__
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, count = (1, x.size) if x.ndim == 1 else x.shape
    out = np.zeros(rows, dtype=np.float32)
    st = lib().oracle_grid_fold(_ptr(x), rows, count, g["partitions"], g["threads"], g["k"],
                                g["rounds"], g["combine_threads"], g["combine_k"],
                                g["combine_rounds"], op, nthreads, _ptr(out))
    return st, out


# ---- row families -----------------------------------------------------------

def rms_norm_f32(x, w, eps_bits=0x358637BD, nthreads=1):
    x = np.ascontiguousarray(x, dtype=np.float32)
    w = np.ascontiguousarray(w, dtype=np.float32)
    rows, extent = x.shape
    stride = 0 if w.ndim == 1 else extent
    y = np.zeros_like(x)
    st = lib().oracle_rms_norm_f32(_ptr(x), _ptr(w), stride, rows, extent, eps_bits, _ptr(y), nthreads)
    return st, y


def rms_norm_bf16(x, w, eps_bits=0x358637BD, nthreads=1):
    x = np.ascontiguousarray(x, dtype=np.uint16)
    w = np.ascontiguousarray(w, dtype=np.uint16)
    rows, extent = x.shape
    stride = 0 if w.ndim == 1 else extent
    y = np.zeros_like(x)
    st = lib().oracle_rms_norm_bf16(_ptr(x), _ptr(w), stride, rows, extent, eps_bits, _ptr(y), nthreads)
    return st, y


def softmax_f32(x, causal_period=0, row_offset=0, nthreads=1):
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, extent = x.shape
    y = np.zeros_like(x)
    st = lib().oracle_softmax_f32(_ptr(x), rows, extent, causal_period, row_offset, _ptr(y), nthreads)
    return st, y


def silu_f32(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    y = np.zeros_like(x)
    st = lib().oracle_silu_f32(_ptr(x), x.size, _ptr(y))
    return st, y


def scale_bias_f32(x, a, b):
    x = np.ascontiguousarray(x, dtype=np.float32)
    a = np.ascontiguousarray(np.atleast_1d(a), dtype=np.float32)
    b = np.ascontiguousarray(np.atleast_1d(b), dtype=np.float32)
    y = np.zeros_like(x)
    st = lib().oracle_scale_bias_f32(_ptr(x), x.size, _ptr(a), int(a.size == 1 and x.size != 1),
                                     _ptr(b), int(b.size == 1 and x.size != 1), _ptr(y))
    return st, y


def gather_rows(table, ids):
    table = np.ascontiguousarray(table)
    ids = np.ascontiguousarray(ids)
    rows = table.shape[0]
    row_bytes = table.strides[0] if table.ndim > 1 else table.itemsize
    out = np.zeros((ids.size,) + table.shape[1:], dtype=table.dtype)
    err = OracleError()
    st = lib().oracle_gather_rows(_ptr(table), rows, row_bytes, _ptr(ids),
                                  int(ids.dtype == np.uint32), ids.size, _ptr(out), C.byref(err))
    return st, out, err


def quantize_i8_rows(x, nthreads=1):
    x = np.ascontiguousarray(x, dtype=np.float32)
    rows, extent = x.shape
    codes = np.zeros((rows, extent), dtype=np.int8)
    scales = np.zeros(rows, dtype=np.float32)
    err = OracleError()
    st = lib().oracle_quantize_i8_rows(_ptr(x), rows, extent, _ptr(codes), _ptr(scales),
                                       C.byref(err), nthreads)
    return st, codes, scales, err


def dequantize_i8_rows(codes, scales, nthreads=1):
    codes = np.ascontiguousarray(codes, dtype=np.int8)
    scales = np.ascontiguousarray(scales, dtype=np.float32)
    rows, extent = codes.shape
    y = np.zeros((rows, extent), dtype=np.float32)
    st = lib().oracle_dequantize_i8_rows(_ptr(codes), _ptr(scales), rows, extent, _ptr(y), nthreads)
    return st, y


def quantize_affine_u8(x, scale, zero_point, maximum):
    x = np.ascontiguousarray(x, dtype=np.float32)
    codes = np.zeros(x.shape, dtype=np.uint8)
    err = OracleError()
    st = lib().oracle_quantize_affine_u8(_ptr(x), x.size, float(np.float32(scale)), zero_point,
                                         maximum, _ptr(codes), C.byref(err))
    return st, codes, err


def dequantize_affine_u8(codes, scale, zero_point):
    codes = np.ascontiguousarray(codes, dtype=np.uint8)
    y = np.zeros(codes.shape, dtype=np.float32)
    st = lib().oracle_dequantize_affine_u8(_ptr(codes), codes.size, float(np.float32(scale)),
                                           zero_point, _ptr(y))
    return st, y


def contract_f32(a, b, nthreads=1):
    a = np.ascontiguousarray(a, dtype=np.float32)
    b = np.ascontiguousarray(b, dtype=np.float32)
    m, k = a.shape
    n = b.shape[0]
    c = np.zeros((m, n), dtype=np.float32)
    st = lib().oracle_contract_f32(_ptr(a), _ptr(b), m, n, k, _ptr(c), nthreads)
    return st, c


def gemm_bf16_silu(a, b, row_begin=0, row_end=None, apply_silu=True, nthreads=1):
    a = np.ascontiguousarray(a, dtype=np.uint16)
    b = np.ascontiguousarray(b, dtype=np.uint16)
    m, k = a.shape
    n = b.shape[0]
    row_end = m if row_end is None else row_end
    c = np.zeros((row_end - row_begin, n), dtype=np.uint16)
    st = lib().oracle_gemm_bf16_silu(_ptr(a), _ptr(b), m, n, k, row_begin, row_end,
                                     int(apply_silu), _ptr(c), nthreads)
    return st, c
