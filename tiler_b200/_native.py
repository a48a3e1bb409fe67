"""ctypes binding of libtiler_cuda.so (the C-ABI declared in include/tiler_cuda.h).

The shared library is built in-tree (``tiler_b200/libtiler_cuda.so``, see
``tiler_b200/build.py``).  There is no fallback: if the library is missing or
cannot be loaded, every entry point raises.
"""
from __future__ import annotations

import ctypes as C
import os
import threading

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "libtiler_cuda.so")
# The payload code a plan artifact carries: the same kernels as an sm_100a cubin.
CUBIN_PATH = os.path.join(HERE, "tiler_kernels.cubin")

OK = 0
INVALID_APPLICATION = 1
SHAPE_TOO_LARGE = 2
GATHER_INDEX_OUT_OF_BOUNDS = 3
NAN_INPUT = 4
UNDECIDED = 5
DEVICE_ERROR = 6
TIMEOUT = 7
UNSUPPORTED = 8
SCALE_DOMAIN = 9
PAYLOAD_REFUSED = 10
WORKSPACE_TOO_SMALL = 11


class Status(C.Structure):
    _fields_ = [("error_key", C.c_uint64), ("value_key", C.c_uint64), ("undecided", C.c_uint32),
                ("timeouts", C.c_uint32), ("reserved", C.c_uint64)]


class Error(C.Structure):
    _fields_ = [("code", C.c_int32), ("undecided", C.c_uint32), ("timeouts", C.c_uint32), ("pad", C.c_uint32),
                ("position", C.c_uint64), ("value", C.c_int64)]


class DeviceFacts(C.Structure):
    _fields_ = [("device", C.c_int32), ("cc_major", C.c_int32), ("cc_minor", C.c_int32),
                ("sm_count", C.c_int32), ("warp_size", C.c_int32), ("max_threads_per_block", C.c_int32),
                ("smem_per_block_optin", C.c_int64), ("l2_bytes", C.c_int64), ("global_mem_bytes", C.c_int64),
                ("name", C.c_char * 96)]


class EntryProps(C.Structure):
    _fields_ = [("num_regs", C.c_int32), ("max_threads_per_block", C.c_int32), ("static_smem_bytes", C.c_int64),
                ("dynamic_smem_bytes", C.c_int64), ("threads_per_block", C.c_int32), ("pad", C.c_int32)]


class Grouping(C.Structure):
    _fields_ = [("partitions", C.c_uint64), ("threads", C.c_uint32), ("k", C.c_uint32), ("rounds", C.c_uint32),
                ("combine_threads", C.c_uint32), ("combine_k", C.c_uint32), ("combine_rounds", C.c_uint32)]

    def as_dict(self) -> dict:
        return {f: int(getattr(self, f)) for f, _ in self._fields_}

    @classmethod
    def from_dict(cls, d: dict) -> "Grouping":
        g = cls()
        for f, _ in cls._fields_:
            setattr(g, f, int(d.get(f, 0)))
        return g


P = C.c_void_p
u64, i64, u32, i32 = C.c_uint64, C.c_int64, C.c_uint32, C.c_int32

SIGNATURES = {
    "tiler_cuda_abi_version": (u32, []),
    "tiler_cuda_context_create": (i32, [i32, C.POINTER(P)]),
    "tiler_cuda_context_destroy": (i32, [P]),
    "tiler_cuda_device_facts_query": (i32, [P, C.POINTER(DeviceFacts)]),
    "tiler_cuda_status_string": (C.c_char_p, [i32]),
    "tiler_cuda_payload_validate": (i32, [P, C.c_char_p, u32, C.POINTER(C.c_char_p), u32, C.POINTER(u32)]),
    "tiler_cuda_entry_count": (u32, []),
    "tiler_cuda_entry_symbol": (C.c_char_p, [u32]),
    "tiler_cuda_entry_query": (i32, [P, C.c_char_p, C.POINTER(EntryProps)]),
    "tiler_cuda_module_load": (i32, [P, C.c_char_p, u64, C.POINTER(P)]),
    "tiler_cuda_sum_exchange_buffer_bytes": (u64, [u64]),
    "tiler_cuda_sum_f32_exchange": (i32, [P, P, P, P, u64, u32, u32, P, u32, P]),
    "tiler_cuda_module_entry": (i32, [P, C.c_char_p, C.POINTER(EntryProps)]),
    "tiler_cuda_context_bind_module": (i32, [P, P]),
    "tiler_cuda_module_launch_count": (i32, [P, C.POINTER(u64)]),
    "tiler_cuda_module_unload": (i32, [P]),
    "tiler_cuda_status_reset": (i32, [P, P]),
    "tiler_cuda_status_fetch": (i32, [P, P, C.POINTER(Error)]),
    "tiler_cuda_status_decode": (i32, [C.POINTER(Status), C.POINTER(Error)]),
    "tiler_cuda_sync": (i32, [P, u64]),
    "tiler_cuda_plan_grouping": (i32, [P, u64, u64, C.POINTER(Grouping)]),
    "tiler_cuda_plan_grouping_for": (i32, [i32, u64, u64, C.POINTER(Grouping)]),
    "tiler_cuda_grouped_workspace_bytes": (u64, [u64, C.POINTER(Grouping)]),
    "tiler_cuda_sum_f32": (i32, [P, P, P, u64, u64, C.POINTER(Grouping), P, u64, P]),
    "tiler_cuda_max_f32": (i32, [P, P, P, u64, u64, C.POINTER(Grouping), P, u64, P]),
    "tiler_cuda_sum_f32_no_alloc": (i32, [P, P, P, u64, u64, C.POINTER(Grouping), P]),
    "tiler_cuda_strict_sum_f32": (i32, [P, P, P, u64, u64, P]),
    "tiler_cuda_partitioned_sum_f32": (i32, [P, P, P, u64, u64, u64, u64, P, u64, P]),
    "tiler_cuda_partitioned_workspace_bytes": (u64, [u64, u64]),
    "tiler_cuda_cooperative_sum_f32": (i32, [P, P, P, u64, u64, u64, u64, u64, i32, P]),
    "tiler_cuda_rms_norm_f32": (i32, [P, P, P, P, P, i64, u64, u64, u32, P]),
    "tiler_cuda_rms_norm_bf16": (i32, [P, P, P, P, P, i64, u64, u64, u32, P]),
    "tiler_cuda_rms_norm_host": (i32, [P, P, P, i32, P, P, P, i64, u64, u64, u32, P, P, u64]),
    "tiler_cuda_rms_norm_quantize_i8": (i32, [P, P, P, P, P, i64, u64, u64, u32, P, P]),
    "tiler_cuda_softmax_masked_f32": (i32, [P, P, P, P, u64, u64, P, u64, u64, P]),
    "tiler_cuda_bounded_wait_selftest": (i32, [P, P, P, u64]),
    "tiler_cuda_ipc_export": (i32, [P, P, P, P]),
    "tiler_cuda_ipc_open": (i32, [P, P, u64, P]),
    "tiler_cuda_ipc_close": (i32, [P, P, u64]),
    "tiler_cuda_gemm_bf16_allgather": (i32, [P, P, P, P, P, u64, u64, u64, i32, u32, u32, P]),
    "tiler_cuda_gemm_bf16_allgather_multicast": (i32, [P, P, P, P, P, u64, u64, u64, i32, u32, u32, P, P]),
    "tiler_cuda_softmax_f32": (i32, [P, P, P, P, u64, u64, u64, u64, P]),
    "tiler_cuda_quantize_i8_rows": (i32, [P, P, P, P, u64, u64, P, P]),
    "tiler_cuda_dequantize_i8_rows": (i32, [P, P, P, P, P, u64, u64, P]),
    "tiler_cuda_quantize_affine_u8": (i32, [P, P, P, P, u64, u32, u32, u32, P]),
    "tiler_cuda_dequantize_affine_u8": (i32, [P, P, P, P, u64, u32, u32, u32, P]),
    "tiler_cuda_silu_f32": (i32, [P, P, P, P, u64, P]),
    "tiler_cuda_scale_bias_f32": (i32, [P, P, P, u64, P, i32, P, i32, P]),
    "tiler_cuda_gather_rows": (i32, [P, P, P, P, u64, u64, P, i32, u64, P]),
    "tiler_cuda_contract_f32": (i32, [P, P, P, P, u64, u64, u64, P]),
    "tiler_cuda_gemm_bf16": (i32, [P, P, P, P, P, u64, u64, u64, i32, P, u64]),
}

_lib = None
_lock = threading.Lock()


class LibraryMissing(RuntimeError):
    pass


def lib() -> C.CDLL:
    """Loads libtiler_cuda.so, raising if it is absent (no fallback path)."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.exists(LIB_PATH):
                raise LibraryMissing(
                    f"{LIB_PATH} is missing: build it with `python -m tiler_b200.build` (nvcc, sm_100a)")
            L = C.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(L, name)
                fn.restype = res
                fn.argtypes = args
            _lib = L
    return _lib


def status_string(code: int) -> str:
    s = lib().tiler_cuda_status_string(code)
    return s.decode() if s else f"status {code}"
