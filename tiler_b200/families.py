"""Torch-facing entry points for the registered operation families.

Each function validates on the host, launches the sm_100a kernel through the
C-ABI on the current CUDA stream, and (``check=True``, the default) waits for
the device status word and raises :class:`TilerCudaError` with the same
refusal the reference's evaluator would give (an out-of-range gather index
with its position / value / extent, a NaN quantize input, ...).  Names and
argument meanings follow crates/tiler-reference (cited per function).

Tensors must be CUDA tensors, contiguous, of the stated dtype; torch supplies
memory and streams only - every byte of arithmetic happens in libtiler_cuda.
"""
from __future__ import annotations

import ctypes as C
import threading

import torch

from . import _native as N


class TilerCudaError(RuntimeError):
    """A refusal from the backend: ``code`` is one of the TILER_CUDA_* status
    codes; for a gather refusal ``position``/``value``/``extent`` mirror
    ReferenceOperationError::GatherIndexOutOfBounds
    (crates/tiler-reference/src/structural.rs:569-585)."""

    def __init__(self, code: int, what: str = "", position=None, value=None, extent=None):
        self.code, self.position, self.value, self.extent = code, position, value, extent
        detail = f" at position {position}" if position is not None else ""
        if value is not None:
            detail += f" (value {value}, extent {extent})"
        super().__init__(f"{what}: {N.status_string(code)}{detail}")


def _check(code: int, what: str):
    if code != N.OK:
        raise TilerCudaError(code, what)


_ctx_lock = threading.Lock()
_contexts: dict = {}


def context(device=None) -> int:
    """The per-device tiler_cuda_context (bind_execution_context)."""
    dev = torch.cuda.current_device() if device is None else int(device)
    with _ctx_lock:
        if dev not in _contexts:
            handle = C.c_void_p()
            _check(N.lib().tiler_cuda_context_create(dev, C.byref(handle)), "context_create")
            _contexts[dev] = handle.value
        return _contexts[dev]


def device_facts(device=None) -> dict:
    f = N.DeviceFacts()
    _check(N.lib().tiler_cuda_device_facts_query(context(device), C.byref(f)), "device_facts")
    return {k: (getattr(f, k).decode() if k == "name" else int(getattr(f, k))) for k, _ in f._fields_}


def _stream() -> int:
    return torch.cuda.current_stream().cuda_stream


def _ptr(t) -> int:
    if t is None:
        return 0
    if not t.is_cuda:
        raise ValueError("tiler_b200 families take CUDA tensors")
    if not t.is_contiguous():
        raise ValueError("tiler_b200 families take contiguous tensors")
    return t.data_ptr()


class StatusWord:
    """A device-resident tiler_cuda_status (32 bytes)."""

    def __init__(self, device=None):
        self.buf = torch.empty(4, dtype=torch.int64, device=device or "cuda")

    @property
    def ptr(self) -> int:
        return self.buf.data_ptr()

    def reset(self):
        _check(N.lib().tiler_cuda_status_reset(_stream(), self.ptr), "status_reset")

    def fetch(self) -> N.Error:
        err = N.Error()
        N.lib().tiler_cuda_status_fetch(_stream(), self.ptr, C.byref(err))
        return err


_status_cache: dict = {}


def _status() -> StatusWord:
    dev = torch.cuda.current_device()
    if dev not in _status_cache:
        _status_cache[dev] = StatusWord(device=f"cuda:{dev}")
    s = _status_cache[dev]
    s.reset()
    return s


def _raise_from(st: StatusWord, what: str, extent=None):
    err = st.fetch()
    if err.code != N.OK:
        value = int(err.value) if err.code == N.GATHER_INDEX_OUT_OF_BOUNDS else None
        raise TilerCudaError(int(err.code), what, position=int(err.position) if err.code not in (
            N.UNDECIDED, N.TIMEOUT) else None, value=value, extent=extent if value is not None else None)


# ---- reductions ---------------------------------------------------------------

def plan_grouping(rows: int, count: int, device=None) -> dict:
    """PhysicalImplementationProvider::propose for a reduction
    (crates/tiler-compiler/src/frontier.rs:3828-4040): the grouping this
    backend declares for a [rows, count] reduction over the last axis."""
    g = N.Grouping()
    _check(N.lib().tiler_cuda_plan_grouping(context(device), rows, count, C.byref(g)), "plan_grouping")
    return g.as_dict()


def grouped_workspace(rows: int, grouping: dict, device=None) -> torch.Tensor:
    """allocate_dispatch: a zeroed workspace for the grouped fold (partials and
    per-row completion tickets, which the kernel leaves zero again)."""
    g = N.Grouping.from_dict(grouping)
    n = int(N.lib().tiler_cuda_grouped_workspace_bytes(rows, C.byref(g)))
    return torch.zeros(max(n, 16), dtype=torch.uint8, device=device or "cuda")


def _reduce(fn_name: str, x: torch.Tensor, grouping, workspace):
    assert x.dtype == torch.float32
    rows = _rows(x)
    count = x.numel() if x.dim() <= 1 else x.shape[-1]
    if grouping is None:
        grouping = plan_grouping(rows, count) if count else {"partitions": 1, "threads": 32, "k": 1, "rounds": 1}
    g = N.Grouping.from_dict(grouping)
    if workspace is None:
        workspace = grouped_workspace(rows, grouping, device=x.device)
    out = torch.empty(rows if x.dim() > 1 else 1, dtype=torch.float32, device=x.device)
    code = getattr(N.lib(), fn_name)(context(), _stream(), _ptr(x), rows, count, C.byref(g), _ptr(workspace),
                                     workspace.numel(), _ptr(out))
    _check(code, fn_name)
    return out if x.dim() > 1 else out.reshape(())


def sum_f32(x: torch.Tensor, grouping: dict | None = None, workspace=None) -> torch.Tensor:
    """Sum over the last axis under a declared grouping (strict_partitioned /
    ADR-0100 composition; crates/tiler-reference/src/evaluate.rs:612-1158)."""
    return _reduce("tiler_cuda_sum_f32", x, grouping, workspace)


def max_f32(x: torch.Tensor, grouping: dict | None = None, workspace=None) -> torch.Tensor:
    """Governed maximum fold over the last axis (maximum_f32, softmax.rs:168-186)."""
    return _reduce("tiler_cuda_max_f32", x, grouping, workspace)


def _rows(x: torch.Tensor) -> int:
    if x.dim() <= 1:
        return 1
    r = 1
    for d in x.shape[:-1]:
        r *= d
    return r


def strict_sum_f32(x: torch.Tensor) -> torch.Tensor:
    """strict_sum (evaluate.rs:498-589): one serial fold per row."""
    rows = _rows(x)
    count = x.numel() if x.dim() <= 1 else x.shape[-1]
    out = torch.empty(rows, dtype=torch.float32, device=x.device)
    _check(N.lib().tiler_cuda_strict_sum_f32(context(), _stream(), _ptr(x), rows, count, _ptr(out)), "strict_sum")
    return out


def partitioned_sum_f32(x: torch.Tensor, partitions: int, per_partition: int) -> torch.Tensor:
    """strict_partitioned_sum (evaluate.rs:749-832)."""
    rows = _rows(x)
    count = x.numel() if x.dim() <= 1 else x.shape[-1]
    ws = torch.empty(max(1, rows * partitions), dtype=torch.float32, device=x.device)
    out = torch.empty(rows, dtype=torch.float32, device=x.device)
    _check(N.lib().tiler_cuda_partitioned_sum_f32(context(), _stream(), _ptr(x), rows, count, partitions,
                                                  per_partition, _ptr(ws), ws.numel() * 4, _ptr(out)),
           "partitioned_sum")
    return out


def cooperative_sum_f32(x: torch.Tensor, participants: int, per_partition: int, rounds: int,
                        participant_major: bool = False) -> torch.Tensor:
    """cooperative_grouped_sum (evaluate.rs:936-1158)."""
    rows = _rows(x)
    count = x.numel() if x.dim() <= 1 else x.shape[-1]
    out = torch.empty(rows, dtype=torch.float32, device=x.device)
    _check(N.lib().tiler_cuda_cooperative_sum_f32(context(), _stream(), _ptr(x), rows, count, participants,
                                                  per_partition, rounds, int(participant_major), _ptr(out)),
           "cooperative_sum")
    return out


# ---- row families -------------------------------------------------------------

EPS_1E6_BITS = 0x358637BD  # RMS_NORM_F32_REFERENCE_EPS_BITS (tiler-ir semantic/rms_norm.rs)


def rms_norm(x: torch.Tensor, w: torch.Tensor, eps_bits: int = EPS_1E6_BITS, out=None, check=True) -> torch.Tensor:
    """RmsNormF32Reference (rms_norm.rs:91-132, :453-489); bf16 x/w take the
    binary32 path and round the result once to bf16.  ``w`` is [extent]
    (broadcast) or the shape of ``x``."""
    assert x.dtype in (torch.float32, torch.bfloat16) and w.dtype == x.dtype
    extent = x.shape[-1]
    rows = x.numel() // extent if extent else 0
    stride = 0 if w.dim() == 1 else extent
    y = torch.empty_like(x) if out is None else out
    st = _status() if check else None
    fn = N.lib().tiler_cuda_rms_norm_f32 if x.dtype == torch.float32 else N.lib().tiler_cuda_rms_norm_bf16
    _check(fn(context(), _stream(), st.ptr if st else 0, _ptr(x), _ptr(w), stride, rows, extent, eps_bits,
              _ptr(y)), "rms_norm")
    if st:
        _raise_from(st, "rms_norm")
    return y


def softmax_masked(x: torch.Tensor, mask: torch.Tensor, row_offset: int = 0, out=None, check=True) -> torch.Tensor:
    """softmax(x + mask[(row_offset + r) mod mask_rows]) over the last axis:
    the program's additive mask tensor fused into the softmax."""
    assert x.dtype == torch.float32 and mask.dtype == torch.float32 and mask.shape[-1] == x.shape[-1]
    extent = x.shape[-1]
    rows = x.numel() // extent if extent else 0
    mask_rows = mask.numel() // extent
    y = torch.empty_like(x) if out is None else out
    st = _status() if check else None
    _check(N.lib().tiler_cuda_softmax_masked_f32(context(), _stream(), st.ptr if st else 0, _ptr(x), rows, extent,
                                                 _ptr(mask), mask_rows, row_offset, _ptr(y)), "softmax_masked")
    if st:
        _raise_from(st, "softmax_masked")
    return y


def rms_norm_quantize_i8(x: torch.Tensor, w: torch.Tensor, eps_bits: int = EPS_1E6_BITS, check=True, out=None):
    """Fused RMS norm -> per-row int8 quantize (f32): the codes and scales of
    quantize_i8_rows(rms_norm(x, w)) without writing y.  ``out`` = (codes,
    scales) to write into."""
    assert x.dtype == torch.float32 and w.dtype == torch.float32
    extent = x.shape[-1]
    rows = x.numel() // extent if extent else 0
    stride = 0 if w.dim() == 1 else extent
    if out is None:
        codes = torch.empty(x.shape, dtype=torch.int8, device=x.device)
        scales = torch.empty(x.shape[:-1], dtype=torch.float32, device=x.device)
    else:
        codes, scales = out
    st = _status() if check else None
    _check(N.lib().tiler_cuda_rms_norm_quantize_i8(context(), _stream(), st.ptr if st else 0, _ptr(x), _ptr(w), stride,
                                                   rows, extent, eps_bits, _ptr(codes), _ptr(scales)),
           "rms_norm_quantize_i8")
    if st:
        _raise_from(st, "rms_norm_quantize_i8")
    return codes, scales


def rms_norm_host(x_host: torch.Tensor, w: torch.Tensor, eps_bits: int = EPS_1E6_BITS, out=None, x_dev=None,
                  y_dev=None, chunk_rows: int = 0, check=True) -> torch.Tensor:
    """RMS norm of host rows (tiler_cuda_rms_norm_host): chunked upload,
    kernel and download overlapped on the copy engines.  ``x_host`` (and
    ``out``) should be pinned; ``x_dev`` / ``y_dev`` are device staging
    tensors of x's shape (made here when not given); ``w`` is on the device.
    Returns the host output after the copies have completed."""
    assert x_host.device.type == "cpu" and x_host.dtype in (torch.float32, torch.bfloat16)
    assert x_host.is_contiguous() and (out is None or (out.device.type == "cpu" and out.is_contiguous()))
    assert w.is_cuda and w.dtype == x_host.dtype
    extent = x_host.shape[-1]
    rows = x_host.numel() // extent if extent else 0
    stride = 0 if w.dim() == 1 else extent
    y = torch.empty(x_host.shape, dtype=x_host.dtype, pin_memory=True) if out is None else out
    xd = torch.empty(x_host.shape, dtype=x_host.dtype, device=w.device) if x_dev is None else x_dev
    yd = torch.empty_like(xd) if y_dev is None else y_dev
    st = _status() if check else None
    _check(N.lib().tiler_cuda_rms_norm_host(context(), _stream(), st.ptr if st else 0,
                                            0 if x_host.dtype == torch.float32 else 1, x_host.data_ptr(), _ptr(xd),
                                            _ptr(w), stride, rows, extent, eps_bits, _ptr(yd), y.data_ptr(),
                                            chunk_rows),
           "rms_norm_host")
    torch.cuda.current_stream().synchronize()
    if st:
        _raise_from(st, "rms_norm_host")
    return y


def softmax(x: torch.Tensor, causal_period: int = 0, row_offset: int = 0, out=None, check=True) -> torch.Tensor:
    """SoftmaxF32Reference over the last axis (softmax.rs:99-137, :260-315);
    ``causal_period`` > 0 applies the block-causal additive -inf mask."""
    assert x.dtype == torch.float32
    extent = x.shape[-1]
    rows = x.numel() // extent if extent else 0
    y = torch.empty_like(x) if out is None else out
    st = _status() if check else None
    _check(N.lib().tiler_cuda_softmax_f32(context(), _stream(), st.ptr if st else 0, _ptr(x), rows, extent,
                                          causal_period, row_offset, _ptr(y)), "softmax")
    if st:
        _raise_from(st, "softmax")
    return y


def quantize_i8_rows(x: torch.Tensor, check=True, out=None):
    """Per-row signed strict-affine quantize (extension of quantization.rs:
    188-247, :404-430).  Returns (codes int8, scales f32), written into
    ``out`` = (codes, scales) when given."""
    assert x.dtype == torch.float32
    extent = x.shape[-1]
    rows = x.numel() // extent
    if out is None:
        codes = torch.empty(x.shape, dtype=torch.int8, device=x.device)
        scales = torch.empty(rows, dtype=torch.float32, device=x.device)
    else:
        codes, scales = out
    st = _status() if check else None
    _check(N.lib().tiler_cuda_quantize_i8_rows(context(), _stream(), st.ptr if st else 0, _ptr(x), rows, extent,
                                               _ptr(codes), _ptr(scales)), "quantize_i8_rows")
    if st:
        _raise_from(st, "quantize_i8_rows")
    return codes, scales


def dequantize_i8_rows(codes: torch.Tensor, scales: torch.Tensor, check=True) -> torch.Tensor:
    """dequantize_one with zero point 0 (quantization.rs:440-451)."""
    extent = codes.shape[-1]
    rows = codes.numel() // extent
    y = torch.empty(codes.shape, dtype=torch.float32, device=codes.device)
    st = _status() if check else None
    _check(N.lib().tiler_cuda_dequantize_i8_rows(context(), _stream(), st.ptr if st else 0, _ptr(codes),
                                                 _ptr(scales), rows, extent, _ptr(y)), "dequantize_i8_rows")
    if st:
        _raise_from(st, "dequantize_i8_rows")
    return y


def _f32_bits(v: float) -> int:
    import struct
    return struct.unpack("<I", struct.pack("<f", v))[0]


def quantize_affine_u8(x: torch.Tensor, scale: float, zero_point: int, maximum: int = 255) -> torch.Tensor:
    """The reference's strict-affine quantize (per-tensor scale, unsigned
    U4/U8 codes; quantization.rs:188-247, :404-430)."""
    codes = torch.empty(x.shape, dtype=torch.uint8, device=x.device)
    st = _status()
    _check(N.lib().tiler_cuda_quantize_affine_u8(context(), _stream(), st.ptr, _ptr(x), x.numel(),
                                                 _f32_bits(scale), zero_point, maximum, _ptr(codes)),
           "quantize_affine_u8")
    _raise_from(st, "quantize_affine_u8")
    return codes


def dequantize_affine_u8(codes: torch.Tensor, scale: float, zero_point: int, maximum: int = 255) -> torch.Tensor:
    y = torch.empty(codes.shape, dtype=torch.float32, device=codes.device)
    st = _status()
    _check(N.lib().tiler_cuda_dequantize_affine_u8(context(), _stream(), st.ptr, _ptr(codes), codes.numel(),
                                                   _f32_bits(scale), zero_point, maximum, _ptr(y)),
           "dequantize_affine_u8")
    _raise_from(st, "dequantize_affine_u8")
    return y


# ---- maps ---------------------------------------------------------------------

def silu(x: torch.Tensor, out=None, check=True) -> torch.Tensor:
    """SiluF32Reference (silu.rs:78-180)."""
    y = torch.empty_like(x) if out is None else out
    st = _status() if check else None
    _check(N.lib().tiler_cuda_silu_f32(context(), _stream(), st.ptr if st else 0, _ptr(x), x.numel(), _ptr(y)),
           "silu")
    if st:
        _raise_from(st, "silu")
    return y


def scale_bias(x: torch.Tensor, a: torch.Tensor, b: torch.Tensor, out=None) -> torch.Tensor:
    """multiply-f32 then add-f32 (standard.rs:105-120): y = (x*a)+b, two
    roundings; a rank-0 ``a``/``b`` broadcasts, otherwise it has x's size."""
    for t in (a, b):
        if t.dim() != 0 and t.numel() != x.numel():
            raise ValueError("scale_bias operands are rank-0 or the size of x")
    y = torch.empty_like(x) if out is None else out
    _check(N.lib().tiler_cuda_scale_bias_f32(context(), _stream(), _ptr(x), x.numel(), _ptr(a), int(a.dim() == 0),
                                             _ptr(b), int(b.dim() == 0), _ptr(y)), "scale_bias")
    return y


def gather_rows(table: torch.Tensor, ids: torch.Tensor, out=None, check=True) -> torch.Tensor:
    """GatherF32Reference over axis 0 (structural.rs:513-606): out[i] =
    table[ids[i]] bit-exactly; int32 or uint32 ids."""
    assert ids.dtype in (torch.int32, torch.uint32)
    rows = table.shape[0]
    row_bytes = table[0].numel() * table.element_size() if rows else 0
    y = torch.empty((ids.numel(),) + tuple(table.shape[1:]), dtype=table.dtype, device=table.device) \
        if out is None else out
    st = _status() if check else None
    _check(N.lib().tiler_cuda_gather_rows(context(), _stream(), st.ptr if st else 0, _ptr(table), rows, row_bytes,
                                          _ptr(ids), int(ids.dtype == torch.uint32), ids.numel(), _ptr(y)),
           "gather_rows")
    if st:
        _raise_from(st, "gather_rows", extent=rows)
    return y


# ---- contraction ---------------------------------------------------------------

def contract_f32(a: torch.Tensor, b: torch.Tensor) -> torch.Tensor:
    """`td,od->to` strict f32 contraction (contraction.rs:558-630)."""
    m, k = a.shape
    n = b.shape[0]
    c = torch.empty((m, n), dtype=torch.float32, device=a.device)
    _check(N.lib().tiler_cuda_contract_f32(context(), _stream(), _ptr(a), _ptr(b), m, n, k, _ptr(c)), "contract_f32")
    return c


def ipc_export(t: torch.Tensor):
    """(64-byte cudaIpc handle, offset) of the device allocation holding t."""
    handle = (C.c_uint8 * 64)()
    offset = C.c_uint64(0)
    _check(N.lib().tiler_cuda_ipc_export(context(), _ptr(t), handle, C.byref(offset)), "ipc_export")
    return bytes(handle), offset.value


def ipc_open(handle: bytes, offset: int) -> int:
    """A peer's exported buffer mapped into this process (device pointer)."""
    out = C.c_void_p()
    h = (C.c_uint8 * 64).from_buffer_copy(handle)
    _check(N.lib().tiler_cuda_ipc_open(context(), h, offset, C.byref(out)), "ipc_open")
    return out.value


def ipc_close(ptr: int, offset: int):
    _check(N.lib().tiler_cuda_ipc_close(context(), ptr, offset), "ipc_close")


def gemm_bf16_allgather(a: torch.Tensor, b_shard: torch.Tensor, blocks, rank: int, world: int,
                        epilogue: str = "silu", check=True):
    """The N-sharded contraction with the all-gather fused into the epilogue:
    C_rank = A x B_shard^T goes into block `rank` of every rank's [world, m,
    n_shard] buffer (``blocks``: each rank's buffer as a device pointer in this
    process).  Complete on a peer once a later collective on the stream has
    completed there."""
    assert a.dtype == torch.bfloat16 and b_shard.dtype == torch.bfloat16 and len(blocks) == world
    m, k = a.shape
    n = b_shard.shape[0]
    arr = (C.c_void_p * world)(*blocks)
    st = _status() if check else None
    _check(N.lib().tiler_cuda_gemm_bf16_allgather(context(), _stream(), st.ptr if st else 0, a.data_ptr(),
                                                  b_shard.data_ptr(), m, n, k, 1 if epilogue == "silu" else 0,
                                                  rank, world, arr), "gemm_bf16_allgather")
    if st:
        _raise_from(st, "gemm_bf16_allgather")


def gemm_bf16_allgather_multicast(a: torch.Tensor, b_shard: torch.Tensor, local_buffer: int, multicast_buffer: int,
                                  rank: int, world: int, epilogue: str = "silu", check=True):
    """The fused N-sharded contraction with the all-gather done by multicast
    stores (multimem.st) into an NVLink multicast mapping of every rank's
    [world, m, n_shard] buffer: ``local_buffer`` is this rank's buffer and
    ``multicast_buffer`` its multicast address."""
    assert a.dtype == torch.bfloat16 and b_shard.dtype == torch.bfloat16
    m, k = a.shape
    n = b_shard.shape[0]
    st = _status() if check else None
    _check(N.lib().tiler_cuda_gemm_bf16_allgather_multicast(context(), _stream(), st.ptr if st else 0, a.data_ptr(),
                                                            b_shard.data_ptr(), m, n, k,
                                                            1 if epilogue == "silu" else 0, rank, world,
                                                            local_buffer, multicast_buffer),
           "gemm_bf16_allgather_multicast")
    if st:
        _raise_from(st, "gemm_bf16_allgather_multicast")


def gemm_bf16(a: torch.Tensor, b: torch.Tensor, epilogue: str = "silu", out=None, check=True) -> torch.Tensor:
    """bf16 A[m,k] x B[n,k] on tcgen05 tensor cores, f32 accumulation,
    optional SiLU epilogue, bf16 output [m,n]."""
    assert a.dtype == torch.bfloat16 and b.dtype == torch.bfloat16
    m, k = a.shape
    n = b.shape[0]
    c = torch.empty((m, n), dtype=torch.bfloat16, device=a.device) if out is None else out
    ldc = c.stride(0)
    st = _status() if check else None
    _check(N.lib().tiler_cuda_gemm_bf16(context(), _stream(), st.ptr if st else 0, a.data_ptr(), b.data_ptr(), m, n,
                                        k, 1 if epilogue == "silu" else 0, c.data_ptr(), ldc), "gemm_bf16")
    if st:
        _raise_from(st, "gemm_bf16")
    return c
