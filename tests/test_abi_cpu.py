"""CPU-side checks of the C-ABI library: it loads, exports every symbol that
include/tiler_cuda.h declares, and its host-only functions behave (no GPU
compute here)."""
import ctypes as C
import os
import re
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
HEADER = os.path.join(ROOT, "include", "tiler_cuda.h")


@pytest.fixture(scope="module")
def native():
    from tiler_b200 import _native
    if not os.path.exists(_native.LIB_PATH):
        from tiler_b200.build import build
        build()
    return _native


def declared_functions():
    text = open(HEADER).read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(tiler_cuda_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(native):
    names = declared_functions()
    assert len(names) >= 30
    out = subprocess.run(["nm", "-D", "--defined-only", native.LIB_PATH], capture_output=True, text=True).stdout
    exported = set(re.findall(r"\bT (tiler_cuda_[a-z0-9_]+)", out))
    missing = [n for n in names if n not in exported]
    assert not missing, missing
    L = native.lib()
    for n in names:
        assert getattr(L, n)


def test_every_declared_symbol_has_a_ctypes_signature(native):
    assert set(declared_functions()) == set(native.SIGNATURES)


def test_host_only_functions(native):
    L = native.lib()
    assert L.tiler_cuda_abi_version() == 1
    assert L.tiler_cuda_status_string(3) == b"gather index out of bounds"
    n = L.tiler_cuda_entry_count()
    syms = [L.tiler_cuda_entry_symbol(i).decode() for i in range(n)]
    assert "tiler_cuda.rms_norm_f32" in syms and "tiler_cuda.gemm_bf16" in syms
    assert L.tiler_cuda_entry_symbol(n) is None


def test_status_decode_mirrors_the_reference_refusal(native):
    L = native.lib()
    st = native.Status(error_key=(4000 << 8) | 3, value_key=(4000 << 32) | (0xFFFFFFF9), undecided=0, timeouts=0)
    err = native.Error()
    assert L.tiler_cuda_status_decode(C.byref(st), C.byref(err)) == 3
    assert (err.position, err.value) == (4000, -7)
    clean = native.Status(error_key=2**64 - 1, value_key=2**64 - 1)
    assert L.tiler_cuda_status_decode(C.byref(clean), C.byref(err)) == 0
    timed = native.Status(error_key=2**64 - 1, value_key=2**64 - 1, timeouts=2)
    assert L.tiler_cuda_status_decode(C.byref(timed), C.byref(err)) == native.TIMEOUT


def test_grouped_workspace_bytes(native):
    L = native.lib()
    g = native.Grouping(partitions=1024, threads=512, k=4, rounds=8, combine_threads=512, combine_k=2,
                        combine_rounds=1)
    assert L.tiler_cuda_grouped_workspace_bytes(1, C.byref(g)) == 4096 + 4
    g.partitions = 1
    assert L.tiler_cuda_grouped_workspace_bytes(1, C.byref(g)) == 0


def test_context_create_refuses_without_a_device(native):
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a device is present")
    except ImportError:
        pass
    L = native.lib()
    h = C.c_void_p()
    assert L.tiler_cuda_context_create(0, C.byref(h)) == native.DEVICE_ERROR
    assert h.value is None
    # entry points refuse a null context before touching the device
    assert L.tiler_cuda_rms_norm_f32(None, None, None, None, None, 0, 1, 1, 0x358637BD, None) == 1


def test_no_closed_copy_calls_in_sources():
    pat = re.compile(r"Memcpy\w*Batch")
    for d, _, files in os.walk(os.path.join(ROOT, "tiler_b200")):
        for f in files:
            if f.endswith((".cu", ".cuh", ".h", ".py", ".cpp")):
                assert not pat.search(open(os.path.join(d, f)).read()), f
