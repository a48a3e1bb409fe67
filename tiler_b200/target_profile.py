"""The CUDA target profile and payload provenance a Rust ``tiler-cuda`` crate
would declare, stated as data.

The reference builds a target profile with ``TargetProfileBuilder``
(crates/tiler-compiler/src/target/builder.rs:97-1439; a non-Metal precedent is
crates/tiler-build/tests/custom_backend/profile.rs:111-253) and ships each
backend payload with ``PayloadMetadata`` provenance
(crates/tiler-artifact/src/program/codec/payload.rs:228-424).  Neither can be
built here (no cargo), so this module states the rows this backend's kernels
honour, in the builder's vocabulary, for the crate to transcribe:

* capability rows from the device facts (``tiler_cuda_device_facts_query``);
* numerics rows: what every kernel in ``csrc/`` does (IEEE RN per operation,
  subnormals preserved, no contraction, no reassociation outside a declared
  grouping, no approximate intrinsics on a result path);
* dtype dispatchability (f32; bf16 through the widening families);
* the subgroup realization the grouped fold uses (width 32, f32, XOR
  shuffle butterfly);
* the payload provenance: nvcc, ``sm_100a``, the Makefile's flags, and the
  entry list of the library's own registry.
"""
from __future__ import annotations

import os
import re
import shutil
import subprocess

from . import _native as N

PROFILE_KEY = "tiler.cuda.sm_100a"
PRODUCER = ("tiler-cuda", 1)
# external guarantees the rows rest on (not measurements of the running device)
NORMATIVE_REFERENCES = ("ieee.754.2019.binary32", "nvidia.ptx-isa.sm_100a")

# B200 / compute capability 10.0 limits used when no device is present
SM100_FACTS = {
    "max_threads_per_block": 1024,
    "warp_size": 32,
    "smem_per_block_optin": 232448,
    "cc_major": 10,
    "cc_minor": 0,
}
GRID_AXIS_THREADS = (1 << 31) - 1  # gridDim.x limit, in blocks of >= 1 thread
BUFFER_BINDINGS = 16               # the widest entry binds 12 pointers (gemm allgather: 8 blocks + a, b, status)


def _facts(facts: dict | None) -> dict:
    out = dict(SM100_FACTS)
    if facts:
        out.update({k: facts[k] for k in SM100_FACTS if k in facts})
    return out


def capability_rows(facts: dict | None = None) -> list:
    f = _facts(facts)
    return [
        ("max_threads_per_grid_axis", GRID_AXIS_THREADS),
        ("max_threads_per_workgroup", f["max_threads_per_block"]),
        ("max_buffer_bindings_per_entry", BUFFER_BINDINGS),
        ("index_arithmetic", "CompleteU64"),
        ("device_address_width", "Bits64"),
        ("device_memory", True),
        ("local_memory_bytes", f["smem_per_block_optin"]),
    ]


def numerics_rows(subject: str = "f32") -> list:
    """(axis, behaviour, support) rows for one scalar subject."""
    rows = []
    for axis in ("input_subnormals", "result_subnormals"):
        rows.append((axis, "Preserve", "Exact"))  # built without -ftz / fast-math
        rows.append((axis, "FlushToZero{PreservesSign}", "Unsupported"))
        rows.append((axis, "FlushToZero{AlwaysPositive}", "Unsupported"))
    rows += [
        ("contraction", "Forbidden", "Exact"),  # -fmad=false; separate roundings spelled out
        ("contraction", "Permitted", "Unsupported"),
        ("reassociation", "Forbidden", "Exact"),
        # reassociation only as the grouping a provider proposal declares (the
        # grid grouping of tiler_cuda_sum_f32 / _max_f32), never elsewhere
        ("reassociation", "Permitted(declared grouping)", "Exact"),
        ("permutation", "Forbidden", "Exact"),
        ("signed_zero", "Forbidden", "Exact"),
        ("reciprocal_transform", "Forbidden", "Exact"),  # out = e * r is the reference's own form
        ("approximate_intrinsics", "Forbidden", "Exact"),  # hardware exp only behind a certification
        ("nan_assumptions", "MakeNoAssumption", "Exact"),
        ("infinity_assumptions", "MakeNoAssumption", "Exact"),
    ]
    return [(subject,) + r for r in rows]


def dtype_rows() -> list:
    return [("f32", "Dispatchable"), ("bf16", "Dispatchable")]


def subgroup_rows(facts: dict | None = None) -> list:
    f = _facts(facts)
    return [({"width": f["warp_size"], "element": "F32", "combine": "XorShuffle"}, "Supported")]


def target_profile(facts: dict | None = None) -> dict:
    """The whole profile as data (declaration name -> rows)."""
    return {
        "key": PROFILE_KEY,
        "source": {"producer": PRODUCER, "references": NORMATIVE_REFERENCES},
        "capability": capability_rows(facts),
        "numerics": numerics_rows("f32"),
        "dtype_dispatchability": dtype_rows(),
        "subgroup_realization": subgroup_rows(facts),
    }


def _makefile_flags() -> tuple:
    mk = os.path.join(os.path.dirname(os.path.abspath(__file__)), "csrc", "Makefile")
    text = open(mk).read().replace("\\\n", " ")
    var = dict(re.findall(r"^(\w+)\s*:=\s*(.*)$", text, flags=re.M))
    arch = var.get("ARCH", "").split()
    compile_flags = [t for t in var.get("NVCCFLAGS", "").split() if t != "$(ARCH)"]
    compile_flags[compile_flags.index("-lineinfo") + 1:compile_flags.index("-lineinfo") + 1] = arch
    return compile_flags, var.get("QUADMATH", "").split()


def _nvcc_version() -> str:
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    try:
        out = subprocess.run([nvcc, "--version"], capture_output=True, text=True, timeout=30).stdout
    except (OSError, subprocess.SubprocessError):
        return "nvcc (version unavailable)"
    m = re.search(r"release [\d.]+, V([\d.]+)", out)
    return f"nvcc {m.group(1)}" if m else "nvcc"


def payload_provenance() -> dict:
    """PayloadMetadata provenance fields (payload.rs:228-424) for
    libtiler_cuda.so."""
    compile_flags, link_flags = _makefile_flags()
    return {
        "toolchain": _nvcc_version(),
        "target": "sm_100a",
        "family": "tiler-cuda",
        "language": "cuda-c++17",
        "platform": "Unversioned",
        "components": ["libtiler_cuda.so"],
        "compile_flags": compile_flags,
        "link_flags": link_flags,
    }


def payload_entries() -> list:
    """[{entry_key, symbol}] from the library's own registry."""
    L = N.lib()
    out = []
    for i in range(int(L.tiler_cuda_entry_count())):
        sym = L.tiler_cuda_entry_symbol(i).decode()
        out.append({"entry_key": sym.split(".", 1)[1], "symbol": sym})
    return out
