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
* the measured cost row ``saturated-parallel-fold-steps``
  (``declare_measured_saturated_parallel_fold_steps``, builder.rs:1344-1375):
  the fold steps the device retires at once when saturated, fitted from a
  dispatch sweep of this library's three sum strategies with the work-span
  model ``sum over stages of (encoder + max(work / P, depth) * step)`` the
  reference's Metal row is fitted with (crates/tiler-build/src/
  metal_declaration.rs:387-421).  Silence (no measurement) declares no row,
  as the reference's cost rows do;
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


COST_ROW_KEY = "cost.saturated-parallel-fold-steps"  # CostRow::SaturatedParallelFoldSteps (rows.rs:399-406)


def fit_work_span(cells: list) -> dict:
    """Least-squares fit of the work-span model
    ``seconds = sum over stages of (encoder + max(work / P, depth) * step)``.

    ``cells``: [{"stages": [(work, depth), ...], "seconds": t}].  P is searched
    on a fine logarithmic grid; for each P the model is linear in (encoder,
    step), solved by least squares on relative residuals.  Returns P, encoder,
    step and the RMS relative residual of the best fit."""
    import numpy as np
    t = np.array([c["seconds"] for c in cells], dtype=np.float64)
    n_st = np.array([len(c["stages"]) for c in cells], dtype=np.float64)
    best = None
    for P in np.exp(np.linspace(np.log(16.0), np.log(1 << 22), 1200)):
        span = np.array([sum(max(w / P, d) for w, d in c["stages"]) for c in cells], dtype=np.float64)
        A = np.stack([n_st / t, span / t], axis=1)  # relative: model / t should be 1
        coef, *_ = np.linalg.lstsq(A, np.ones_like(t), rcond=None)
        if coef[0] < 0 or coef[1] <= 0:
            continue
        res = float(np.sqrt(np.mean((A @ coef - 1.0) ** 2)))
        if best is None or res < best["residual"]:
            best = {"parallel_steps": float(P), "encoder_s": float(coef[0]), "step_s": float(coef[1]),
                    "residual": res}
    if best is None:
        raise ValueError("no admissible work-span fit (negative encoder or step at every P)")
    return best


def measure_fold_cells(fam, torch, repeats: int = 20) -> list:
    """The dispatch sweep on the current device: strict serial sums (one
    thread per row: work rows*count, depth count), partitioned sums (two
    stages: the partials, then their strict fold) and the declared-grouping
    sum (one stage: depth k*rounds + 5 + warp slots per round, then the
    partials).  Inputs stay L2-resident (at most 64 MiB); each cell is the
    mean of ``repeats`` back-to-back launches after a warm-up."""
    dev = "cuda"
    gen = torch.Generator(dev).manual_seed(11)
    cells = []

    def timed(fn):
        # the repeats captured in one CUDA graph, so host call overhead leaves
        # no gaps between the launches being timed
        fn()
        torch.cuda.synchronize()
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, capture_error_mode="thread_local"):
            for _ in range(repeats):
                fn()
        graph.replay()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize()
        e0.record()
        graph.replay()
        e1.record()
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1e3 / repeats

    for rows, count in [(128, 256), (1024, 256), (8192, 256), (65536, 64), (262144, 64), (32, 4096), (512, 2048),
                        (4096, 1024), (16384, 512), (16, 16384)]:
        x = torch.rand(rows, count, device=dev, generator=gen)
        cells.append({"strategy": "strict", "rows": rows, "count": count, "stages": [(rows * count, count)],
                      "seconds": timed(lambda: fam.strict_sum_f32(x))})
        for parts in (16, 64):
            if count % parts == 0 and count // parts >= 4:
                per = count // parts
                cells.append({"strategy": "partitioned", "rows": rows, "count": count, "partitions": parts,
                              "stages": [(rows * count, per), (rows * parts, parts)],
                              "seconds": timed(lambda: fam.partitioned_sum_f32(x, parts, per))})
        del x
    for n in (1 << 16, 1 << 18, 1 << 20, 1 << 22, 1 << 24):
        x = torch.rand(n, device=dev, generator=gen)
        g = fam.plan_grouping(1, n)
        ws = fam.grouped_workspace(1, g)
        slots = g["threads"] // 32
        depth = g["k"] * g["rounds"] + g["rounds"] * (5 + slots) + g["partitions"]
        cells.append({"strategy": "grouped", "rows": 1, "count": n, "grouping": g, "stages": [(n, depth)],
                      "seconds": timed(lambda: fam.sum_f32(x, g, ws))})
        del x, ws
    return cells


def cost_rows(measured_steps: int | None = None) -> list:
    """The cost rows this profile declares: the measured
    saturated-parallel-fold-steps row when a measurement is given, otherwise
    none (a cost row's silence states no preference)."""
    if measured_steps is None:
        return []
    if measured_steps <= 0:
        raise ValueError("a cost row value is positive")
    return [(COST_ROW_KEY, int(measured_steps), "MeasuredEnvironment")]


def target_profile(facts: dict | None = None, measured_fold_steps: int | None = None) -> dict:
    """The whole profile as data (declaration name -> rows)."""
    return {
        "key": PROFILE_KEY,
        "source": {"producer": PRODUCER, "references": NORMATIVE_REFERENCES},
        "capability": capability_rows(facts),
        "numerics": numerics_rows("f32"),
        "dtype_dispatchability": dtype_rows(),
        "subgroup_realization": subgroup_rows(facts),
        "cost": cost_rows(measured_fold_steps),
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
    """PayloadMetadata provenance fields (payload.rs:228-424) for the sm_100a
    code (tiler_kernels.cubin, launched by libtiler_cuda.so)."""
    compile_flags, link_flags = _makefile_flags()
    return {
        "toolchain": _nvcc_version(),
        "target": "sm_100a",
        "family": "tiler-cuda",
        "language": "cuda-c++17",
        "platform": "Unversioned",
        # the tools that produced the code (ToolComponent {role, version})
        "components": [{"role": "cuda-compiler", "version": _nvcc_version().replace("nvcc ", "")}],
        # what the payload carries: the code bytes and the host library that launches them
        "artifacts": ["tiler_kernels.cubin", "libtiler_cuda.so"],
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


def _main():
    import sys
    if "--rust" in sys.argv:
        os.makedirs(os.path.dirname(RUST_PATH), exist_ok=True)
        with open(RUST_PATH, "w") as f:
            f.write(render_rust(measured_fold_steps=MEASURED_FOLD_STEPS))
        print(RUST_PATH)
        return
    # the dispatch sweep and its fit on cuda:0
    import json

    import torch

    from . import families

    cells = measure_fold_cells(families, torch)
    fit = fit_work_span(cells)
    print(json.dumps({"device": torch.cuda.get_device_name(0), "fit": fit,
                      "cost": cost_rows(round(fit["parallel_steps"])),
                      "cells": [{k: v for k, v in c.items() if k != "stages"} | {"stages": c["stages"]}
                                for c in cells]}))


# ---- Rust source for the tiler-cuda crate ---------------------------------------
#
# The rows above rendered as the crate's own declaration code: one
# TargetProfileBuilder call per row (method names and argument types as in
# crates/tiler-compiler/src/target/builder.rs:97-1439, sources as in the
# custom-backend precedent crates/tiler-build/tests/custom_backend/
# profile.rs:102-253 and the measured cost row as in crates/tiler-build/src/
# metal_declaration.rs:1012-1016), and the PayloadMetadata the artifact carries
# for the sm_100a cubin (crates/tiler-artifact/src/program/codec/payload.rs:
# 228-424).  ``tiler_b200/rust/tiler_cuda_profile.rs`` is this rendering,
# regenerated by ``python -m tiler_b200.target_profile --rust``; a CPU test
# keeps the committed file equal to it.

_SUBNORMAL_RUST = {
    "Preserve": "SubnormalMode::Preserve",
    "FlushToZero{PreservesSign}": "SubnormalMode::FlushToZero { zero_sign: FlushedZeroSign::PreservesSign }",
    "FlushToZero{AlwaysPositive}": "SubnormalMode::FlushToZero { zero_sign: FlushedZeroSign::AlwaysPositive }",
}
_PERMISSION_AXES = ("contraction", "reassociation", "permutation", "signed_zero", "reciprocal_transform")
_RUST_DTYPES = {"f32": "F32::resolved_type()", "bf16": "Bf16::resolved_type()"}


def _rust_str(s: str) -> str:
    return '"' + s.replace("\\", "\\\\").replace('"', '\\"') + '"'


def render_rust(facts: dict | None = None, measured_fold_steps: int | None = None, provenance: dict | None = None,
                entries: list | None = None) -> str:
    """The crate's profile and payload declarations as Rust source text."""
    prof = target_profile(facts, measured_fold_steps)
    prov = provenance if provenance is not None else payload_provenance()
    if entries is None:  # the entries whose kernels the code payload carries
        entries = [e for e in payload_entries() if e["symbol"] in MODULE_ENTRY_SYMBOLS]
    ents = entries
    L = []
    w = L.append
    w("// The tiler-cuda crate's target profile and payload metadata.")
    w("// Generated from tiler_b200/target_profile.py by")
    w("// `python -m tiler_b200.target_profile --rust`; regenerate, do not edit.")
    w("")
    w(f"pub const PROFILE_KEY: &str = {_rust_str(prof['key'])};")
    producer, revision = prof["source"]["producer"]
    w(f"pub const PRODUCER: &str = {_rust_str(producer)};")
    w("")
    w("fn guarantee(reference: &str) -> Result<TargetFactSource, TargetProfileBuildError> {")
    w(f"    let producer = TargetFactProducerIdentity::new(PRODUCER.to_owned(), {revision})")
    w("        .map_err(|_| TargetProfileBuildError::InvalidProducerClaim)?;")
    w("    let reference = TargetNormativeReferenceIdentity::new(reference.to_owned(), 1)")
    w("        .map_err(|_| TargetProfileBuildError::InvalidProducerClaim)?;")
    w("    Ok(TargetFactSource::external_guarantee(producer, reference))")
    w("}")
    w("")
    w("/// The sm_100a profile.  `cost_source` carries the measurement context of")
    w("/// the fold-step sweep (nvcc build, the B200 execution environment).")
    w("pub fn cuda_sm100a_profile(")
    w("    cost_source: Option<TargetCompileProfileMeasurementSource>,")
    w(") -> Result<TargetProfile, TargetProfileBuildError> {")
    w("    let key = TargetProfileKey::new(PROFILE_KEY.to_owned())")
    w("        .map_err(|_| TargetProfileBuildError::InvalidProducerClaim)?;")
    w("    let mut builder = TargetProfileBuilder::new(key);")
    ieee, ptx = prof["source"]["references"]
    w(f"    let ieee = guarantee({_rust_str(ieee)})?;")
    w(f"    let ptx = guarantee({_rust_str(ptx)})?;")
    w("")
    w("    // capability rows (tiler_cuda_device_facts_query)")
    for name, value in prof["capability"]:
        if name == "index_arithmetic":
            arg = f"IndexArithmeticSupport::{value}"
        elif name == "device_address_width":
            arg = f"DeviceAddressWidth::{value}"
        elif name == "device_memory":
            arg = "true" if value else "false"
        else:
            arg = str(int(value))
        w(f"    builder.declare_{name}({arg}, ptx.clone())?;")
    w("")
    w("    // numerics rows: what every kernel does (IEEE binary32, one rounding per operator)")
    w("    let f32_subject = ScalarArithmetic::f32();")
    for subject, axis, behaviour, support in prof["numerics"]:
        if axis in ("input_subnormals", "result_subnormals"):
            arg = _SUBNORMAL_RUST[behaviour]
        elif axis in _PERMISSION_AXES:
            arg = "NumericalPermission::Permitted" if behaviour.startswith("Permitted") else \
                "NumericalPermission::Forbidden"
        elif axis == "approximate_intrinsics":
            arg = f"ApproximationEnvelope::{behaviour}"
        else:
            arg = f"ExceptionalValueAssumption::{behaviour}"
        if behaviour == "Permitted(declared grouping)":
            w("    // permitted only as the grouping a provider proposal declares (the grid grouping)")
        w(f"    builder.declare_{axis}(f32_subject.clone(), {arg}, ScalarSupport::{support}, ieee.clone())?;")
    w("")
    w("    // dtype dispatchability")
    for dtype, verdict in prof["dtype_dispatchability"]:
        w(f"    builder.declare_dtype_dispatchability({_RUST_DTYPES[dtype]}, DTypeDispatchability::{verdict}, "
          "ptx.clone())?;")
    w("")
    w("    // the subgroup realization of the grouped fold's butterfly")
    for subj, verdict in prof["subgroup_realization"]:
        w("    let subject = SubgroupRealizationSubject::new(")
        w(f"        SubgroupWidth::new({subj['width']}).map_err(|_| TargetProfileBuildError::InvalidProducerClaim)?,")
        w(f"        ArithmeticType::{subj['element']},")
        w("        SubgroupTransfer::InRangeXorShuffle,")
        w("    )")
        w("    .map_err(|_| TargetProfileBuildError::InvalidProducerClaim)?;")
        support = "Realized" if verdict == "Supported" else "Unrealizable"
        w(f"    builder.declare_subgroup_realization(subject, SubgroupSupport::{support}, ptx.clone())?;")
    w("")
    w("    // the measured cost row (a dispatch sweep on one B200; silence states no preference)")
    rows = prof["cost"]
    if rows:
        _, steps, _ = rows[0]
        w("    if let Some(source) = cost_source {")
        w(f"        builder.declare_measured_saturated_parallel_fold_steps({int(steps)}, source)?;")
        w("    }")
    else:
        w("    let _ = cost_source;")
    w("    builder.build()")
    w("}")
    w("")
    w("/// PayloadMetadata for the sm_100a cubin (`code` = tiler_kernels.cubin).")
    w("pub fn cuda_payload_metadata(source_representation: RepresentationKey) -> PayloadMetadata {")
    w("    PayloadMetadata {")
    w("        source_representation,")
    w("        source: Vec::new(),")
    w("        provenance: PayloadProvenance {")
    for field in ("toolchain", "target", "family", "language"):
        w(f"            {field}: {_rust_str(prov[field])}.to_owned(),")
    w("            platform: PayloadPlatform::Unversioned,")
    w("            components: vec![")
    for comp in prov["components"]:
        w(f"                ToolComponent {{ role: {_rust_str(comp['role'])}.to_owned(), "
          f"version: {_rust_str(comp['version'])}.to_owned() }},")
    w("            ],")
    w("            compile_flags: vec![" + ", ".join(f"{_rust_str(f)}.to_owned()" for f in prov["compile_flags"]) + "],")
    w("            link_flags: vec![" + ", ".join(f"{_rust_str(f)}.to_owned()" for f in prov["link_flags"]) + "],")
    w("        },")
    w("        entries: vec![")
    for e in ents:
        w(f"            PayloadEntryMapping {{ entry_key: BackendEntryKey::new({_rust_str(e['entry_key'])}.to_owned())"
          f".expect(\"entry key\"), symbol: {_rust_str(e['symbol'])}.to_owned(), transports: Vec::new() }},")
    w("        ],")
    w("        obligations: vec![PayloadTargetObligation { key: \"subgroup-width\".to_owned(), value: \"32\".to_owned() }],")
    w("    }")
    w("}")
    return "\n".join(L) + "\n"


# Entries whose kernels tiler_kernels.cubin carries (tiler_cuda_module_entry
# accepts exactly these; csrc/launch.cuh lists the kernels).
MODULE_ENTRY_SYMBOLS = ("tiler_cuda.sum_f32.grouped", "tiler_cuda.max_f32.grouped", "tiler_cuda.rms_norm_f32",
                        "tiler_cuda.rms_norm_bf16", "tiler_cuda.rms_norm_quantize_i8")
RUST_PATH = os.path.join(os.path.dirname(os.path.abspath(__file__)), "rust", "tiler_cuda_profile.rs")
# the fold-step row as measured on one B200 (python -m tiler_b200.target_profile)
MEASURED_FOLD_STEPS = 10571


if __name__ == "__main__":
    _main()
