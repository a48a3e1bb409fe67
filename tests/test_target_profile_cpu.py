"""The target profile and payload provenance rows, checked against the
library and the build (no GPU)."""
import re

from tiler_b200 import _native as N
from tiler_b200 import provider, target_profile as tp


def test_profile_rows_match_what_the_backend_checks():
    prof = tp.target_profile()
    caps = dict(prof["capability"])
    assert caps["max_threads_per_workgroup"] == 1024
    assert caps["local_memory_bytes"] == 232448  # 227 KB opt-in shared memory per block
    assert caps["index_arithmetic"] == "CompleteU64" and caps["device_address_width"] == "Bits64"
    # the subgroup width the payload validation requires (an equality)
    (sub, support), = prof["subgroup_realization"]
    assert sub["width"] == provider.SUBGROUP_WIDTH == 32 and support == "Supported"
    numerics = {(axis, behaviour): support for _, axis, behaviour, support in prof["numerics"]}
    assert numerics[("input_subnormals", "Preserve")] == "Exact"
    assert numerics[("result_subnormals", "FlushToZero{PreservesSign}")] == "Unsupported"
    assert numerics[("contraction", "Forbidden")] == "Exact"
    assert numerics[("contraction", "Permitted")] == "Unsupported"
    assert numerics[("approximate_intrinsics", "Forbidden")] == "Exact"
    # device facts override the stated limits
    caps = dict(tp.capability_rows({"max_threads_per_block": 512, "smem_per_block_optin": 100}))
    assert caps["max_threads_per_workgroup"] == 512 and caps["local_memory_bytes"] == 100


def test_payload_provenance_states_the_build():
    prov = tp.payload_provenance()
    assert prov["target"] == "sm_100a" and prov["platform"] == "Unversioned"
    flags = prov["compile_flags"]
    # the numerics the profile declares rest on these flags
    assert "-fmad=false" in flags and not any("ftz" in f or "fast-math" in f for f in flags)
    assert "arch=compute_100a,code=sm_100a" in flags
    assert re.match(r"nvcc", prov["toolchain"])


def test_payload_entries_are_the_registry():
    L = N.lib()
    entries = tp.payload_entries()
    assert len(entries) == L.tiler_cuda_entry_count() > 10
    for e in entries:
        assert e["symbol"] == "tiler_cuda." + e["entry_key"]
    keys = {e["entry_key"] for e in entries}
    assert {"rms_norm_f32", "softmax_f32", "gemm_bf16", "sum_f32.grouped", "rms_norm_quantize_i8"} <= keys


def test_work_span_fit_recovers_a_known_model():
    """The cost-row fit on cells generated from a stated model (P = 4736
    steps at once, 3 us per stage, 2 ns per step) with 2 % noise."""
    import numpy as np
    rng = np.random.default_rng(4)
    P, enc, step = 4736.0, 3e-6, 2e-9
    cells = []
    for rows, count in [(128, 256), (1024, 256), (8192, 256), (65536, 64), (262144, 64), (32, 4096), (512, 2048),
                        (4096, 1024), (16384, 512), (16, 16384)]:
        for stages in ([(rows * count, count)], [(rows * count, count // 16), (rows * 16, 16)]):
            t = sum(enc + max(w / P, d) * step for w, d in stages) * (1 + 0.02 * rng.standard_normal())
            cells.append({"stages": stages, "seconds": t})
    fit = tp.fit_work_span(cells)
    assert abs(fit["parallel_steps"] / P - 1) < 0.1
    assert abs(fit["step_s"] / step - 1) < 0.1
    assert fit["residual"] < 0.05
    prof = tp.target_profile(measured_fold_steps=round(fit["parallel_steps"]))
    (key, value, scope), = prof["cost"]
    assert key == "cost.saturated-parallel-fold-steps" and scope == "MeasuredEnvironment" and value > 0
    assert tp.target_profile()["cost"] == []  # silence without a measurement


def test_committed_rust_declarations_are_the_rendering_of_these_rows():
    """tiler_b200/rust/tiler_cuda_profile.rs is what the crate compiles: it
    must be the current rendering, one builder call per row."""
    text = tp.render_rust(measured_fold_steps=tp.MEASURED_FOLD_STEPS)
    assert open(tp.RUST_PATH).read() == text, "regenerate with python -m tiler_b200.target_profile --rust"
    prof = tp.target_profile(measured_fold_steps=tp.MEASURED_FOLD_STEPS)
    calls = re.findall(r"builder\.(declare_\w+)\(", text)
    want = len(prof["capability"]) + len(prof["numerics"]) + len(prof["dtype_dispatchability"]) + \
        len(prof["subgroup_realization"]) + len(prof["cost"])
    assert len(calls) == want
    # every declaration is one of TargetProfileBuilder's own methods
    # (crates/tiler-compiler/src/target/builder.rs:97-1439)
    builder_methods = {
        "declare_max_threads_per_grid_axis", "declare_max_threads_per_workgroup",
        "declare_max_buffer_bindings_per_entry", "declare_index_arithmetic", "declare_device_address_width",
        "declare_device_memory", "declare_local_memory_bytes", "declare_input_subnormals",
        "declare_result_subnormals", "declare_contraction", "declare_reassociation", "declare_permutation",
        "declare_signed_zero", "declare_reciprocal_transform", "declare_approximate_intrinsics",
        "declare_nan_assumptions", "declare_infinity_assumptions", "declare_dtype_dispatchability",
        "declare_subgroup_realization", "declare_measured_saturated_parallel_fold_steps"}
    assert set(calls) <= builder_methods
    caps = dict(prof["capability"])
    assert f"declare_local_memory_bytes({caps['local_memory_bytes']}," in text
    assert f"declare_measured_saturated_parallel_fold_steps({tp.MEASURED_FOLD_STEPS}, source)" in text
    # braces and parentheses balance
    assert text.count("{") == text.count("}") and text.count("(") == text.count(")")
    # the payload metadata names exactly the entries the cubin carries, and the build flags
    syms = re.findall(r'symbol: "([^"]+)"', text)
    assert sorted(syms) == sorted(tp.MODULE_ENTRY_SYMBOLS)
    registry = {e["symbol"] for e in tp.payload_entries()}
    assert set(syms) <= registry
    assert '"-fmad=false".to_owned()' in text and '"sm_100a".to_owned()' in text
