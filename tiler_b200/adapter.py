"""The runtime device seam for tiler-cuda.

Mirrors moderately-ai/tiler's ``RuntimeAdapter`` (crates/tiler-runtime/src/
adapter.rs:260-511) and the order ``route_with_adapter`` drives it in
(adapter.rs:545-678):

  bind_execution_context -> observe_target_environment -> validate_payload
  (per entry) -> observe_live_device -> prepare_entries ->
  observe_prepared_entry -> plan_dispatch -> COMMIT -> allocate_dispatch ->
  dispatch

Everything before the commit may *refuse* (a typed :class:`Refusal`, the
program may be routed elsewhere); after the one-way commit there is no
fallback and any error is a :class:`Failure` (adapter.rs:664-677, :693-800).
The adapter owns every device object it creates.  Device work goes through
the C-ABI (libtiler_cuda.so) only.
"""
from __future__ import annotations

import ctypes as C
from dataclasses import dataclass, field

from . import _native as N


class Refusal(Exception):
    """A pre-commit refusal: the route may be retried on another adapter."""

    def __init__(self, phase: str, code: int, detail: str = ""):
        self.phase, self.code, self.detail = phase, code, detail
        super().__init__(f"{phase} refused: {N.status_string(code) if code else ''} {detail}".strip())


class Failure(Exception):
    """A post-commit failure: there is no fallback."""

    def __init__(self, phase: str, code: int, detail: str = ""):
        self.phase, self.code, self.detail = phase, code, detail
        super().__init__(f"{phase} failed: {N.status_string(code) if code else ''} {detail}".strip())


@dataclass(frozen=True)
class Binding:
    """One buffer binding (RoutedBinding, crates/tiler-runtime/src/load/
    route.rs:145-191): name, role (input/output) and byte length."""
    name: str
    role: str
    nbytes: int


@dataclass(frozen=True)
class Entry:
    """One payload entry: its key, the library symbol realizing it, its
    bindings and whether zero work skips the dispatch (route.rs:69-97)."""
    entry_key: str
    symbol: str
    bindings: tuple = ()
    zero_work_skips_dispatch: bool = True


@dataclass(frozen=True)
class Payload:
    """The backend payload a plan artifact carries (PayloadMetadata,
    crates/tiler-artifact/src/program/codec/payload.rs:228-424)."""
    target: str
    subgroup_width: int
    entries: tuple
    provenance: dict = field(default_factory=dict)
    # PayloadContent.code: the compiled code bytes (an sm_100a cubin of this
    # library's kernels, tiler_b200/tiler_kernels.cubin), or None to run the
    # library's built-in copies
    code: bytes | None = None


@dataclass
class Launch:
    """A dispatch request: the entry and its runtime arguments."""
    entry_key: str
    args: dict


@dataclass
class PreparedEntry:
    entry: Entry
    props: dict


@dataclass
class DispatchPlan:
    launches: list
    workspace_bytes: int = 0


class CudaRuntimeAdapter:
    """RuntimeAdapter over libtiler_cuda.  ``executor`` maps an entry symbol
    to a callable(args, workspace) that launches it (default: the torch-facing
    families); tests may inject a host executor and a fake native library."""

    def __init__(self, device: int = 0, native=None, executor=None):
        self.device = device
        self.native = native or N.lib()
        self.executor = executor
        self.ctx = None
        self.facts = None
        self.trace: list = []
        self.committed = False
        self.module = None  # the loaded payload code (tiler_cuda_module*)

    # ---- pre-commit phases (may refuse) ------------------------------------
    def bind_execution_context(self):
        self.trace.append("bind_execution_context")
        handle = C.c_void_p()
        st = self.native.tiler_cuda_context_create(self.device, C.byref(handle))
        if st != N.OK:
            raise Refusal("bind_execution_context", st, f"device {self.device}")
        self.ctx = handle.value

    def observe_target_environment(self) -> dict:
        self.trace.append("observe_target_environment")
        f = N.DeviceFacts()
        st = self.native.tiler_cuda_device_facts_query(self.ctx, C.byref(f))
        if st != N.OK:
            raise Refusal("observe_target_environment", st)
        self.facts = {k: (getattr(f, k).decode() if k == "name" else int(getattr(f, k))) for k, _ in f._fields_}
        return self.facts

    def validate_payload(self, payload: Payload):
        self.trace.append("validate_payload")
        syms = [e.symbol.encode() for e in payload.entries]
        arr = (C.c_char_p * max(1, len(syms)))(*syms)
        refused = C.c_uint32(0)
        st = self.native.tiler_cuda_payload_validate(self.ctx, payload.target.encode(), payload.subgroup_width, arr,
                                                     len(syms), C.byref(refused))
        if st != N.OK:
            which = payload.entries[refused.value].symbol if refused.value < len(payload.entries) else ""
            raise Refusal("validate_payload", st, which)
        if payload.code is not None:
            handle = C.c_void_p()
            st = self.native.tiler_cuda_module_load(self.ctx, payload.code, len(payload.code), C.byref(handle))
            if st != N.OK:
                raise Refusal("validate_payload", st, "payload code")
            self.module = handle.value

    def observe_live_device(self) -> dict:
        self.trace.append("observe_live_device")
        return self.observe_target_environment()

    def prepare_entries(self, payload: Payload) -> dict:
        self.trace.append("prepare_entries")
        prepared = {}
        for e in payload.entries:
            props = N.EntryProps()
            if self.module is not None:  # the entry as the payload's own code carries it
                st = self.native.tiler_cuda_module_entry(self.module, e.symbol.encode(), C.byref(props))
            else:
                st = self.native.tiler_cuda_entry_query(self.ctx, e.symbol.encode(), C.byref(props))
            if st != N.OK:
                raise Refusal("prepare_entries", st, e.symbol)
            prepared[e.entry_key] = PreparedEntry(e, {k: int(getattr(props, k)) for k, _ in props._fields_})
        return prepared

    def observe_prepared_entry(self, prepared: PreparedEntry) -> dict:
        self.trace.append("observe_prepared_entry")
        p = prepared.props
        if p["threads_per_block"] > p["max_threads_per_block"]:
            raise Refusal("observe_prepared_entry", N.UNSUPPORTED, prepared.entry.symbol)
        return p

    def plan_dispatch(self, prepared: dict, launches: list) -> DispatchPlan:
        self.trace.append("plan_dispatch")
        for ln in launches:
            if ln.entry_key not in prepared:
                raise Refusal("plan_dispatch", N.INVALID_APPLICATION, f"unknown entry {ln.entry_key}")
        return DispatchPlan(launches=list(launches))

    # ---- post-commit phases (fail, never fall back) ------------------------
    def allocate_dispatch(self, plan: DispatchPlan):
        self.trace.append("allocate_dispatch")
        return {}

    def dispatch(self, prepared: dict, plan: DispatchPlan, workspace) -> list:
        self.trace.append("dispatch")
        results = []
        # the payload's code is bound to the context the executor launches on
        # for the duration of the dispatch
        exec_ctx = None
        if self.module is not None and self.executor is None:
            from . import families as F
            exec_ctx = F.context(self.device)
            st = self.native.tiler_cuda_context_bind_module(exec_ctx, self.module)
            if st != N.OK:
                raise Failure("dispatch", st, "binding the payload code")
        try:
            for ln in plan.launches:
                entry = prepared[ln.entry_key].entry
                run = (self.executor or _default_executor)(entry.symbol)
                try:
                    results.append(run(ln.args))
                except Exception as exc:  # no fallback after the commit
                    code = getattr(exc, "code", N.DEVICE_ERROR)
                    raise Failure("dispatch", code, f"{entry.symbol}: {exc}") from exc
        finally:
            if exec_ctx is not None:
                self.native.tiler_cuda_context_bind_module(exec_ctx, None)
        return results

    def module_launches(self) -> int:
        """Launches that ran from the payload's own code so far."""
        if self.module is None:
            return 0
        n = C.c_uint64()
        self.native.tiler_cuda_module_launch_count(self.module, C.byref(n))
        return int(n.value)

    def close(self):
        if self.module is not None and self.native is not None:
            import torch
            if torch.cuda.is_available():
                torch.cuda.synchronize(self.device)  # its launches have finished
            self.native.tiler_cuda_module_unload(self.module)
            self.module = None
        if self.ctx is not None and self.native is not None:
            self.native.tiler_cuda_context_destroy(self.ctx)
            self.ctx = None


def route_with_adapter(payload: Payload, launches: list, adapter: CudaRuntimeAdapter):
    """Drives the adapter through the routing phases in the reference's order
    and commits once (crates/tiler-runtime/src/adapter.rs:545-678)."""
    adapter.bind_execution_context()
    adapter.observe_target_environment()
    adapter.validate_payload(payload)
    adapter.observe_live_device()
    prepared = adapter.prepare_entries(payload)
    for p in prepared.values():
        adapter.observe_prepared_entry(p)
    plan = adapter.plan_dispatch(prepared, launches)
    adapter.trace.append("commit")
    adapter.committed = True
    workspace = adapter.allocate_dispatch(plan)
    return adapter.dispatch(prepared, plan, workspace)


def _default_executor(symbol: str):
    from . import families as F
    table = {
        "tiler_cuda.rms_norm_f32": lambda a: F.rms_norm(a["x"], a["w"], a.get("eps_bits", F.EPS_1E6_BITS)),
        "tiler_cuda.rms_norm_bf16": lambda a: F.rms_norm(a["x"], a["w"], a.get("eps_bits", F.EPS_1E6_BITS)),
        "tiler_cuda.softmax_f32": lambda a: F.softmax(a["x"], a.get("causal_period", 0), a.get("row_offset", 0)),
        "tiler_cuda.softmax_masked_f32": lambda a: F.softmax_masked(a["x"], a["mask"], a.get("row_offset", 0)),
        "tiler_cuda.sum_f32.grouped": lambda a: F.sum_f32(a["x"], a.get("grouping")),
        "tiler_cuda.max_f32.grouped": lambda a: F.max_f32(a["x"], a.get("grouping")),
        "tiler_cuda.sum_f32.strict": lambda a: F.strict_sum_f32(a["x"]),
        "tiler_cuda.sum_f32.partitioned": lambda a: F.partitioned_sum_f32(a["x"], a["partitions"],
                                                                           a["per_partition"]),
        "tiler_cuda.sum_f32.cooperative": lambda a: F.cooperative_sum_f32(a["x"], a["participants"],
                                                                           a["per_partition"], a["rounds"],
                                                                           a.get("participant_major", False)),
        "tiler_cuda.quantize_i8_rows": lambda a: F.quantize_i8_rows(a["x"]),
        "tiler_cuda.rms_norm_quantize_i8": lambda a: F.rms_norm_quantize_i8(a["x"], a["w"],
                                                                             a.get("eps_bits", F.EPS_1E6_BITS)),
        "tiler_cuda.dequantize_i8_rows": lambda a: F.dequantize_i8_rows(a["codes"], a["scales"]),
        "tiler_cuda.quantize_affine_u8": lambda a: F.quantize_affine_u8(a["x"], a["scale"], a["zero_point"],
                                                                         a.get("maximum", 255)),
        "tiler_cuda.dequantize_affine_u8": lambda a: F.dequantize_affine_u8(a["codes"], a["scale"],
                                                                             a["zero_point"], a.get("maximum", 255)),
        "tiler_cuda.silu_f32": lambda a: F.silu(a["x"]),
        "tiler_cuda.scale_bias_f32": lambda a: F.scale_bias(a["x"], a["a"], a["b"]),
        "tiler_cuda.gather_rows": lambda a: F.gather_rows(a["table"], a["ids"]),
        "tiler_cuda.contract_f32": lambda a: F.contract_f32(a["a"], a["b"]),
        "tiler_cuda.gemm_bf16": lambda a: F.gemm_bf16(a["a"], a["b"], a.get("epilogue", "silu")),
    }
    if symbol not in table:
        raise Failure("dispatch", N.UNSUPPORTED, symbol)
    return table[symbol]
