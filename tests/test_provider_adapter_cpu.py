"""Host logic of the provider and runtime-adapter seams (no GPU)."""
import ctypes as C

import numpy as np
import pytest

from tiler_b200 import _native as N
from tiler_b200 import adapter as A
from tiler_b200 import provider as P


def test_governed_partition_restates_the_compiler_split():
    # physical.rs:2780-2799: largest divisor <= isqrt(C) with >= 2 partitions
    assert P.governed_partition(1 << 24) == (4096, 4096)
    assert P.governed_partition(12) == (4, 3)
    assert P.governed_partition(3) is None
    assert P.governed_partition(101) is None  # prime: no split
    assert P.governed_partition(4) == (2, 2)


def test_grid_plan_is_canonical_and_verified():
    prov = P.CudaPhysicalProvider(sm_count=148)
    for rows, count in [(1, 1 << 24), (3, 100_003), (8192, 4096), (1, 1), (7, 12288)]:
        props, declines = prov.propose(P.ReductionSubject("sum", rows, count))
        strategies = {p.strategy for p in props}
        assert "serial" in strategies and "grid-composition" in strategies
        for p in props:
            assert P.verify(P.ReductionSubject("sum", rows, count), p), p


def test_grid_plan_matches_the_oracle_identities(oracle_lib):
    """A one-partition, one-warp, k=1, one-round grid grouping over 32
    contributors is the ascending butterfly alone; a planned grouping folds
    every contributor exactly once (the sum of ones is exact)."""
    x = np.ones((2, 100_003), np.float32)
    g = P.plan_grid_grouping(2, 100_003)
    st, y = oracle_lib.grid_fold(x, g)
    assert st == 0 and (y == 100_003).all()


def test_reassociation_refused_keeps_only_the_serial_fold():
    prov = P.CudaPhysicalProvider()
    props, declines = prov.propose(P.ReductionSubject("sum", 1, 1 << 20, reassociation=False))
    assert [p.strategy for p in props] == ["serial"]
    assert {d.cause for d in declines} == {"NumericalPermissionRefused"}
    # the maximum needs no permission: any grouping is bit-exact
    props, _ = prov.propose(P.ReductionSubject("maximum", 1, 1 << 20, reassociation=False))
    assert [p.strategy for p in props] == ["grid-composition"]


def test_empty_maximum_is_declined():
    props, declines = P.CudaPhysicalProvider().propose(P.ReductionSubject("maximum", 4, 0))
    assert not props and declines[0].rule == "maximum.empty-domain-has-no-identity"


def test_provenance():
    pv = P.CudaPhysicalProvider().provenance()
    assert pv["target"] == "sm_100a" and pv["subgroup_width"] == 32 and pv["abi_version"] == 1


class FakeNative:
    """A device stand-in for the adapter's pre-commit phases."""

    def __init__(self, cc=(10, 0), warp=32):
        self.cc, self.warp = cc, warp
        self.real = N.lib()

    def tiler_cuda_context_create(self, device, out):
        C.cast(out, C.POINTER(C.c_void_p))[0] = 0x1234
        return N.OK

    def tiler_cuda_context_destroy(self, ctx):
        return N.OK

    def tiler_cuda_device_facts_query(self, ctx, out):
        f = C.cast(out, C.POINTER(N.DeviceFacts))[0]
        f.cc_major, f.cc_minor, f.warp_size, f.sm_count, f.max_threads_per_block = *self.cc, self.warp, 148, 1024
        f.name = b"fake"
        return N.OK

    def tiler_cuda_payload_validate(self, ctx, target, width, syms, n, refused):
        if target != b"sm_100a" or width != 32 or self.cc != (10, 0) or self.warp != 32:
            return N.PAYLOAD_REFUSED
        known = {self.real.tiler_cuda_entry_symbol(i) for i in range(self.real.tiler_cuda_entry_count())}
        for i in range(n):
            if syms[i] not in known:
                C.cast(refused, C.POINTER(C.c_uint32))[0] = i
                return N.PAYLOAD_REFUSED
        return N.OK

    def tiler_cuda_entry_query(self, ctx, sym, out):
        p = C.cast(out, C.POINTER(N.EntryProps))[0]
        p.max_threads_per_block, p.threads_per_block = 1024, 256
        return N.OK


def payload(symbols, target="sm_100a", width=32):
    return A.Payload(target, width, tuple(A.Entry(f"e{i}", s) for i, s in enumerate(symbols)))


def test_route_runs_the_phases_in_the_reference_order():
    calls = []
    ad = A.CudaRuntimeAdapter(native=FakeNative(), executor=lambda sym: (lambda args: calls.append(sym) or sym))
    out = A.route_with_adapter(payload(["tiler_cuda.rms_norm_f32", "tiler_cuda.sum_f32.grouped"]),
                               [A.Launch("e0", {}), A.Launch("e1", {})], ad)
    assert out == ["tiler_cuda.rms_norm_f32", "tiler_cuda.sum_f32.grouped"]
    assert ad.trace == ["bind_execution_context", "observe_target_environment", "validate_payload",
                        "observe_live_device", "observe_target_environment", "prepare_entries",
                        "observe_prepared_entry", "observe_prepared_entry", "plan_dispatch", "commit",
                        "allocate_dispatch", "dispatch"]


@pytest.mark.parametrize("kw", [dict(target="sm_90a"), dict(width=64)])
def test_wrong_target_or_subgroup_width_is_refused_before_commit(kw):
    ad = A.CudaRuntimeAdapter(native=FakeNative())
    with pytest.raises(A.Refusal) as e:
        A.route_with_adapter(payload(["tiler_cuda.rms_norm_f32"], **kw), [], ad)
    assert e.value.phase == "validate_payload" and not ad.committed


def test_unknown_entry_symbol_is_refused_with_its_name():
    ad = A.CudaRuntimeAdapter(native=FakeNative())
    with pytest.raises(A.Refusal) as e:
        A.route_with_adapter(payload(["tiler_cuda.rms_norm_f32", "tiler_cuda.no_such_entry"]), [], ad)
    assert e.value.detail == "tiler_cuda.no_such_entry"


def test_a_device_of_another_architecture_is_refused():
    ad = A.CudaRuntimeAdapter(native=FakeNative(cc=(9, 0)))
    with pytest.raises(A.Refusal):
        A.route_with_adapter(payload(["tiler_cuda.rms_norm_f32"]), [], ad)


def test_failure_after_commit_has_no_fallback():
    def boom(sym):
        def run(args):
            raise RuntimeError("device fault")
        return run
    ad = A.CudaRuntimeAdapter(native=FakeNative(), executor=boom)
    with pytest.raises(A.Failure) as e:
        A.route_with_adapter(payload(["tiler_cuda.rms_norm_f32"]), [A.Launch("e0", {})], ad)
    assert ad.committed and e.value.phase == "dispatch"


def test_no_device_refuses_at_bind():
    try:
        import torch
        if torch.cuda.is_available():
            pytest.skip("a device is present")
    except ImportError:
        pass
    ad = A.CudaRuntimeAdapter()
    with pytest.raises(A.Refusal) as e:
        A.route_with_adapter(payload(["tiler_cuda.rms_norm_f32"]), [], ad)
    assert e.value.phase == "bind_execution_context"
