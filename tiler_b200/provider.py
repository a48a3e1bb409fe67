"""The physical-provider seam for tiler-cuda.

Mirrors moderately-ai/tiler's ``PhysicalImplementationProvider``
(crates/tiler-compiler/src/frontier.rs:1507-1527): a provider states its
provenance and, for a reduction subject, proposes realizations, each naming
the grouping it computes, with a structural cost estimate
(``PhysicalCostEstimate::structural(dispatches, threads, temp_bytes)``,
frontier.rs:386-397), or declines a strategy with a ``StrategyDeclineCause``
(frontier.rs:1311-1384).  The host re-verifies a proposal before using it
(physical_provider.rs:27-46): :func:`verify` restates the coverage rules the
kernels and the oracle enforce.

Everything here is host logic: proposals are planned for a stated SM count
through the device-free C-ABI entry ``tiler_cuda_plan_grouping_for``.
"""
from __future__ import annotations

import ctypes as C
import math
from dataclasses import dataclass, field

from . import _native as N

PROVIDER_NAME = "tiler-cuda.reductions"
PROVIDER_VERSION = 1
TARGET = "sm_100a"
SUBGROUP_WIDTH = 32  # an equality, never a floor (docs/decisions/0094 decision 7)


@dataclass(frozen=True)
class ReductionSubject:
    """One reduction occurrence: ``rows`` independent outputs, each folding
    ``count`` contiguous contributors (the last axis).  ``family`` is
    ``"sum"`` (tiler::strict-serial-sum-f32) or ``"maximum"``;
    ``reassociation`` is the request's numerical permission
    (NumericalContract, session.rs:1793-1888)."""
    family: str
    rows: int
    count: int
    reassociation: bool = True


@dataclass(frozen=True)
class CostEstimate:
    dispatches: int
    threads: int
    temp_bytes: int


@dataclass(frozen=True)
class Proposal:
    strategy: str
    entry_symbol: str
    grouping: dict = field(default_factory=dict)
    cost: CostEstimate = CostEstimate(1, 1, 0)


@dataclass(frozen=True)
class Decline:
    strategy: str
    cause: str        # NumericalPermissionRefused | NoAdmissibleShape | Unrepresentable
    rule: str
    extent: int = 0


def governed_partition(contributors: int):
    """The compiler's governed split: the largest divisor <= isqrt(C) that
    leaves at least two partitions (crates/tiler-compiler/src/physical.rs:
    2780-2799).  Returns (partitions, contributors_per_partition) or None."""
    if contributors < 4:
        return None
    candidate = math.isqrt(contributors)
    while candidate >= 2:
        if contributors % candidate == 0:
            partitions = contributors // candidate
            if partitions >= 2:
                return partitions, candidate
        candidate -= 1
    return None


def plan_grid_grouping(rows: int, count: int, sm_count: int = 148) -> dict | None:
    """The grid + ADR-0100 composition grouping the backend declares."""
    g = N.Grouping()
    st = N.lib().tiler_cuda_plan_grouping_for(sm_count, rows, count, C.byref(g))
    return g.as_dict() if st == N.OK else None


def verify(subject: ReductionSubject, proposal: Proposal) -> bool:
    """Host re-verification of a proposed grouping (coverage exactly once;
    ADR-0100 canonicality T*k*(R-1) < n <= T*k*R; warp-multiple widths)."""
    g = proposal.grouping
    if proposal.strategy == "serial":
        return True
    if proposal.strategy == "governed-split":
        return g["partitions"] * g["per_partition"] == subject.count and g["partitions"] >= 1
    if proposal.strategy == "grid-composition":
        P, T, k, R = g["partitions"], g["threads"], g["k"], g["rounds"]
        if P < 1 or subject.count % P or T % 32 or not 0 < T <= 1024 or k < 1 or R < 1:
            return False
        per = subject.count // P
        if not (T * k * (R - 1) < per <= T * k * R):
            return False
        ct = g["combine_threads"]
        if ct:
            ck, cr = g["combine_k"], g["combine_rounds"]
            if ct % 32 or ct > T or not (ct * ck * (cr - 1) < P <= ct * ck * cr):
                return False
        return True
    return False


class CudaPhysicalProvider:
    """PhysicalImplementationProvider for the reduction families."""

    def __init__(self, sm_count: int = 148):
        self.sm_count = sm_count

    def provenance(self) -> dict:
        return {"name": PROVIDER_NAME, "version": PROVIDER_VERSION, "target": TARGET,
                "subgroup_width": SUBGROUP_WIDTH, "abi_version": int(N.lib().tiler_cuda_abi_version())}

    def propose(self, subject: ReductionSubject):
        """Returns (proposals, declines).  The serial fold is always
        admissible; reassociating groupings need the reassociation permission
        (a declared grouping consumes reassociation alone, ADR-0100 decision
        1); the maximum has no identity, so an empty domain is refused."""
        proposals, declines = [], []
        fam = subject.family
        if fam not in ("sum", "maximum"):
            return [], [Decline("*", "NoAdmissibleShape", "tiler-cuda.family-not-realized")]
        if fam == "maximum" and subject.count == 0:
            return [], [Decline("*", "NoAdmissibleShape", "maximum.empty-domain-has-no-identity", 0)]
        serial_symbol = "tiler_cuda.sum_f32.strict" if fam == "sum" else "tiler_cuda.max_f32.grouped"
        if fam == "sum":
            proposals.append(Proposal("serial", serial_symbol, {},
                                      CostEstimate(1, max(1, subject.rows), 0)))
        if not subject.reassociation:
            declines.append(Decline("grid-composition", "NumericalPermissionRefused", "reassociation"))
            declines.append(Decline("governed-split", "NumericalPermissionRefused", "reassociation"))
            if fam == "maximum":
                # the maximum is associative and commutative: any grouping is
                # bit-exact (softmax/tests.rs:118), so it needs no permission
                g = plan_grid_grouping(subject.rows, subject.count, self.sm_count)
                if g:
                    proposals.append(self._grid(subject, g, "tiler_cuda.max_f32.grouped"))
            return proposals, declines
        g = plan_grid_grouping(subject.rows, subject.count, self.sm_count) if subject.count else None
        if g:
            sym = "tiler_cuda.sum_f32.grouped" if fam == "sum" else "tiler_cuda.max_f32.grouped"
            proposals.append(self._grid(subject, g, sym))
        else:
            declines.append(Decline("grid-composition", "NoAdmissibleShape", "grid.no-divisor-partition",
                                    subject.count))
        if fam == "sum":
            split = governed_partition(subject.count)
            if split:
                P, per = split
                proposals.append(Proposal("governed-split", "tiler_cuda.sum_f32.partitioned",
                                          {"partitions": P, "per_partition": per},
                                          CostEstimate(2, subject.rows * P, subject.rows * P * 4)))
            else:
                declines.append(Decline("governed-split", "NoAdmissibleShape", "split.no-divisor",
                                        subject.count))
        return proposals, declines

    def _grid(self, subject, g, symbol):
        ws = int(N.lib().tiler_cuda_grouped_workspace_bytes(subject.rows, C.byref(N.Grouping.from_dict(g))))
        return Proposal("grid-composition", symbol, g,
                        CostEstimate(1, subject.rows * g["partitions"] * g["threads"], ws))
