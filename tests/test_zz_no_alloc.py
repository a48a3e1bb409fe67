"""The allocation-free grouped sum, tiler_cuda_sum_f32_no_alloc.

It exists for callers that cannot allocate device memory when they reduce
(their buffers are planned by someone else, or their loop must not call
cudaMalloc): its workspace is a fixed array inside the library.  This file
calls it through the C-ABI and holds it to the workspace-taking entry point,
bit for bit, on two calls in a row (the array keeps the previous call's
contents, so the second call checks that nothing stale leaks in).  It is
named so pytest collects it last.
"""
import ctypes as C

import numpy as np
import pytest

from golden_util import seeded_normal

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def lib_ctx():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from tiler_b200 import _native as N
    from tiler_b200 import families
    return N, families.context(), families


def _call_no_alloc(N, ctx, x, rows, count, g, out):
    stream = torch.cuda.current_stream().cuda_stream
    return N.lib().tiler_cuda_sum_f32_no_alloc(ctx, stream, x.data_ptr(), rows, count, C.byref(g), out.data_ptr())


@pytest.mark.parametrize("rows,count", [(1, 1 << 24), (3, 100_003), (8, 65536)])
def test_no_alloc_sum_matches_the_workspace_entry_point_twice(lib_ctx, rows, count):
    N, ctx, fam = lib_ctx
    for call in range(2):
        x = torch.from_numpy(seeded_normal(100 * call + rows, rows * count).reshape(rows, count) * 10).cuda()
        gd = fam.plan_grouping(rows, count)
        g = N.Grouping.from_dict(gd)
        want = fam.sum_f32(x, gd)
        got = torch.full((rows,), float("nan"), device="cuda")
        assert _call_no_alloc(N, ctx, x, rows, count, g, got) == N.OK
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int32), want.view(torch.int32)), (call, got, want)


def test_no_alloc_sum_refuses_sizes_beyond_its_array(lib_ctx):
    N, ctx, fam = lib_ctx
    x = torch.zeros(2048, 64, device="cuda")
    g = N.Grouping(partitions=2, threads=32, k=1, rounds=1)
    out = torch.empty(2048, device="cuda")
    assert _call_no_alloc(N, ctx, x, 2048, 64, g, out) == N.SHAPE_TOO_LARGE
    g = N.Grouping(partitions=1 << 17, threads=32, k=1, rounds=1)
    x = torch.zeros(1 << 17, device="cuda")
    assert _call_no_alloc(N, ctx, x, 1, 1 << 17, g, out) == N.SHAPE_TOO_LARGE


def _explicit(partitions):
    # one round of 32 lanes x 4 contiguous per partition: 128 contributors each
    return {"partitions": partitions, "threads": 32, "k": 4, "rounds": 1}


@pytest.mark.parametrize("rows,partitions,accepted", [
    (1024, 64, True),     # rows at the limit, rows x partitions exactly 65536
    (1024, 65, False),    # one partition past the partial-sum limit
    (1025, 2, False),     # one row past the row limit
    (16, 1, True),        # a single partition: forwarded, no workspace needed
])
def test_no_alloc_sum_at_and_past_its_limits(lib_ctx, rows, partitions, accepted):
    N, ctx, fam = lib_ctx
    gd = _explicit(partitions)
    count = partitions * 128
    x = torch.from_numpy(seeded_normal(rows + partitions, rows * count).reshape(rows, count)).cuda()
    got = torch.full((rows,), float("nan"), device="cuda")
    status = _call_no_alloc(N, ctx, x, rows, count, N.Grouping.from_dict(gd), got)
    if not accepted:
        assert status == N.SHAPE_TOO_LARGE
        return
    assert status == N.OK
    want = fam.sum_f32(x, gd)
    torch.cuda.synchronize()
    assert torch.equal(got.view(torch.int32), want.view(torch.int32))


def test_no_alloc_sum_refused_call_leaves_the_next_one_exact(lib_ctx):
    """A refused call between two good calls must not disturb the array: the
    second good call still matches the workspace entry point bit for bit."""
    N, ctx, fam = lib_ctx
    rows, count = 64, 1 << 16
    gd = fam.plan_grouping(rows, count)
    g = N.Grouping.from_dict(gd)
    for call in range(2):
        x = torch.from_numpy(seeded_normal(7 + call, rows * count).reshape(rows, count) * 3).cuda()
        got = torch.full((rows,), float("nan"), device="cuda")
        assert _call_no_alloc(N, ctx, x, rows, count, g, got) == N.OK
        want = fam.sum_f32(x, gd)
        torch.cuda.synchronize()
        assert torch.equal(got.view(torch.int32), want.view(torch.int32)), call
        # refused: a lane count that is not a whole number of warps
        bad = N.Grouping.from_dict({**gd, "threads": 33})
        assert _call_no_alloc(N, ctx, x, rows, count, bad, got) == N.INVALID_APPLICATION
