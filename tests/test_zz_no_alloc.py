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
