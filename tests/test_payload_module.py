"""The payload-code boundary: a plan artifact's code bytes (an sm_100a cubin
built from this library's kernel sources) are loaded through the C-ABI
(validate_payload / prepare_entries, crates/tiler-runtime/src/adapter.rs:
639-657), bound to a context, and are then what launches: the module's launch
counter moves and the results match the oracle bit for bit.  Images the
device cannot run, or that do not carry this C-ABI's version, are refused
before any dispatch."""
import ctypes as C
import subprocess

import numpy as np
import pytest

from golden_util import seeded_normal, seeded_uniform

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def env():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from tiler_b200 import _native as N
    from tiler_b200 import families as fam
    return N, fam, fam.context()


def _load(N, ctx, code):
    m = C.c_void_p()
    st = N.lib().tiler_cuda_module_load(ctx, code, len(code), C.byref(m))
    return st, m.value


def _count(N, m):
    n = C.c_uint64()
    assert N.lib().tiler_cuda_module_launch_count(m, C.byref(n)) == N.OK
    return n.value


def test_module_launches_rms_and_grouped_sum_bit_exact(env, oracle_lib):
    N, fam, ctx = env
    L = N.lib()
    code = open(N.CUBIN_PATH, "rb").read()
    st, m = _load(N, ctx, code)
    assert st == N.OK and m
    try:
        props = N.EntryProps()
        assert L.tiler_cuda_module_entry(m, b"tiler_cuda.rms_norm_f32", C.byref(props)) == N.OK
        assert props.threads_per_block <= props.max_threads_per_block and props.num_regs > 0
        # an entry whose kernel the module does not carry is refused
        assert L.tiler_cuda_module_entry(m, b"tiler_cuda.softmax_f32", C.byref(props)) == N.PAYLOAD_REFUSED
        assert L.tiler_cuda_context_bind_module(ctx, m) == N.OK
        before = _count(N, m)
        x = seeded_normal(31, 300 * 4096).reshape(300, 4096)
        w = seeded_uniform(32, 4096, 0.5, 1.5)
        got = fam.rms_norm(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda()).cpu().numpy()
        _, want = oracle_lib.rms_norm_f32(x, w, nthreads=8)
        assert (got.view(np.uint32) == want.view(np.uint32)).all()
        xb = oracle_lib.f32_to_bf16(x)
        wb = oracle_lib.f32_to_bf16(w)
        gotb = fam.rms_norm(torch.from_numpy(xb.view(np.int16)).cuda().view(torch.bfloat16),
                            torch.from_numpy(wb.view(np.int16)).cuda().view(torch.bfloat16))
        _, wantb = oracle_lib.rms_norm_bf16(xb, wb, nthreads=8)
        assert (gotb.view(torch.int16).cpu().numpy().view(np.uint16) == wantb).all()
        s = seeded_uniform(33, 1 << 22, -1.0, 1.0)
        g = fam.plan_grouping(1, s.size)
        total = fam.sum_f32(torch.from_numpy(s).cuda(), g).cpu().numpy()
        _, wants = oracle_lib.grid_fold(s, g)
        assert total.reshape(-1).view(np.uint32)[0] == np.asarray(wants).view(np.uint32).ravel()[0]
        torch.cuda.synchronize()
        assert _count(N, m) - before == 3  # all three ran from the module
        # unbound: the library's own kernels run again
        assert L.tiler_cuda_context_bind_module(ctx, None) == N.OK
        fam.rms_norm(torch.from_numpy(x).cuda(), torch.from_numpy(w).cuda())
        torch.cuda.synchronize()
        assert _count(N, m) - before == 3
    finally:
        L.tiler_cuda_context_bind_module(ctx, None)
        torch.cuda.synchronize()
        assert L.tiler_cuda_module_unload(m) == N.OK


def test_images_that_are_not_this_librarys_sm_100a_code_are_refused(env, tmp_path):
    N, fam, ctx = env
    # not an image at all: refused before the driver sees it
    assert _load(N, ctx, b"\0" * 4096)[0] == N.PAYLOAD_REFUSED
    assert _load(N, ctx, b"// .version 8.7\n.target sm_100a\n" + b" " * 100)[0] == N.PAYLOAD_REFUSED
    src = tmp_path / "k.cu"
    src.write_text('extern "C" __global__ void k(float* p) { p[threadIdx.x] = 1.0f; }\n')
    for arch, why in (("sm_90a", "another architecture"), ("sm_100a", "no C-ABI version")):
        out = tmp_path / f"k_{arch}.cubin"
        r = subprocess.run(["nvcc", "-cubin", f"-arch={arch}", "-o", str(out), str(src)], capture_output=True)
        if r.returncode != 0:
            pytest.skip("nvcc unavailable: " + r.stderr.decode()[:200])
        st, m = _load(N, ctx, out.read_bytes())
        assert st == N.PAYLOAD_REFUSED and not m, why


def test_adapter_routes_a_payload_that_carries_code(env, oracle_lib):
    N, fam, ctx = env
    from tiler_b200 import adapter as A
    code = open(N.CUBIN_PATH, "rb").read()
    x = seeded_normal(41, 64 * 4096).reshape(64, 4096)
    w = seeded_uniform(42, 4096, 0.5, 1.5)
    payload = A.Payload("sm_100a", 32, (A.Entry("rms", "tiler_cuda.rms_norm_f32"),), code=code)
    ad = A.CudaRuntimeAdapter()
    try:
        out = A.route_with_adapter(payload, [A.Launch("rms", {"x": torch.from_numpy(x).cuda(),
                                                               "w": torch.from_numpy(w).cuda()})], ad)
        torch.cuda.synchronize()
        assert ad.module_launches() == 1
    finally:
        ad.close()
    _, want = oracle_lib.rms_norm_f32(x, w)
    assert (out[0].cpu().numpy().view(np.uint32) == want.view(np.uint32)).all()
    # a payload whose code lacks an entry's kernel is refused before the commit
    bad = A.Payload("sm_100a", 32, (A.Entry("sm", "tiler_cuda.softmax_f32"),), code=code)
    ad = A.CudaRuntimeAdapter()
    try:
        with pytest.raises(A.Refusal) as e:
            A.route_with_adapter(bad, [A.Launch("sm", {"x": torch.zeros(4, 2048, device="cuda")})], ad)
        assert e.value.phase == "prepare_entries" and not ad.committed
    finally:
        ad.close()
