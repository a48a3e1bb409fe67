"""Parity of the CUDA path (through the C-ABI) with the CPU oracle and with the
reference's own golden vectors.  Bit-exact for integer / index / grouped-fold
work and for every family whose reference arithmetic the kernel restates;
the bf16 contraction is held to the BASELINE tolerance (1e-2 relative)."""
import hashlib

import time

import numpy as np
import pytest

from golden_util import bits_of, f, fbits, fvals, h, load, prng_values, seeded_normal, seeded_uniform

torch = pytest.importorskip("torch")
pytestmark = pytest.mark.gpu

G = load()


@pytest.fixture(scope="module")
def fam():
    if not torch.cuda.is_available():
        pytest.skip("needs a CUDA device")
    from tiler_b200 import families
    families.context()
    return families


def cuda(a):
    return torch.from_numpy(np.ascontiguousarray(a)).cuda()


def host(t):
    torch.cuda.synchronize()
    return t.cpu().numpy()


def assert_bits_equal(got, want, what=""):
    g = np.ascontiguousarray(got).view(np.uint32).ravel()
    w = np.ascontiguousarray(want).view(np.uint32).ravel()
    bad = np.nonzero(g != w)[0]
    assert bad.size == 0, f"{what}: {bad.size} mismatches, first at {bad[:5]}: got {g[bad[:5]]} want {w[bad[:5]]}"


# ---- golden vectors through the CUDA path -----------------------------------

def test_silu_boundary_corpus_on_device(fam):
    args = fbits([a for a, _ in G["silu"]["cases"]])
    y = host(fam.silu(cuda(args)))
    assert bits_of(y) == [h(w) for _, w in G["silu"]["cases"]]


def test_rms_norm_corpus_on_device(fam):
    eps = h(G["rms_norm"]["eps_bits"])
    for case in G["rms_norm"]["cases"]:
        x = (fbits(case["x_bits"]) if "x_bits" in case else fvals(case["x"]))[None, :]
        w = np.array(case["w"], np.float32)
        y = host(fam.rms_norm(cuda(x), cuda(w), eps))
        assert bits_of(y) == [h(v) for v in case["y"]], case["cite"]
    for case in G["rms_norm"]["uniform"]:
        x = np.full((1, case["extent"]), case["fill"], np.float32)
        if case["hole_last"]:
            x[0, -1] = 0
        y = bits_of(host(fam.rms_norm(cuda(x), cuda(np.ones(case["extent"], np.float32)), eps)))
        assert y[0] == h(case["y0"]) and y[-1] == h(case["ylast"]), case["cite"]


def test_softmax_corpus_on_device(fam):
    for case in G["softmax"]["cases"]:
        x = (fbits(case["x_bits"]) if "x_bits" in case else fvals(case["x"]))[None, :]
        y = host(fam.softmax(cuda(x)))
        want = [h(case["y_all"])] * x.size if "y_all" in case else [h(v) for v in case["y"]]
        assert bits_of(y) == want, case["cite"]


def test_sum_goldens_on_device(fam):
    S = G["sums"]
    for case in S["strict"]:
        x = (fbits(case["x_bits"]) if "x_bits" in case else fvals(case["x"])).reshape(case["rows"], case["count"])
        y = host(fam.strict_sum_f32(cuda(x)))
        want = [h(v) for v in case["y"]] if isinstance(case["y"][0], str) else bits_of(case["y"])
        assert bits_of(y) == want
    for case in S["partitioned"]:
        x = (fbits(case["x_bits"]) if "x_bits" in case else fvals(case["x"])).reshape(case["rows"], case["count"])
        y = host(fam.partitioned_sum_f32(cuda(x), case["partitions"], case["per"]))
        want = [h(v) for v in case["y_bits"]] if "y_bits" in case else bits_of(case["y"])
        assert bits_of(y) == want, case["cite"]
    for case in S["cooperative"]:
        x = fvals(case["x"]).reshape(case["rows"], case["count"])
        y = host(fam.cooperative_sum_f32(cuda(x), case["participants"], case["per"], case["rounds"],
                                         case["participant_major"]))
        if "y" in case:
            assert bits_of(y) == bits_of(case["y"])
        else:
            assert bits_of(y)[0] == bits_of([case["y0"]])[0]


def test_quantize_affine_goldens_on_device(fam):
    for c in G["quantize_affine"]["quantize"]:
        x = fbits([c["x_bits"]]) if "x_bits" in c else np.array([c["x"]], np.float32)
        codes = host(fam.quantize_affine_u8(cuda(x), c["scale"], c["zero_point"], c["maximum"]))
        assert int(codes[0]) == c["code"]
    for nb in G["quantize_affine"]["nan_refused"]:
        with pytest.raises(fam.TilerCudaError) as e:
            fam.quantize_affine_u8(cuda(fbits(["0x3f800000", nb])), 0.5, 8, 15)
        assert e.value.code == 4 and e.value.position == 1
    for c in G["quantize_affine"]["dequantize"]:
        y = host(fam.dequantize_affine_u8(cuda(np.array([c["code"]], np.uint8)), c["scale"], c["zero_point"]))
        assert bits_of(y)[0] == h(c["y_bits"])


def test_gather_conformance_on_device(fam):
    Gt = G["gather"]
    table = np.arange(15, dtype=np.int32).reshape(5, 3)
    for case in Gt["cases"]:
        if not case["ids"]:
            continue
        y = host(fam.gather_rows(cuda(table), cuda(np.array(case["ids"], np.int32))))
        assert y.ravel().tolist() == case["bits"], case["cite"]
    for case in Gt["refused"]:
        with pytest.raises(fam.TilerCudaError) as e:
            fam.gather_rows(cuda(table), cuda(np.array(case["ids"], np.int32)))
        assert (e.value.position, e.value.value, e.value.extent) == (case["position"], case["value"], case["extent"])
    p = Gt["payloads"]
    src = np.array([h(b) for b in p["source_bits"]], np.uint32).view(np.int32)
    y = host(fam.gather_rows(cuda(src), cuda(np.array(p["ids"], np.int32))))
    assert y.view(np.uint32).tolist() == [h(b) for b in p["bits"]]


@pytest.mark.parametrize("cell_id", ["w_decode_kv", "w_prefill_q", "w_prefill_mlp_in", "w_prefill_mlp_out",
                                     "w_prefill_o", "w_vocab_slice"])
def test_contraction_profile_digests_on_device(fam, cell_id):
    P = G["contraction_profile_cells"]
    cell = next(c for c in P["cells"] if c["id"] == cell_id)
    seed = h(P["workload_seed"])
    a = prng_values(seed, cell["m"] * cell["k"]).reshape(cell["m"], cell["k"])
    b = prng_values(seed ^ h(P["right_seed_mask"]), cell["n"] * cell["k"]).reshape(cell["n"], cell["k"])
    c = host(fam.contract_f32(cuda(a), cuda(b)))
    assert hashlib.sha256(c.astype("<f4").tobytes()).hexdigest() == cell["sha256"]


# ---- seeded parity against the oracle -----------------------------------------

@pytest.mark.parametrize("rows,count", [(1, 1 << 24), (1, 1 << 20), (3, 100_003), (4, 65536), (1, 1), (2, 5000),
                                        (7, 4096 * 3)])
def test_grouped_sum_and_max_match_declared_grouping(fam, oracle_lib, rows, count):
    x = seeded_uniform(11 + count, rows * count).reshape(rows, count)
    g = fam.plan_grouping(rows, count)
    got = host(fam.sum_f32(cuda(x), g))
    st, want = oracle_lib.grid_fold(x, g, op=0, nthreads=8)
    assert st == 0
    assert_bits_equal(got, want, f"sum {g}")
    got = host(fam.max_f32(cuda(x), g))
    _, want = oracle_lib.grid_fold(x, g, op=1, nthreads=8)
    assert_bits_equal(got, want, "max")
    # the maximum is order-free: any grouping equals the strict fold
    _, strict = oracle_lib.strict_max(x)
    assert_bits_equal(got, strict, "max vs strict")


def test_grouped_sum_reports_a_difference_against_the_neighbouring_grouping(fam, oracle_lib):
    """The perturbation the reference's conformance runs demand: the kernel
    result must differ from a neighbouring grouping's on these operands, so
    the bit equality above is not vacuous."""
    count = 1 << 22
    x = (seeded_normal(5, count) * 1e4).astype(np.float32)
    g = fam.plan_grouping(1, count)
    got = host(fam.sum_f32(cuda(x), g))
    _, strict = oracle_lib.strict_sum(x)
    _, part = oracle_lib.partitioned_sum(x, 2048, count // 2048)
    assert bits_of(got) != bits_of(strict) or bits_of(got) != bits_of(part)


def test_explicit_groupings_including_padding_and_strict_combine(fam, oracle_lib):
    x = seeded_normal(9, 3 * 12_000).reshape(3, 12_000)
    for g in [dict(partitions=1, threads=64, k=1, rounds=188, combine_threads=0, combine_k=0, combine_rounds=0),
              dict(partitions=4, threads=128, k=4, rounds=6, combine_threads=0, combine_k=0, combine_rounds=0),
              dict(partitions=100, threads=64, k=2, rounds=1, combine_threads=64, combine_k=1, combine_rounds=2),
              dict(partitions=3, threads=1024, k=4, rounds=1, combine_threads=32, combine_k=1, combine_rounds=1)]:
        got = host(fam.sum_f32(cuda(x), g))
        st, want = oracle_lib.grid_fold(x, g, op=0)
        assert st == 0
        assert_bits_equal(got, want, str(g))


def test_reference_vocabulary_sums_match_the_oracle(fam, oracle_lib):
    x = seeded_normal(3, 4 * 4096).reshape(4, 4096) * 100
    assert_bits_equal(host(fam.strict_sum_f32(cuda(x))), oracle_lib.strict_sum(x)[1])
    assert_bits_equal(host(fam.partitioned_sum_f32(cuda(x), 64, 64)), oracle_lib.partitioned_sum(x, 64, 64)[1])
    for pm in (False, True):
        assert_bits_equal(host(fam.cooperative_sum_f32(cuda(x), 32, 8, 16, pm)),
                          oracle_lib.cooperative_sum(x, 32, 8, 16, pm)[1])


def test_serial_folds_at_every_batch_boundary(fam, oracle_lib):
    """The strict and partitioned folds at lengths around the load batch (8):
    1..40 and a few long ragged rows."""
    for count in list(range(1, 41)) + [1000, 4097]:
        x = seeded_normal(count, 3 * count).reshape(3, count) * 1e3
        assert_bits_equal(host(fam.strict_sum_f32(cuda(x))), oracle_lib.strict_sum(x)[1], f"strict {count}")
    for parts, per in [(3, 7), (5, 9), (2, 17), (4, 24)]:
        x = seeded_normal(per, 2 * parts * per).reshape(2, parts * per) * 1e3
        assert_bits_equal(host(fam.partitioned_sum_f32(cuda(x), parts, per)),
                          oracle_lib.partitioned_sum(x, parts, per)[1], f"partitioned {parts}x{per}")


def test_empty_sum_is_positive_zero_and_empty_max_is_refused(fam):
    x = torch.empty((3, 0), dtype=torch.float32, device="cuda")
    assert bits_of(host(fam.strict_sum_f32(x))) == [0, 0, 0]
    with pytest.raises(Exception):
        fam.max_f32(x, dict(partitions=1, threads=32, k=1, rounds=1))


@pytest.mark.parametrize("rows,extent,full_w", [(8192, 4096, False), (300, 4096, True), (37, 1000, False),
                                                (5, 12, True), (1, 4096, False), (129, 2048, False)])
def test_rms_norm_f32_matches_oracle(fam, oracle_lib, rows, extent, full_w):
    x = seeded_normal(rows * 7 + extent, rows * extent).reshape(rows, extent)
    w = seeded_uniform(3, rows * extent if full_w else extent, 0.5, 1.5)
    w = w.reshape(rows, extent) if full_w else w
    got = host(fam.rms_norm(cuda(x), cuda(w)))
    st, want = oracle_lib.rms_norm_f32(x, w, nthreads=8)
    assert st == 0
    assert_bits_equal(got, want, f"rms f32 {rows}x{extent}")


@pytest.mark.parametrize("rows,extent", [(8192, 4096), (77, 4096), (9, 100), (300, 4088), (50, 1000), (149, 4096)])
def test_rms_norm_bf16_matches_oracle(fam, oracle_lib, rows, extent):
    """The streamed bf16 kernel with full 1 KB chunks (4096), a short last
    chunk (4088), only short chunks (1000) and about one row per CTA (149
    rows); 100 elements (200-byte rows) take the unaligned kernel."""
    x = oracle_lib.f32_to_bf16(seeded_normal(rows + extent, rows * extent).reshape(rows, extent))
    w = oracle_lib.f32_to_bf16(seeded_uniform(4, extent, 0.5, 1.5))
    xt = cuda(x.view(np.int16)).view(torch.bfloat16)
    wt = cuda(w.view(np.int16)).view(torch.bfloat16)
    got = host(fam.rms_norm(xt, wt).view(torch.int16)).view(np.uint16)
    st, want = oracle_lib.rms_norm_bf16(x, w, nthreads=8)
    assert st == 0
    assert (got == want).all(), f"{(got != want).sum()} bf16 mismatches"


@pytest.mark.parametrize("extent,eps_bits", [(1, 1), (1, 0x358637BD), (4, 1), (4, 0x358637BD)])
def test_rms_norm_scale_sweeps_the_certified_rsqrt(fam, oracle_lib, extent, eps_bits):
    """Millions of rows whose mean square t spans every binade (subnormal t,
    overflow to +inf included), so the certified reciprocal square root of
    the row scale is decided against the oracle's over ~2^21 distinct t."""
    rows = 1 << 21
    rng = np.random.default_rng(extent * 7 + eps_bits % 97)
    mant = rng.integers(0, 1 << 23, rows * extent, dtype=np.uint32)
    expo = rng.integers(127 - 80, 127 + 70, rows * extent, dtype=np.uint32)
    sign = rng.integers(0, 2, rows * extent, dtype=np.uint32) << 31
    x = (sign | (expo << 23) | mant).view(np.float32).reshape(rows, extent)
    w = np.ones(extent, np.float32)
    got = host(fam.rms_norm(cuda(x), cuda(w), eps_bits=eps_bits))
    st, want = oracle_lib.rms_norm_f32(x, w, eps_bits=eps_bits, nthreads=16)
    assert st == 0
    assert_bits_equal(got, want, f"rms f32 rsqrt sweep extent {extent} eps {eps_bits:#x}")


def _fold_stress_rows(seed, rows, extent):
    """Rows that drive the warp-cooperative strict fold of the squares through
    every event it has: binade crossings from tiny first squares, exact ties
    (coarse value grids), running values below 2^-103 (folded one at a time),
    overflow to +inf, NaN and inf inputs, all-zero and subnormal rows."""
    rng = np.random.default_rng(seed)
    x = rng.standard_normal((rows, extent)).astype(np.float32)
    for r in range(rows):
        kind = r % 14
        v = x[r]
        if kind == 1:
            v[:] = np.round(v * 8) / 8  # squares on a coarse grid: ties
        elif kind == 2:
            v[:] = np.round(v * 64) / 64
        elif kind == 3:
            v[:] = np.ldexp(v, -60)  # running value near 2^-103..2^-120
        elif kind == 4:
            v[:] = np.ldexp(v, -75)  # squares underflow toward subnormals
        elif kind == 5:
            v[:] = np.ldexp(v, 62)  # the fold overflows to +inf
        elif kind == 6:
            v[0] = 1e-30  # the fold starts tiny, then jumps
        elif kind == 7:
            v[:] = 0.0
        elif kind == 8:
            v[rng.integers(extent)] = np.nan
        elif kind == 9:
            v[rng.integers(extent)] = np.inf
        elif kind == 10:
            v[:] = np.ldexp(v, rng.integers(-40, 40, extent)).astype(np.float32)
        elif kind == 11:
            v[:] = np.sqrt(rng.integers(0, 4096, extent)).astype(np.float32)
        elif kind == 12:
            v[:] = np.ldexp(np.float32(1.0), -140) * rng.integers(1, 64, extent)  # subnormal inputs
        elif kind == 13:
            v[rng.integers(extent)] = np.inf
            v[rng.integers(extent)] = np.nan
    return x


@pytest.mark.parametrize("extent", [4096, 4092, 1000, 260, 8])
def test_rms_norm_f32_fold_stress_rows_match_oracle(fam, oracle_lib, extent):
    rows = 14 * 9
    x = _fold_stress_rows(extent, rows, extent)
    w = seeded_uniform(6, extent, 0.5, 1.5)
    got = host(fam.rms_norm(cuda(x), cuda(w)))
    st, want = oracle_lib.rms_norm_f32(x, w, nthreads=8)
    assert st == 0
    assert_bits_equal(got, want, f"rms f32 stress {extent}")


@pytest.mark.parametrize("extent", [4096, 8192, 1000, 8])
def test_rms_norm_bf16_fold_stress_rows_match_oracle(fam, oracle_lib, extent):
    rows = 14 * 9
    x = oracle_lib.f32_to_bf16(_fold_stress_rows(extent + 1, rows, extent))
    w = oracle_lib.f32_to_bf16(seeded_uniform(8, extent, 0.5, 1.5))
    xt = cuda(x.view(np.int16)).view(torch.bfloat16)
    wt = cuda(w.view(np.int16)).view(torch.bfloat16)
    got = host(fam.rms_norm(xt, wt).view(torch.int16)).view(np.uint16)
    st, want = oracle_lib.rms_norm_bf16(x, w, nthreads=8)
    assert st == 0
    bad = np.argwhere(got != want)
    assert bad.size == 0, f"{len(bad)} mismatches, first {bad[:4].tolist()}"


def test_rms_norm_quantize_fusion_fold_stress_rows(fam, oracle_lib):
    extent = 4096
    x = _fold_stress_rows(99, 14 * 4, extent)
    keep = [r for r in range(x.shape[0]) if r % 14 not in (4, 5, 7, 8, 9, 12, 13)]  # rows the quantize refuses
    x = np.ascontiguousarray(x[keep])
    w = seeded_uniform(5, extent, 0.5, 1.5)
    st, y = oracle_lib.rms_norm_f32(x, w, nthreads=8)
    st, wc, ws, _ = oracle_lib.quantize_i8_rows(y, nthreads=8)
    if st != 0:
        pytest.skip("stress rows outside the quantize domain")
    codes, scales = fam.rms_norm_quantize_i8(cuda(x), cuda(w))
    assert (host(codes) == wc).all()
    assert_bits_equal(host(scales), ws)


def test_rms_norm_bf16_special_values_match_oracle(fam, oracle_lib):
    # rows whose outputs are NaN (NaN or inf input), overflow to inf (huge
    # weight), fall to bf16 subnormals (one huge and many tiny inputs), are
    # all zero, or sit on bf16 rounding ties; per-row weights
    extent = 4096
    rows = 8
    base = seeded_normal(41, rows * extent).reshape(rows, extent)
    x = base.copy()
    w = np.ones((rows, extent), np.float32)
    x[0, 17] = np.nan
    x[1, 3000] = np.inf
    w[2, :] = 3.0e38
    x[3, :] = 1e-30
    x[3, 5] = 1e30
    x[4, :] = 0.0
    x[5, :] = -x[5, :]
    w[6, :] = np.float32(1.0) + np.float32(2.0 ** -8)  # products land on bf16 ties often
    x[7, ::2] = np.float32(2.0 ** -126)
    xb = oracle_lib.f32_to_bf16(x)
    wb = oracle_lib.f32_to_bf16(w)
    xt = cuda(xb.view(np.int16)).view(torch.bfloat16)
    wt = cuda(wb.view(np.int16)).view(torch.bfloat16)
    got = host(fam.rms_norm(xt, wt).view(torch.int16)).view(np.uint16)
    st, want = oracle_lib.rms_norm_bf16(xb, wb)
    assert st == 0
    bad = np.argwhere(got != want)
    assert bad.size == 0, f"{len(bad)} mismatches, first {bad[:4].tolist()}: {got[tuple(bad[0])]:#x} vs {want[tuple(bad[0])]:#x}"


@pytest.mark.parametrize("rows,extent,period", [(2048, 2048, 2048), (64, 2048, 0), (33, 1000, 0), (16, 8192, 16),
                                                (5, 6, 3)])
def test_softmax_matches_oracle(fam, oracle_lib, rows, extent, period):
    x = seeded_normal(rows + extent, rows * extent, std=3.0).reshape(rows, extent)
    got = host(fam.softmax(cuda(x), causal_period=period))
    st, want = oracle_lib.softmax_f32(x, causal_period=period, nthreads=8)
    assert st == 0
    assert_bits_equal(got, want, f"softmax {rows}x{extent}")


@pytest.mark.parametrize("rows,extent,mask_rows,row_offset", [(64, 2048, 64, 0), (100, 1000, 16, 5), (7, 8, 3, 2)])
def test_softmax_with_a_mask_tensor_matches_oracle(fam, oracle_lib, rows, extent, mask_rows, row_offset):
    # softmax(x + mask[(row_offset + r) mod mask_rows]): the add rounds once and
    # canonicalizes NaN, then the reference softmax
    x = seeded_normal(rows + 3, rows * extent).reshape(rows, extent) * 3
    mask = seeded_normal(mask_rows + 1, mask_rows * extent).reshape(mask_rows, extent)
    mask[seeded_uniform(6, mask_rows * extent, 0, 1).reshape(mask_rows, extent) < 0.3] = -np.inf
    x[3 % rows, 1] = np.inf  # +inf + finite = +inf: that row's maximum is +inf
    got = host(fam.softmax_masked(cuda(x), cuda(mask), row_offset=row_offset))
    with np.errstate(invalid="ignore"):
        t = x + mask[(row_offset + np.arange(rows)) % mask_rows]
    t[np.isnan(t)] = np.array([0x7FC00000], np.uint32).view(np.float32)[0]
    st, want = oracle_lib.softmax_f32(t, nthreads=8)
    assert st == 0
    assert_bits_equal(got, want, "masked softmax")


@pytest.mark.parametrize("extent", [1000, 2048])
def test_softmax_mask_tensor_trailing_runs_match_oracle(fam, oracle_lib, extent):
    """Mask rows ending in -inf runs of every length around the warp's scan
    step (0 .. extent, the whole row included), a NaN mask entry, and x that
    is NaN, +inf or -inf under a run (NaN and +inf poison the row)."""
    tails = [0, 1, 3, 4, 5, 31, 32, 33, 127, 128, 129, 130, extent // 2, extent - 4, extent - 1, extent]
    mask = seeded_normal(extent, len(tails) * extent).reshape(len(tails), extent)
    for i, tl in enumerate(tails):
        if tl:
            mask[i, extent - tl:] = -np.inf
    mask[2, 10] = -np.inf  # an interior -inf before a live entry
    mask[4, extent - 6] = np.nan  # a NaN entry just before the run
    rows = 4 * len(tails)
    x = seeded_normal(extent + 7, rows * extent).reshape(rows, extent) * 3
    for i, tl in enumerate(tails):
        if tl:
            x[len(tails) + i, extent - 1] = np.nan
            x[2 * len(tails) + i, extent - tl] = np.inf
            x[3 * len(tails) + i, extent - 1] = -np.inf
    got = host(fam.softmax_masked(cuda(x), cuda(mask)))
    with np.errstate(invalid="ignore"):
        t = x + mask[np.arange(rows) % len(tails)]
    t[np.isnan(t)] = np.array([0x7FC00000], np.uint32).view(np.float32)[0]
    st, want = oracle_lib.softmax_f32(t, nthreads=8)
    assert st == 0
    assert_bits_equal(got, want, f"masked softmax trailing runs, extent {extent}")


def test_softmax_causal_mask_tensor_equals_the_in_kernel_mask(fam):
    # the 0 / -inf block-causal mask as a tensor gives the in-kernel mask's bits,
    # poisoned rows (NaN or +inf under the mask) included
    rows, extent = 4096, 2048
    gen = torch.Generator("cuda").manual_seed(21)
    x = torch.randn(rows, extent, device="cuda", generator=gen) * 3
    x[5, 2000] = float("nan")
    x[6, 1999] = float("inf")
    col = torch.arange(extent, device="cuda")
    mask = torch.where(col[None, :] > torch.arange(extent, device="cuda")[:, None], float("-inf"), 0.0)
    got = fam.softmax_masked(x, mask.contiguous())
    want = fam.softmax(x, causal_period=extent)
    assert torch.equal(got.view(torch.int32), want.view(torch.int32))


def test_softmax_full_config_sampled_rows(fam, oracle_lib):
    rows, extent = 65536, 2048
    x = torch.randn(rows, extent, device="cuda", generator=torch.Generator("cuda").manual_seed(1)) * 3
    y = host(fam.softmax(x, causal_period=2048))
    xs = x.cpu().numpy()
    sample = np.arange(0, rows, 509)
    st, want = oracle_lib.softmax_f32(xs[sample], causal_period=0, nthreads=8)
    # the oracle call above sees unmasked rows; apply the mask explicitly
    masked = xs[sample].copy()
    for i, r in enumerate(sample):
        masked[i, (r % 2048) + 1:] = masked[i, (r % 2048) + 1:] + np.float32(-np.inf)
    st, want = oracle_lib.softmax_f32(masked, nthreads=8)
    assert_bits_equal(y[sample], want, "softmax full-config sample")
    # size-independent property: each row's masked tail is exactly +0.0
    assert (y[2047, :] > 0).all() and (y[0, 1:] == 0).all()


def test_silu_random_bit_patterns_match_oracle(fam, oracle_lib):
    rng = np.random.default_rng(17)
    bits = rng.integers(0, 2**32, size=1 << 20, dtype=np.uint64).astype(np.uint32)
    x = bits.view(np.float32)
    dense = seeded_normal(2, 1 << 20, std=20.0)
    for arr in (x, dense):
        got = host(fam.silu(cuda(arr)))
        _, want = oracle_lib.silu_f32(arr)
        assert_bits_equal(got, want, "silu")


def test_silu_dense_sweep_and_ragged_tail_match_oracle(fam, oracle_lib):
    """x dense over [-120, 120] (every exponent band of exp(-x), both range
    guards at -89 and 104) at a length that leaves a 3-element tail."""
    x = np.linspace(-120, 120, (1 << 21) + 3, dtype=np.float32)
    got = host(fam.silu(cuda(x)))
    _, want = oracle_lib.silu_f32(x)
    assert_bits_equal(got, want, "silu sweep")


def test_silu_staged_division_matches_ieee_division_on_every_argument(fam):
    """The staged SiLU map divides by Markstein's method (hardware reciprocal
    estimate, one Newton step, one remainder correction) and the unaligned
    form by the IEEE division; over every binary32 argument (2^32 bit
    patterns, in chunks) the two give the same bits.  The unaligned form is
    reached through a buffer offset by one element."""
    chunk = 1 << 28
    base = torch.arange(chunk, dtype=torch.int64, device="cuda")
    xbuf = torch.empty(chunk + 1, dtype=torch.float32, device="cuda")
    ya = torch.empty(chunk, dtype=torch.float32, device="cuda")
    ybuf = torch.empty(chunk + 1, dtype=torch.float32, device="cuda")
    for c in range(1 << 32 >> 28):
        v = base + c * chunk
        v = torch.where(v >= (1 << 31), v - (1 << 32), v).to(torch.int32).view(torch.float32)
        xs = xbuf[1:]
        xs.copy_(v)
        fam.silu(v, out=ya, check=False)
        fam.silu(xs, out=ybuf[1:], check=False)
        diff = ya.view(torch.int32) != ybuf[1:].view(torch.int32)
        n = int(diff.sum())
        assert n == 0, f"chunk {c}: {n} mismatches, first arguments " + str(
            [hex(int(u) & 0xffffffff) for u in v.view(torch.int32)[torch.nonzero(diff)[:4].flatten()]])


def test_softmax_exp_band_sweep_matches_oracle(fam, oracle_lib):
    """Every exponent band the certified exp covers: rows of x with max 0, so
    exp(x) is evaluated on [-104, 0] densely."""
    x = -np.linspace(0, 110, 1 << 16, dtype=np.float32).reshape(32, 2048)
    x[:, 0] = 0
    got = host(fam.softmax(cuda(x)))
    _, want = oracle_lib.softmax_f32(x, nthreads=8)
    assert_bits_equal(got, want, "exp sweep")


@pytest.mark.parametrize("n,offset", [(1, 0), (3, 0), (4, 0), (2047, 0), (2048 * 5 + 1, 0), (9999, 1), (9999, 3),
                                      (3_000_001, 0)])
def test_elementwise_maps_sizes_and_alignment(fam, oracle_lib, n, offset):
    """The staged maps (16-byte aligned x and y: bulk-copied tiles, a partial
    last tile, a tail of n % 4 elements) and the unaligned grid-stride form."""
    x = seeded_normal(5, n + offset, std=30.0)
    xd = cuda(x)[offset:]
    yd = torch.empty(n + offset, device="cuda")[offset:]
    got = host(fam.silu(xd, out=yd))
    _, want = oracle_lib.silu_f32(x[offset:])
    assert_bits_equal(got, want, f"silu n={n} offset={offset}")
    a, b = np.float32(0.75), np.float32(1.0e-3)
    got = host(fam.scale_bias(xd, torch.tensor(a).cuda(), torch.tensor(b).cuda(), out=yd))
    _, want = oracle_lib.scale_bias_f32(x[offset:], a, b)
    assert_bits_equal(got, want, f"scale_bias n={n} offset={offset}")


def test_scale_bias_matches_oracle(fam, oracle_lib):
    x = seeded_normal(1, 100_001)
    a = np.float32(1.0000001)
    b = np.float32(-3.5)
    got = host(fam.scale_bias(cuda(x), torch.tensor(a).cuda(), torch.tensor(b).cuda()))
    _, want = oracle_lib.scale_bias_f32(x, a, b)
    assert_bits_equal(got, want)
    a2 = seeded_normal(2, 100_001)
    got = host(fam.scale_bias(cuda(x), cuda(a2), torch.tensor(b).cuda()))
    with pytest.raises(ValueError):
        fam.scale_bias(cuda(x), cuda(a2[:10]), torch.tensor(b).cuda())
    _, want = oracle_lib.scale_bias_f32(x, a2, np.array([b]))
    assert_bits_equal(got, want)


# shapes on both sides of the staged kernels' limits: quantize stages rows of
# at most 16 KB with extent % 4 == 0; decode stages extent % 16 == 0 up to 4096
@pytest.mark.parametrize("rows,extent", [(16384, 4096), (3, 1001), (37, 4096), (5, 4100), (9, 4092), (4, 8192),
                                         (300, 16), (2, 4)])
def test_quantize_decode_match_oracle(fam, oracle_lib, rows, extent):
    x = seeded_normal(rows, rows * extent).reshape(rows, extent)
    codes, scales = fam.quantize_i8_rows(cuda(x))
    st, wc, ws, _ = oracle_lib.quantize_i8_rows(x, nthreads=8)
    assert st == 0
    assert (host(codes) == wc).all()
    assert_bits_equal(host(scales), ws)
    y = host(fam.dequantize_i8_rows(codes, scales))
    _, wy = oracle_lib.dequantize_i8_rows(wc, ws, nthreads=8)
    assert_bits_equal(y, wy)


@pytest.mark.parametrize("rows,extent,full_w", [(8192, 4096, False), (37, 1024, True), (300, 16, False)])
def test_rms_norm_quantize_fusion_matches_the_composed_oracle(fam, oracle_lib, rows, extent, full_w):
    # the fused family equals quantize_i8_rows(rms_norm_f32(x, w)) bit for bit
    x = seeded_normal(rows + 7, rows * extent).reshape(rows, extent)
    w = seeded_uniform(5, rows * extent if full_w else extent, 0.5, 1.5)
    w = w.reshape(rows, extent) if full_w else w
    codes, scales = fam.rms_norm_quantize_i8(cuda(x), cuda(w))
    st, y = oracle_lib.rms_norm_f32(x, w, nthreads=8)
    assert st == 0
    st, wc, ws, _ = oracle_lib.quantize_i8_rows(y, nthreads=8)
    assert st == 0
    assert (host(codes) == wc).all()
    assert_bits_equal(host(scales), ws)


def test_rms_norm_quantize_fusion_refusals(fam):
    extent = 256
    x = seeded_normal(9, 4 * extent).reshape(4, extent)
    w = np.ones(extent, np.float32)
    bad = x.copy()
    bad[2, 100] = np.nan  # the whole y row is NaN: its first column is reported
    with pytest.raises(fam.TilerCudaError) as e:
        fam.rms_norm_quantize_i8(cuda(bad), cuda(w))
    assert e.value.code == 4 and e.value.position == 2 * extent
    zero = x.copy()
    zero[1, :] = 0.0  # y = 0: the scale is +0, not positive-normal
    with pytest.raises(fam.TilerCudaError) as e:
        fam.rms_norm_quantize_i8(cuda(zero), cuda(w))
    assert e.value.code == 9 and e.value.position == 1 * extent
    with pytest.raises(fam.TilerCudaError):  # extent not a multiple of 4
        fam.rms_norm_quantize_i8(cuda(x[:, :255].copy()), cuda(w[:255].copy()))


def test_quantize_half_integer_ties_are_exact(fam, oracle_lib):
    # rows whose quotients land on k + 0.5 exactly and within an ulp of it
    s = np.float32(127.0) / np.float32(127.0)
    row = np.array([127.0, 0.5, 1.5, 2.5, -0.5, -1.5, 63.5, np.nextafter(np.float32(2.5), np.float32(3)),
                    np.nextafter(np.float32(2.5), np.float32(2))], np.float32)
    x = np.tile(row, (4, 1)) * np.array([[1.0], [0.5], [3.0], [1e-3]], np.float32)
    codes, scales = fam.quantize_i8_rows(cuda(x))
    st, wc, ws, _ = oracle_lib.quantize_i8_rows(x)
    assert (host(codes) == wc).all() and s == 1


def test_quantize_refusals(fam):
    x = np.ones((3, 8), np.float32)
    x[1, 5] = np.nan
    with pytest.raises(fam.TilerCudaError) as e:
        fam.quantize_i8_rows(cuda(x))
    assert e.value.code == 4 and e.value.position == 13
    with pytest.raises(fam.TilerCudaError) as e:
        fam.quantize_i8_rows(cuda(np.zeros((2, 8), np.float32)))
    assert e.value.code == 9 and e.value.position == 0


@pytest.mark.parametrize("dtype,rows,extent,chunk", [(torch.float32, 8192, 4096, 0), (torch.float32, 1000, 1024, 300),
                                                    (torch.bfloat16, 777, 4096, 100), (torch.float32, 17, 256, 0),
                                                    (torch.bfloat16, 1000, 1024, 0)])
def test_rms_norm_host_buffers_match_the_device_path(fam, dtype, rows, extent, chunk):
    # chunked upload / kernel / download gives the device path's bits, for a
    # broadcast weight row and for a per-row weight matrix
    gen = torch.Generator().manual_seed(rows)
    x = torch.randn(rows, extent, generator=gen).to(dtype).pin_memory()
    for w_full in (False, True):
        w = (torch.rand((rows, extent) if w_full else (extent,), generator=gen) + 0.5).to(dtype).cuda()
        want = fam.rms_norm(x.cuda(), w).cpu()
        got = fam.rms_norm_host(x, w, chunk_rows=chunk)
        assert torch.equal(got.view(torch.int16 if dtype == torch.bfloat16 else torch.int32),
                           want.view(torch.int16 if dtype == torch.bfloat16 else torch.int32))


def test_quantize_staged_rows_refusals_and_extremes(fam, oracle_lib):
    # 4096-wide rows take the shared-memory staged kernel: the first NaN of
    # the earliest refused row is reported, and extreme magnitudes (largest
    # finite, smallest subnormal) code like the oracle
    x = seeded_normal(4, 4 * 4096).reshape(4, 4096)
    x[0, 17] = np.float32(3.4028235e38)
    x[1, 5] = np.float32(1e-45)
    codes, scales = fam.quantize_i8_rows(cuda(x))
    st, wc, ws, _ = oracle_lib.quantize_i8_rows(x)
    assert st == 0 and (host(codes) == wc).all()
    assert_bits_equal(host(scales), ws)
    bad = x.copy()
    bad[2, 3000] = np.nan
    bad[2, 3500] = np.nan
    bad[3, 10] = np.inf
    with pytest.raises(fam.TilerCudaError) as e:
        fam.quantize_i8_rows(cuda(bad))
    assert e.value.code == 4 and e.value.position == 2 * 4096 + 3000


def test_a_bounded_device_wait_that_runs_out_reports_a_timeout_and_the_context_stays_usable(fam, oracle_lib):
    # the wait every kernel uses, on an mbarrier phase nothing completes, with a
    # 20 ms limit: the status word reports TIMEOUT and later launches still work
    from tiler_b200 import _native as N
    st = fam.StatusWord()
    st.reset()
    t0 = time.monotonic()
    assert N.lib().tiler_cuda_bounded_wait_selftest(fam.context(), torch.cuda.current_stream().cuda_stream,
                                                    st.ptr, 20_000_000) == 0
    torch.cuda.synchronize()
    assert time.monotonic() - t0 < 5.0
    assert st.fetch().code == N.TIMEOUT
    x = seeded_normal(3, 8 * 64).reshape(8, 64)
    w = np.ones(64, np.float32)
    got = host(fam.rms_norm(cuda(x), cuda(w)))
    _, want = oracle_lib.rms_norm_f32(x, w)
    assert_bits_equal(got, want)


def test_gather_full_config_is_bit_exact(fam):
    gen = torch.Generator("cuda").manual_seed(3)
    table = (torch.randn(128256, 4096, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    ids = torch.randint(0, 128256, (8192,), device="cuda", dtype=torch.int32, generator=gen)
    got = fam.gather_rows(table, ids)
    want = table.index_select(0, ids.long())
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    bad = ids.clone()
    bad[4000] = -7
    bad[5000] = 128256
    with pytest.raises(fam.TilerCudaError) as e:
        fam.gather_rows(table, bad)
    assert (e.value.position, e.value.value, e.value.extent) == (4000, -7, 128256)


@pytest.mark.parametrize("m,n,k", [(128, 256, 64), (256, 512, 1024), (384, 768, 512), (512, 256, 192), (1024, 1280, 320)])
def test_gemm_bf16_silu_matches_oracle(fam, oracle_lib, m, n, k):
    a = oracle_lib.f32_to_bf16(seeded_normal(m + k, m * k).reshape(m, k))
    b = oracle_lib.f32_to_bf16(seeded_normal(n + k, n * k).reshape(n, k) * 0.05)
    at = cuda(a.view(np.int16)).view(torch.bfloat16)
    bt = cuda(b.view(np.int16)).view(torch.bfloat16)
    for epi in ("none", "silu"):
        got = oracle_lib.bf16_to_f32(host(fam.gemm_bf16(at, bt, epilogue=epi).view(torch.int16)).view(np.uint16))
        st, want = oracle_lib.gemm_bf16_silu(a, b, apply_silu=(epi == "silu"), nthreads=8)
        want = oracle_lib.bf16_to_f32(want)
        err = np.abs(got - want) / np.maximum(np.abs(want), 1e-2)
        assert err.max() <= 1e-2, f"{epi}: max rel err {err.max()}"


def test_gemm_bf16_writes_a_strided_output_inside_its_columns(fam):
    # C with a row pitch wider than n (ldc = n + 256): the TMA-stored boxes land
    # in C's columns only; the padding keeps its sentinel
    m, n, k = 256, 512, 256
    gen = torch.Generator("cuda").manual_seed(11)
    a = (torch.randn(m, k, device="cuda", generator=gen) * 0.1).to(torch.bfloat16)
    b = (torch.randn(n, k, device="cuda", generator=gen) * 0.1).to(torch.bfloat16)
    want = fam.gemm_bf16(a, b, epilogue="silu")
    wide = torch.full((m, n + 256), -7.0, device="cuda", dtype=torch.bfloat16)
    got = fam.gemm_bf16(a, b, epilogue="silu", out=wide[:, :n])
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))
    assert (wide[:, n:] == -7.0).all()


def test_gemm_bf16_full_config_sampled_rows(fam, oracle_lib):
    m, n, k = 8192, 14336, 4096
    gen = torch.Generator("cuda").manual_seed(5)
    a = (torch.randn(m, k, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    b = (torch.randn(n, k, device="cuda", generator=gen) * 0.02).to(torch.bfloat16)
    c = fam.gemm_bf16(a, b, epilogue="silu")
    # one row from each CTA of every 256-row pair tile (rows 0-127 of a tile
    # come from the first CTA's accumulator, 128-255 from the second's), plus
    # the tile edges at both ends
    rng = np.random.default_rng(17)
    rows = sorted({0, 1, 127, 128, 255, 4095, 8191} |
                  {t * 256 + h * 128 + int(rng.integers(0, 128)) for t in range(m // 256) for h in range(2)})
    an = a.view(torch.int16).cpu().numpy().view(np.uint16)
    bn = b.view(torch.int16).cpu().numpy().view(np.uint16)
    got = oracle_lib.bf16_to_f32(c.view(torch.int16).cpu().numpy().view(np.uint16)[rows])
    want = np.stack([oracle_lib.bf16_to_f32(oracle_lib.gemm_bf16_silu(an, bn, r, r + 1, nthreads=8)[1])[0]
                     for r in rows])
    err = np.abs(got - want) / np.maximum(np.abs(want), 1e-3)
    assert err.max() <= 1e-2, f"max rel err {err.max()}"


def test_gemm_silu_epilogue_is_the_bf16_rounding_of_the_certified_silu(fam, oracle_lib):
    """With one-hot rows of A, each accumulator equals one bf16 value of B
    exactly, so C = bf16(SiLU(v)) must equal the oracle's rounding of the
    certified binary32 SiLU bit for bit, across the whole bf16 grid that
    SiLU maps to finite values."""
    grid = np.arange(0, 1 << 16, dtype=np.uint32).astype(np.uint16)
    vals = oracle_lib.bf16_to_f32(grid)
    keep = grid[np.isfinite(vals) & (np.abs(vals) < 200)]
    n = 256
    cols = ((keep.size + n - 1) // n) * n
    bvals = np.zeros(cols, np.uint16)
    bvals[:keep.size] = keep
    k = 64
    m = 256  # rows 0 and 128: the first rows of both CTAs of a cta_group::2 pair
    a = np.zeros((m, k), np.uint16)
    a[np.arange(m), np.arange(m) % k] = oracle_lib.f32_to_bf16(np.ones(1, np.float32))[0]
    b = np.zeros((cols, k), np.uint16)
    b[:, 0] = bvals  # only row 0 of A (one-hot at column 0) picks column 0 of B
    at = cuda(a.view(np.int16)).view(torch.bfloat16)
    bt = cuda(b.view(np.int16)).view(torch.bfloat16)
    c = host(fam.gemm_bf16(at, bt, epilogue="silu").view(torch.int16)).view(np.uint16)
    got = c[0, :keep.size]
    # the oracle contraction of row 0 (1 * v summed with 0 * 0 terms: -0 becomes +0, as in the reference fold)
    _, want = oracle_lib.gemm_bf16_silu(a, b, 0, 1, nthreads=8)
    want = want[0, :keep.size]
    bad = np.nonzero(got != want)[0]
    assert bad.size == 0, (bad[:5], keep[bad[:5]], got[bad[:5]], want[bad[:5]])
    # row 128 is one-hot at column 0 as well
    assert np.array_equal(c[128, :keep.size], want)


def test_route_a_program_through_the_runtime_adapter(fam, oracle_lib):
    from tiler_b200 import adapter as A
    x = seeded_normal(40, 64 * 4096).reshape(64, 4096)
    w = seeded_uniform(41, 4096, 0.5, 1.5)
    ad = A.CudaRuntimeAdapter(device=torch.cuda.current_device())
    payload = A.Payload("sm_100a", 32, (A.Entry("rms", "tiler_cuda.rms_norm_f32"),
                                          A.Entry("sum", "tiler_cuda.sum_f32.grouped")))
    out = A.route_with_adapter(payload, [A.Launch("rms", {"x": cuda(x), "w": cuda(w)}),
                                         A.Launch("sum", {"x": cuda(x.reshape(-1))})], ad)
    ad.close()
    assert_bits_equal(host(out[0]), oracle_lib.rms_norm_f32(x, w)[1])
    g = fam.plan_grouping(1, x.size)
    assert_bits_equal(host(out[1]).reshape(1), oracle_lib.grid_fold(x.reshape(-1), g)[1])
    assert ad.trace.index("commit") < ad.trace.index("dispatch")


def test_saturated_parallel_fold_steps_is_measured(fam):
    """The measured cost row: the dispatch sweep over the three sum
    strategies fits the work-span model with a positive P and step."""
    from tiler_b200 import target_profile as tp
    cells = tp.measure_fold_cells(fam, torch, repeats=5)
    assert {c["strategy"] for c in cells} == {"strict", "partitioned", "grouped"}
    fit = tp.fit_work_span(cells)
    assert fit["parallel_steps"] > 32 and fit["step_s"] > 0 and fit["residual"] < 1.0
    (key, value, _), = tp.cost_rows(round(fit["parallel_steps"]))
    assert key == tp.COST_ROW_KEY and value > 0
