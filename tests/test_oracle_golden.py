"""Pins the CPU oracle against the known-answer vectors of the reference's own
tests (tests/golden/reference_vectors.json, each citing its file:line).
CPU only."""
import hashlib

import numpy as np
import pytest

from golden_util import bits_of, f, fbits, fvals, h, load, prng_values

G = load()


def _x(case, key="x"):
    return fbits(case[key + "_bits"]) if key + "_bits" in case else fvals(case[key])


def test_certified_exp(oracle_lib):
    for arg, want in G["exp"]["cases"]:
        assert bits_of([oracle_lib.exp(f(arg))])[0] == h(want), arg
    v = oracle_lib.exp(f(G["exp"]["subnormal_at"][0]))
    assert 0 < v < np.finfo(np.float32).tiny


def test_certified_rsqrt(oracle_lib):
    for arg, want in G["rsqrt"]["cases"]:
        assert bits_of([oracle_lib.rsqrt(f(arg))])[0] == h(want), arg
    for arg in G["rsqrt"]["nan_for"]:
        assert np.isnan(oracle_lib.rsqrt(f(arg)))
    sep = G["rsqrt"]["not_equal_to_one_over_sqrt"]
    eps = f(sep["argument"])
    composed = np.float32(1.0) / np.sqrt(eps)
    assert bits_of([composed])[0] == h(sep["composed"])
    assert bits_of([oracle_lib.rsqrt(eps)])[0] != h(sep["composed"])


def test_silu_boundary_corpus(oracle_lib):
    for arg, want in G["silu"]["cases"]:
        _, y = oracle_lib.silu_f32(fbits([arg]))
        assert bits_of(y)[0] == h(want), arg


def test_maximum(oracle_lib):
    for a, b, want in G["maximum"]["cases"]:
        assert bits_of([oracle_lib.maximum(f(a), f(b))])[0] == h(want), (a, b)


def test_rms_norm_corpus(oracle_lib):
    eps = h(G["rms_norm"]["eps_bits"])
    for case in G["rms_norm"]["cases"]:
        x = _x(case)[None, :]
        w = np.array(case["w"], dtype=np.float32)
        st, y = oracle_lib.rms_norm_f32(x, w, eps)
        assert st == 0
        assert bits_of(y) == [h(v) for v in case["y"]], case["cite"]
    for case in G["rms_norm"]["uniform"]:
        x = np.full((1, case["extent"]), case["fill"], dtype=np.float32)
        if case["hole_last"]:
            x[0, -1] = 0.0
        _, y = oracle_lib.rms_norm_f32(x, np.ones(case["extent"], np.float32), eps)
        assert bits_of(y)[0] == h(case["y0"]) and bits_of(y)[-1] == h(case["ylast"]), case["cite"]


def test_rms_norm_refuses_bad_eps(oracle_lib):
    x = np.ones((1, 4), np.float32)
    for eps in (0, 0x80000000, 0x7F800000, 0x7FC00000):
        st, _ = oracle_lib.rms_norm_f32(x, np.ones(4, np.float32), eps)
        assert st == oracle_lib.INVALID_APPLICATION


def test_softmax_corpus(oracle_lib):
    for case in G["softmax"]["cases"]:
        x = _x(case)[None, :]
        st, y = oracle_lib.softmax_f32(x)
        assert st == 0
        want = [h(case["y_all"])] * x.size if "y_all" in case else [h(v) for v in case["y"]]
        assert bits_of(y) == want, case["cite"]
    for case in G["softmax"]["row_sums"]:
        _, y = oracle_lib.softmax_f32(fvals(case["x"])[None, :])
        _, s = oracle_lib.strict_sum(y)
        assert bits_of(s)[0] == h(case["strict_sum"]), case["cite"]


def test_softmax_causal_mask_is_the_added_minus_infinity(oracle_lib):
    rng = np.random.default_rng(7)
    x = rng.standard_normal((8, 4)).astype(np.float32) * 3
    _, masked = oracle_lib.softmax_f32(x, causal_period=4)
    explicit = x.copy()
    for r in range(8):
        for c in range(4):
            if c > r % 4:
                explicit[r, c] = explicit[r, c] + np.float32(-np.inf)
    _, want = oracle_lib.softmax_f32(explicit)
    assert bits_of(masked) == bits_of(want)


def test_strict_and_split_sums(oracle_lib):
    S = G["sums"]
    for case in S["strict"]:
        x = (_x(case)).reshape(case["rows"], case["count"])
        st, y = oracle_lib.strict_sum(x)
        want = [h(v) for v in case["y"]] if isinstance(case["y"][0], str) else bits_of(case["y"])
        assert bits_of(y) == want, case["cite"]
    for case in S["partitioned"]:
        x = _x(case).reshape(case["rows"], case["count"])
        st, y = oracle_lib.partitioned_sum(x, case["partitions"], case["per"])
        assert st == 0
        want = [h(v) for v in case["y_bits"]] if "y_bits" in case else bits_of(case["y"])
        assert bits_of(y) == want, case["cite"]
    for case in S["partitioned_refused"]:
        x = np.ones((case["rows"], case["count"]), np.float32)
        for p, c in case["pairs"]:
            st, _ = oracle_lib.partitioned_sum(x, p, c)
            assert st == oracle_lib.INVALID_APPLICATION
    for case in S["cooperative"]:
        x = _x(case).reshape(case["rows"], case["count"])
        st, y = oracle_lib.cooperative_sum(x, case["participants"], case["per"], case["rounds"],
                                           case["participant_major"])
        assert st == 0
        if "y" in case:
            assert bits_of(y) == bits_of(case["y"]), case["cite"]
        else:
            assert bits_of(y)[0] == bits_of([case["y0"]])[0], case["cite"]
    for case in S["cooperative_refused"]:
        x = np.ones((case["rows"], case["count"]), np.float32)
        for p, c, r in case["groupings"]:
            st, _ = oracle_lib.cooperative_sum(x, p, c, r)
            assert st == oracle_lib.INVALID_APPLICATION


def test_one_round_cooperative_is_partitioned_and_one_partition_is_strict(oracle_lib):
    """The identities crates/tiler-reference/src/tests.rs:1885-1983 states."""
    rng = np.random.default_rng(3)
    x = (rng.standard_normal((3, 96)) * 1e3).astype(np.float32)
    _, coop = oracle_lib.cooperative_sum(x, 8, 12, 1)
    _, part = oracle_lib.partitioned_sum(x, 8, 12)
    assert bits_of(coop) == bits_of(part)
    _, one = oracle_lib.partitioned_sum(x, 1, 96)
    _, strict = oracle_lib.strict_sum(x)
    assert bits_of(one) == bits_of(strict)


def test_composition_reduces_to_reference_groupings(oracle_lib):
    """With every lane but lane 0 padded away the ADR-0100 composition is not
    a reference grouping; but with k covering a whole warp row (one warp,
    one round) lane folds + butterfly collapse checks are exercised against a
    direct restatement, and a fully-padded tail is identity-neutral."""
    rng = np.random.default_rng(5)
    seq = (rng.standard_normal(1000) * 100).astype(np.float32)
    # one warp, k=32, one round: lanes fold 32 contiguous, butterfly ascending
    st, v = oracle_lib.compose_fold(seq[:1024 - 24], 32, 32, 1)
    assert st == 0
    lanes = []
    s = seq[:1000]
    for l in range(32):
        chunk = s[l * 32:(l + 1) * 32]
        if chunk.size == 0:
            lanes.append(np.float32(-0.0))
            continue
        acc = chunk[0]
        for c in chunk[1:]:
            acc = np.float32(acc + c)
        lanes.append(acc)
    lanes = np.array(lanes, np.float32)
    m = 1
    while m < 32:
        lanes = np.array([np.float32(lanes[i] + lanes[i ^ m]) for i in range(32)], np.float32)
        m <<= 1
    assert bits_of([v])[0] == bits_of([lanes[0]])[0]
    # the canonicality rule of ADR-0100 decision 2: no all-padding round
    assert oracle_lib.compose_fold(seq[:64], 32, 1, 3)[0] == oracle_lib.INVALID_APPLICATION


def test_negative_zero_survives_the_composition(oracle_lib):
    """ADR-0100 decision 5: the peeled round 0 keeps a -0.0 row -0.0."""
    seq = np.full(100, -0.0, np.float32)
    st, v = oracle_lib.compose_fold(seq, 32, 1, 4)
    assert st == 0 and bits_of([v])[0] == 0x80000000


def test_quantize_affine(oracle_lib):
    Q = G["quantize_affine"]
    for c in Q["quantize"]:
        x = fbits([c["x_bits"]]) if "x_bits" in c else np.array([c["x"]], np.float32)
        st, codes, _ = oracle_lib.quantize_affine_u8(x, c["scale"], c["zero_point"], c["maximum"])
        assert st == 0 and int(codes[0]) == c["code"]
    for nb in Q["nan_refused"]:
        st, _, err = oracle_lib.quantize_affine_u8(fbits([nb]), 0.5, 8, 15)
        assert st == oracle_lib.NAN_INPUT and err.position == 0
    for c in Q["dequantize"]:
        st, y = oracle_lib.dequantize_affine_u8(np.array([c["code"]], np.uint8), c["scale"], c["zero_point"])
        assert bits_of(y)[0] == h(c["y_bits"])


def test_quantize_i8_rows_extension(oracle_lib):
    x = np.array([[0.0, 1.0, -2.0, 0.5], [3.0, -3.0, 1.5, 0.75]], np.float32)
    st, codes, scales, _ = oracle_lib.quantize_i8_rows(x)
    assert st == 0
    assert scales[0] == np.float32(2.0) / np.float32(127.0)
    assert codes[0].tolist() == [0, 64, -127, 32]   # 63.5 -> 64 (ties to even), 31.75 -> 32
    assert codes[1].tolist() == [127, -127, 64, 32]  # 63.5 -> 64, 31.75 -> 32
    st, y = oracle_lib.dequantize_i8_rows(codes, scales)
    assert bits_of(y)[0] == 0 and y[0, 2] == np.float32(-127) * scales[0]
    x[1, 2] = np.nan
    st, *_, err = oracle_lib.quantize_i8_rows(x)
    assert st == oracle_lib.NAN_INPUT and err.position == 6
    st, *_, err = oracle_lib.quantize_i8_rows(np.zeros((2, 3), np.float32))
    assert st == oracle_lib.SCALE_DOMAIN and err.position == 0


def test_gather_conformance(oracle_lib):
    Gt = G["gather"]
    table = np.arange(Gt["positional_source_rows"] * Gt["row_width"], dtype=np.uint32).reshape(
        Gt["positional_source_rows"], Gt["row_width"])
    for case in Gt["cases"]:
        st, out, _ = oracle_lib.gather_rows(table, np.array(case["ids"], np.uint32))
        assert st == 0 and out.ravel().tolist() == case["bits"], case["cite"]
    for case in Gt["refused"]:
        st, _, err = oracle_lib.gather_rows(table, np.array(case["ids"], np.uint32))
        assert st == oracle_lib.GATHER_INDEX_OUT_OF_BOUNDS
        assert (err.position, err.value, err.extent) == (case["position"], case["value"], case["extent"])
    p = Gt["payloads"]
    src = np.array([h(b) for b in p["source_bits"]], np.uint32)
    st, out, _ = oracle_lib.gather_rows(src, np.array(p["ids"], np.uint32))
    assert out.tolist() == [h(b) for b in p["bits"]]
    st, _, err = oracle_lib.gather_rows(table, np.array([1, -1], np.int32))
    assert st == oracle_lib.GATHER_INDEX_OUT_OF_BOUNDS and err.position == 1 and err.value == -1


def test_multiply_add_two_roundings(oracle_lib):
    c = G["multiply_add_two_roundings"]
    st, y = oracle_lib.scale_bias_f32(fbits([c["x_bits"]]), fbits([c["a_bits"]]), np.float32(c["b"]))
    assert bits_of(y)[0] == h(c["y_bits"])


@pytest.mark.parametrize("cell_id", ["w_decode_kv", "w_prefill_q", "w_vocab_slice", "w_prefill_o"])
def test_contraction_profile_digests(oracle_lib, cell_id):
    P = G["contraction_profile_cells"]
    cell = next(c for c in P["cells"] if c["id"] == cell_id)
    seed = h(P["workload_seed"])
    a = prng_values(seed, cell["m"] * cell["k"]).reshape(cell["m"], cell["k"])
    b = prng_values(seed ^ h(P["right_seed_mask"]), cell["n"] * cell["k"]).reshape(cell["n"], cell["k"])
    st, c = oracle_lib.contract_f32(a, b, nthreads=8)
    assert st == 0
    assert hashlib.sha256(c.astype("<f4").tobytes()).hexdigest() == cell["sha256"]


def test_bf16_round_to_nearest_even(oracle_lib):
    cases = {0x3F808000: 0x3F80, 0x3F818000: 0x3F82, 0x3F808001: 0x3F81, 0x7F7FFFFF: 0x7F80,
             0x00000001: 0x0000, 0x00008000: 0x0000, 0x00018000: 0x0002, 0x80000000: 0x8000,
             0x7FC01234: 0x7FC0, 0xFF800000: 0xFF80}
    for b, want in cases.items():
        v = np.array([b], np.uint32).view(np.float32)
        assert int(oracle_lib.f32_to_bf16(v)[0]) == want
        assert int(oracle_lib.lib().oracle_f32_to_bf16(float(v[0]))) == want
