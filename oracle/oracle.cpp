// CPU parity oracle — TEST INFRASTRUCTURE ONLY (see oracle.h for the pinning
// statement).  Every function cites the moderately-ai/tiler reference
// file:line whose semantics it restates.  Build: oracle/Makefile
// (-O2 -ffp-contract=off, no fast-math: one IEEE rounding per operator).
#include "oracle.h"

#include <math.h>
#include <quadmath.h>
#include <string.h>

#include <algorithm>
#include <functional>
#include <thread>
#include <vector>

namespace {

constexpr uint32_t kCanonicalNanBits = 0x7fc00000u;  // tiler-ir semantic/operation.rs:21

float from_bits(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
uint32_t to_bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

// canonicalize_arithmetic_f32 — crates/tiler-reference/src/lib.rs:144-150
float canon(float v) { return isnan(v) ? from_bits(kCanonicalNanBits) : v; }

// Runs body(begin, end) over [0, n) split across up to nthreads threads.
void parallel_rows(uint64_t n, int32_t nthreads, const std::function<void(uint64_t, uint64_t)>& body) {
  int32_t t = nthreads < 1 ? 1 : nthreads;
  if (t == 1 || n < 2) { body(0, n); return; }
  if ((uint64_t)t > n) t = (int32_t)n;
  std::vector<std::thread> pool;
  uint64_t chunk = (n + t - 1) / t;
  for (int32_t i = 0; i < t; ++i) {
    uint64_t b = i * chunk, e = std::min(n, b + chunk);
    if (b >= e) break;
    pool.emplace_back(body, b, e);
  }
  for (auto& th : pool) th.join();
}

// Certification of a quad-precision candidate against the binary32 rounding
// midpoints, the role `rounds_to` plays in crates/tiler-reference/src/silu.rs:286-304
// and rms_norm.rs:394-411: the value is decided only when the enclosure
// [q - err, q + err] lies strictly between the two midpoints around f.
bool certified(__float128 q, float f) {
  const __float128 err = fabsq(q) * 0x1p-100Q;
  if (isinf(f)) {
    const __float128 threshold = 0x1p128Q - 0x1p103Q;  // silu.rs:246-249
    return q - err > threshold;
  }
  __float128 fv = f;
  __float128 lower, upper;
  if (f == 0.0f) {
    lower = 0;  // a positive exponential has nothing below zero (silu.rs:291-295)
    upper = (fv + (__float128)from_bits(1)) / 2;
    return q - err > lower && q + err < upper;
  }
  float below = nextafterf(f, -INFINITY), above = nextafterf(f, INFINITY);
  lower = (fv + (__float128)below) / 2;
  upper = isinf(above) ? (0x1p128Q - 0x1p103Q) : (fv + (__float128)above) / 2;
  return q - err > lower && q + err < upper;
}

}  // namespace

extern "C" {

float oracle_canonicalize(float v) { return canon(v); }

// maximum_f32 — crates/tiler-reference/src/softmax.rs:168-186 (IEEE 754-2019
// `maximum`: NaN-propagating, opposite zeros decided by AND of the bits).
float oracle_maximum(float a, float b) {
  if (isnan(a) || isnan(b)) return from_bits(kCanonicalNanBits);
  if (a == b) return from_bits(to_bits(a) & to_bits(b));
  return a > b ? a : b;
}

// certified_exp_strict — crates/tiler-reference/src/silu.rs:220-277.
float oracle_exp(float x, int32_t* undecided) {
  if (isnan(x)) return from_bits(kCanonicalNanBits);
  if (x >= 89.0f) return INFINITY;    // EXPONENTIAL_OVERFLOW_GUARD, silu.rs:71
  if (x <= -104.0f) return 0.0f;      // EXPONENTIAL_UNDERFLOW_GUARD, silu.rs:74
  if (x == 0.0f) return 1.0f;
  __float128 q = expq((__float128)x);
  float f = (float)q;  // one RNE rounding of the quad value
  if (!certified(q, f) && undecided) *undecided = 1;
  return f;
}

// certified_rsqrt_strict — crates/tiler-reference/src/rms_norm.rs:238-293.
float oracle_rsqrt(float t, int32_t* undecided) {
  if (isnan(t)) return from_bits(kCanonicalNanBits);
  if (isinf(t) && t > 0) return 0.0f;
  if (t == 0.0f) return signbit(t) ? -INFINITY : INFINITY;
  if (t < 0.0f) return from_bits(kCanonicalNanBits);
  __float128 q = 1 / sqrtq((__float128)t);
  float f = (float)q;
  // An even power of two has a dyadic, exactly representable reciprocal root.
  if ((__float128)f * (__float128)f * (__float128)t == 1) return f;
  if (!certified(q, f) && undecided) *undecided = 1;
  return f;
}

// silu_f32_under — crates/tiler-reference/src/silu.rs:158-180.
float oracle_silu(float x, int32_t* undecided) {
  if (isnan(x)) return from_bits(kCanonicalNanBits);
  if (isinf(x)) return x > 0 ? x : from_bits(kCanonicalNanBits);
  float e = oracle_exp(-x, undecided);
  float d = 1.0f + e;
  return canon(x / d);
}

// Bf16Format::round of a binary32 value: one RNE rounding, canonical NaN
// 0x7fc0 — crates/tiler-reference/src/bf16.rs:393-580.
uint16_t oracle_f32_to_bf16(float v) {
  if (isnan(v)) return 0x7fc0;
  uint32_t b = to_bits(v);
  b += 0x7fffu + ((b >> 16) & 1u);
  return (uint16_t)(b >> 16);
}

float oracle_bf16_to_f32(uint16_t b) { return from_bits((uint32_t)b << 16); }

// ---- reductions ----------------------------------------------------------

// strict_sum — crates/tiler-reference/src/evaluate.rs:498-589: seeded at the
// first contributor, empty domain commits +0.0, result canonicalized.
int32_t oracle_strict_sum(const float* x, uint64_t rows, uint64_t count, float* out) {
  for (uint64_t r = 0; r < rows; ++r) {
    if (count == 0) { out[r] = 0.0f; continue; }
    const float* s = x + r * count;
    float acc = s[0];
    for (uint64_t i = 1; i < count; ++i) acc = canon(acc + s[i]);
    out[r] = canon(acc);
  }
  return ORACLE_OK;
}

// strict_partial_sums + strict_partitioned_sum —
// crates/tiler-reference/src/evaluate.rs:612-832.
int32_t oracle_partitioned_sum(const float* x, uint64_t rows, uint64_t count,
                               uint64_t partitions, uint64_t per, float* out) {
  if (partitions == 0 || partitions * per != count) return ORACLE_INVALID_APPLICATION;
  std::vector<float> partials(partitions);
  for (uint64_t r = 0; r < rows; ++r) {
    for (uint64_t p = 0; p < partitions; ++p) {
      if (per == 0) { partials[p] = 0.0f; continue; }
      const float* s = x + r * count + p * per;
      float acc = s[0];
      for (uint64_t i = 1; i < per; ++i) acc = canon(acc + s[i]);
      partials[p] = canon(acc);
    }
    oracle_strict_sum(partials.data(), 1, partitions, out + r);
  }
  return ORACLE_OK;
}

// cooperative_grouped_sum / fold_cooperative_sequence —
// crates/tiler-reference/src/evaluate.rs:844-1158 (CooperativeGrouping:
// RoundMajor cell r*P+p, ParticipantMajor cell p*R+r; each fold seeded at its
// first contributor, round 0 seeds the total).
int32_t oracle_cooperative_sum(const float* x, uint64_t rows, uint64_t count,
                               uint64_t participants, uint64_t per, uint64_t rounds,
                               int32_t participant_major, float* out) {
  if (participants == 0 || per == 0 || rounds == 0 || participants * per * rounds != count)
    return ORACLE_INVALID_APPLICATION;
  for (uint64_t row = 0; row < rows; ++row) {
    const float* s = x + row * count;
    float total = 0.0f;
    for (uint64_t r = 0; r < rounds; ++r) {
      float staged = 0.0f;
      for (uint64_t p = 0; p < participants; ++p) {
        uint64_t cell = participant_major ? p * rounds + r : r * participants + p;
        const float* c = s + cell * per;
        float partial = c[0];
        for (uint64_t i = 1; i < per; ++i) partial = canon(partial + c[i]);
        staged = p == 0 ? partial : canon(staged + partial);
      }
      total = r == 0 ? staged : canon(total + staged);
    }
    out[row] = canon(total);
  }
  return ORACLE_OK;
}

}  // extern "C"

namespace {

inline float fold_op(int32_t op, float a, float b) {
  return op == 0 ? canon(a + b) : oracle_maximum(a, b);
}

// The ADR-0096/0100 two-level composition with rounds, restated from
// docs/decisions/0100-admit-the-multi-round-two-level-reduction-composition.md
// decisions 1-5 and docs/decisions/0096-...md decisions 1,5,6 and
// docs/decisions/0094-...md decision 4 (no reference evaluator exists):
//   block index (r, g, l) -> r*T + g*32 + l, each block k contiguous
//   contributors folded strictly; an ascending-mask XOR butterfly
//   (1,2,4,8,16) over the 32 lanes, result lane 0; a strict fold over the G
//   staged warp slots; round totals folded in ascending order, round 0 peeled.
//   Tail padding only, with the two-sided identity -0.0 (sum) or -inf (max).
float compose_fold_seq(const float* seq, uint64_t n, uint32_t T, uint32_t k, uint32_t R, int32_t op) {
  const float identity = op == 0 ? from_bits(0x80000000u) : from_bits(0xff800000u);
  const uint32_t G = T / 32;
  float total = 0.0f;
  std::vector<float> lanes(32), slots(G);
  for (uint32_t r = 0; r < R; ++r) {
    for (uint32_t g = 0; g < G; ++g) {
      for (uint32_t l = 0; l < 32; ++l) {
        uint64_t base = ((uint64_t)r * T + (uint64_t)g * 32 + l) * k;
        float v = base < n ? seq[base] : identity;
        for (uint32_t i = 1; i < k; ++i) {
          float c = base + i < n ? seq[base + i] : identity;
          v = fold_op(op, v, c);
        }
        lanes[l] = v;
      }
      for (uint32_t m = 1; m < 32; m <<= 1) {
        float next[32];
        for (uint32_t l = 0; l < 32; ++l) next[l] = fold_op(op, lanes[l], lanes[l ^ m]);
        for (uint32_t l = 0; l < 32; ++l) lanes[l] = next[l];
      }
      slots[g] = lanes[0];
    }
    float staged = slots[0];
    for (uint32_t g = 1; g < G; ++g) staged = fold_op(op, staged, slots[g]);
    total = r == 0 ? staged : fold_op(op, total, staged);
  }
  return canon(total);
}

bool composition_canonical(uint64_t n, uint32_t T, uint32_t k, uint32_t R) {
  if (T == 0 || T % 32 != 0 || k == 0 || R == 0 || n == 0) return false;
  uint64_t per_round = (uint64_t)T * k;
  return per_round * (R - 1) < n && n <= per_round * R;  // ADR-0100 decision 2
}

}  // namespace

extern "C" {

int32_t oracle_compose_fold(const float* seq, uint64_t n, uint32_t threads, uint32_t k,
                            uint32_t rounds, int32_t op, float* out) {
  if (!composition_canonical(n, threads, k, rounds)) return ORACLE_INVALID_APPLICATION;
  *out = compose_fold_seq(seq, n, threads, k, rounds, op);
  return ORACLE_OK;
}

int32_t oracle_grid_fold(const float* x, uint64_t rows, uint64_t count, uint64_t partitions,
                         uint32_t threads, uint32_t k, uint32_t rounds, uint32_t combine_threads,
                         uint32_t combine_k, uint32_t combine_rounds, int32_t op,
                         int32_t nthreads, float* out) {
  if (partitions == 0 || count % partitions != 0) return ORACLE_INVALID_APPLICATION;
  uint64_t per = count / partitions;
  if (!composition_canonical(per, threads, k, rounds)) return ORACLE_INVALID_APPLICATION;
  if (combine_threads != 0 && !composition_canonical(partitions, combine_threads, combine_k, combine_rounds))
    return ORACLE_INVALID_APPLICATION;
  std::vector<float> partials(rows * partitions);
  parallel_rows(rows * partitions, nthreads, [&](uint64_t b, uint64_t e) {
    for (uint64_t i = b; i < e; ++i)
      partials[i] = compose_fold_seq(x + i * per, per, threads, k, rounds, op);
  });
  for (uint64_t r = 0; r < rows; ++r) {
    const float* p = partials.data() + r * partitions;
    if (combine_threads == 0) {
      float acc = p[0];
      for (uint64_t i = 1; i < partitions; ++i) acc = fold_op(op, acc, p[i]);
      out[r] = canon(acc);
    } else {
      out[r] = compose_fold_seq(p, partitions, combine_threads, combine_k, combine_rounds, op);
    }
  }
  return ORACLE_OK;
}

// Strict maximum fold (identity-less: empty refused) — softmax.rs:273-279.
int32_t oracle_strict_max(const float* x, uint64_t rows, uint64_t count, float* out) {
  if (count == 0) return ORACLE_INVALID_APPLICATION;
  for (uint64_t r = 0; r < rows; ++r) {
    const float* s = x + r * count;
    float m = s[0];
    for (uint64_t i = 1; i < count; ++i) m = oracle_maximum(m, s[i]);
    out[r] = canon(m);
  }
  return ORACLE_OK;
}

}  // extern "C"

// ---- row families ----------------------------------------------------------

namespace {

// RowGeometry::row_scale — crates/tiler-reference/src/rms_norm.rs:136-194:
// strict left fold of x*x seeded at the first square, mean = total / N
// (division), t = mean + eps, scale = correctly rounded 1/sqrt(t).
float rms_row_scale(const float* x, uint64_t extent, float eps) {
  float total = 0.0f;
  for (uint64_t i = 0; i < extent; ++i) {
    float sq = x[i] * x[i];
    total = i == 0 ? sq : total + sq;
  }
  float mean = extent == 0 ? total : total / (float)extent;
  return oracle_rsqrt(mean + eps, nullptr);
}

bool eps_admitted(uint32_t eps_bits) {
  float eps = from_bits(eps_bits);
  return eps > 0.0f && isfinite(eps);  // rms_norm.rs:465-467
}

}  // namespace

extern "C" {

// normalize_dense — crates/tiler-reference/src/rms_norm.rs:453-489:
// y = w * (x * scale), two roundings in that order, NaN canonicalized.
int32_t oracle_rms_norm_f32(const float* x, const float* w, int64_t w_row_stride,
                            uint64_t rows, uint64_t extent, uint32_t eps_bits,
                            float* y, int32_t nthreads) {
  if (!eps_admitted(eps_bits) || extent > (1ull << 24)) return ORACLE_INVALID_APPLICATION;
  const float eps = from_bits(eps_bits);
  parallel_rows(rows, nthreads, [&](uint64_t b, uint64_t e) {
    for (uint64_t r = b; r < e; ++r) {
      const float* xr = x + r * extent;
      const float* wr = w + (int64_t)r * w_row_stride;
      float scale = rms_row_scale(xr, extent, eps);
      for (uint64_t i = 0; i < extent; ++i) {
        float normalized = xr[i] * scale;
        y[r * extent + i] = canon(wr[i] * normalized);
      }
    }
  });
  return ORACLE_OK;
}

// Config extension (no bf16 RMS in the reference): bf16 x and w widen
// exactly to binary32, the f32 path above runs, the result rounds once to
// bf16 (RNE, canonical NaN 0x7fc0).
int32_t oracle_rms_norm_bf16(const uint16_t* x, const uint16_t* w, int64_t w_row_stride,
                             uint64_t rows, uint64_t extent, uint32_t eps_bits,
                             uint16_t* y, int32_t nthreads) {
  if (!eps_admitted(eps_bits) || extent > (1ull << 24)) return ORACLE_INVALID_APPLICATION;
  const float eps = from_bits(eps_bits);
  parallel_rows(rows, nthreads, [&](uint64_t b, uint64_t e) {
    std::vector<float> xf(extent);
    for (uint64_t r = b; r < e; ++r) {
      for (uint64_t i = 0; i < extent; ++i) xf[i] = oracle_bf16_to_f32(x[r * extent + i]);
      const uint16_t* wr = w + (int64_t)r * w_row_stride;
      float scale = rms_row_scale(xf.data(), extent, eps);
      for (uint64_t i = 0; i < extent; ++i) {
        float normalized = xf[i] * scale;
        y[r * extent + i] = oracle_f32_to_bf16(oracle_bf16_to_f32(wr[i]) * normalized);
      }
    }
  });
  return ORACLE_OK;
}

// row_softmax — crates/tiler-reference/src/softmax.rs:260-315: strict
// maximum fold, e_i = certified exp(x_i - m), strict left fold of e seeded
// at e_0, r = 1/d, out_i = e_i * r, NaN canonicalized.  The causal mask is
// the program's upstream add of -inf (standard.rs:211-221): element (row,
// col) becomes x + (-inf) when col > (row_offset + row) mod causal_period.
int32_t oracle_softmax_f32(const float* x, uint64_t rows, uint64_t extent,
                           uint64_t causal_period, uint64_t row_offset,
                           float* y, int32_t nthreads) {
  if (extent == 0) return ORACLE_OK;
  parallel_rows(rows, nthreads, [&](uint64_t b, uint64_t e) {
    std::vector<float> v(extent);
    for (uint64_t r = b; r < e; ++r) {
      const float* xr = x + r * extent;
      uint64_t diag = causal_period ? (row_offset + r) % causal_period : 0;
      for (uint64_t i = 0; i < extent; ++i)
        v[i] = (causal_period && i > diag) ? xr[i] + (-INFINITY) : xr[i];
      float m = v[0];
      for (uint64_t i = 1; i < extent; ++i) m = oracle_maximum(m, v[i]);
      for (uint64_t i = 0; i < extent; ++i) v[i] = oracle_exp(v[i] - m, nullptr);
      float d = v[0];
      for (uint64_t i = 1; i < extent; ++i) d = d + v[i];
      float rcp = 1.0f / d;
      for (uint64_t i = 0; i < extent; ++i) y[r * extent + i] = canon(v[i] * rcp);
    }
  });
  return ORACLE_OK;
}

// SiluF32Reference::evaluate — crates/tiler-reference/src/silu.rs:78-110.
int32_t oracle_silu_f32(const float* x, uint64_t n, float* y) {
  for (uint64_t i = 0; i < n; ++i) y[i] = canon(oracle_silu(x[i], nullptr));
  return ORACLE_OK;
}

// `binary` Multiply then Add — crates/tiler-reference/src/evaluate.rs:448-485
// and standard.rs:105-120: y = (x*a) + b with two roundings; a rank-0 operand
// broadcasts.
int32_t oracle_scale_bias_f32(const float* x, uint64_t n, const float* a, int32_t a_scalar,
                              const float* b, int32_t b_scalar, float* y) {
  for (uint64_t i = 0; i < n; ++i) {
    float p = canon(x[i] * (a_scalar ? a[0] : a[i]));
    y[i] = canon(p + (b_scalar ? b[0] : b[i]));
  }
  return ORACLE_OK;
}

// GatherF32Reference — crates/tiler-reference/src/structural.rs:513-606 with
// decide_gather_index (tiler-ir semantic/gather.rs:438): rows are copied
// bit-exactly; the first out-of-range index (in position order) refuses the
// whole operation with {position, value, extent}.  i32 ids (negative = out
// of range) are the config extension of the reference's u32 ids.
int32_t oracle_gather_rows(const void* table, uint64_t table_rows, uint64_t row_bytes,
                           const void* ids, int32_t ids_unsigned, uint64_t n_ids,
                           void* out, oracle_error* err) {
  for (uint64_t i = 0; i < n_ids; ++i) {
    int64_t v = ids_unsigned ? (int64_t)((const uint32_t*)ids)[i] : (int64_t)((const int32_t*)ids)[i];
    if (v < 0 || (uint64_t)v >= table_rows) {
      if (err) { err->code = ORACLE_GATHER_INDEX_OUT_OF_BOUNDS; err->position = i; err->value = v; err->extent = table_rows; }
      return ORACLE_GATHER_INDEX_OUT_OF_BOUNDS;
    }
    memcpy((char*)out + i * row_bytes, (const char*)table + (uint64_t)v * row_bytes, row_bytes);
  }
  return ORACLE_OK;
}

// Config extension of strict-affine quantize (crates/tiler-reference/src/
// quantization.rs:404-430): signed codes, per-row scale = maximum|x| / 127
// (the maximum fold of softmax.rs:168-186 over |x|, then one division), zero
// point 0, code = RNE(clamp(x/scale + 0, -127, 127)).  A NaN element refuses
// (quantization.rs:411-413); a scale outside positive-normal refuses
// (read_scale_value, quantization.rs:377-379).  The first error in
// row-major order is reported.
int32_t oracle_quantize_i8_rows(const float* x, uint64_t rows, uint64_t extent,
                                int8_t* codes, float* scales, oracle_error* err,
                                int32_t nthreads) {
  if (extent == 0) return ORACLE_INVALID_APPLICATION;
  std::vector<uint64_t> first_error(rows, UINT64_MAX);
  std::vector<int32_t> error_code(rows, 0);
  parallel_rows(rows, nthreads, [&](uint64_t b, uint64_t e) {
    for (uint64_t r = b; r < e; ++r) {
      const float* xr = x + r * extent;
      float m = fabsf(xr[0]);
      uint64_t nan_at = UINT64_MAX;
      for (uint64_t i = 0; i < extent; ++i) {
        if (isnan(xr[i]) && nan_at == UINT64_MAX) nan_at = i;
        if (i) m = oracle_maximum(m, fabsf(xr[i]));
      }
      if (nan_at != UINT64_MAX) { first_error[r] = r * extent + nan_at; error_code[r] = ORACLE_NAN_INPUT; continue; }
      float scale = m / 127.0f;
      scales[r] = scale;
      if (!isnormal(scale) || scale <= 0.0f) { first_error[r] = r * extent; error_code[r] = ORACLE_SCALE_DOMAIN; continue; }
      for (uint64_t i = 0; i < extent; ++i) {
        float s = xr[i] / scale;
        float t = s + 0.0f;
        float c = std::min(std::max(t, -127.0f), 127.0f);
        codes[r * extent + i] = (int8_t)nearbyintf(c);  // default rounding mode: ties-to-even
      }
    }
  });
  for (uint64_t r = 0; r < rows; ++r) {
    if (error_code[r]) {
      if (err) { err->code = error_code[r]; err->position = first_error[r]; err->value = 0; err->extent = rows * extent; }
      return error_code[r];
    }
  }
  return ORACLE_OK;
}

// dequantize_one — crates/tiler-reference/src/quantization.rs:440-451 with
// zero point 0: code 0 decodes to +0.0, else code * scale (one rounding).
int32_t oracle_dequantize_i8_rows(const int8_t* codes, const float* scales, uint64_t rows,
                                  uint64_t extent, float* y, int32_t nthreads) {
  parallel_rows(rows, nthreads, [&](uint64_t b, uint64_t e) {
    for (uint64_t r = b; r < e; ++r)
      for (uint64_t i = 0; i < extent; ++i) {
        int8_t c = codes[r * extent + i];
        y[r * extent + i] = c == 0 ? 0.0f : (float)c * scales[r];
      }
  });
  return ORACLE_OK;
}

// The reference's own strict-affine family (per-tensor scale, unsigned U4/U8
// codes): quantize_one / dequantize_one, quantization.rs:404-451, with the
// scale domain of read_scale_value (:356-381).
int32_t oracle_quantize_affine_u8(const float* x, uint64_t n, float scale, uint32_t zero_point,
                                  uint32_t maximum, uint8_t* codes, oracle_error* err) {
  if (!isnormal(scale) || scale <= 0.0f || (maximum != 15 && maximum != 255) || zero_point > maximum)
    return ORACLE_INVALID_APPLICATION;
  for (uint64_t i = 0; i < n; ++i) {
    if (isnan(x[i])) {
      if (err) { err->code = ORACLE_NAN_INPUT; err->position = i; err->value = 0; err->extent = n; }
      return ORACLE_NAN_INPUT;
    }
    float s = x[i] / scale;
    float t = s + (float)zero_point;
    float c = std::min(std::max(t, 0.0f), (float)maximum);
    codes[i] = (uint8_t)nearbyintf(c);
  }
  return ORACLE_OK;
}

int32_t oracle_dequantize_affine_u8(const uint8_t* codes, uint64_t n, float scale,
                                    uint32_t zero_point, float* y) {
  if (!isnormal(scale) || scale <= 0.0f || zero_point > 255) return ORACLE_INVALID_APPLICATION;
  for (uint64_t i = 0; i < n; ++i) {
    int32_t d = (int32_t)codes[i] - (int32_t)zero_point;
    y[i] = codes[i] == zero_point ? 0.0f : (float)d * scale;
  }
  return ORACLE_OK;
}

// ---- contraction -------------------------------------------------------

// evaluate_outputs — crates/tiler-reference/src/contraction.rs:558-630 for
// the profile's `td,od->to` structure (contraction_profile_cells.rs:224-236):
// seed = first product, product and accumulation rounded separately.
int32_t oracle_contract_f32(const float* a, const float* b, uint64_t m, uint64_t n,
                            uint64_t k, float* c, int32_t nthreads) {
  if (k == 0) return ORACLE_INVALID_APPLICATION;
  parallel_rows(m, nthreads, [&](uint64_t rb, uint64_t re) {
    for (uint64_t i = rb; i < re; ++i)
      for (uint64_t j = 0; j < n; ++j) {
        const float* ar = a + i * k;
        const float* br = b + j * k;
        float acc = canon(ar[0] * br[0]);
        for (uint64_t d = 1; d < k; ++d) acc = canon(acc + canon(ar[d] * br[d]));
        c[i * n + j] = canon(acc);
      }
  });
  return ORACLE_OK;
}

// Config extension: bf16 operands widened exactly to binary32 (a bf16 x bf16
// product is exact in binary32), the contraction's strict f32 fold, the SiLU
// epilogue of silu.rs:158-180, one RNE rounding to bf16.
int32_t oracle_gemm_bf16_silu(const uint16_t* a, const uint16_t* b, uint64_t m, uint64_t n,
                              uint64_t k, uint64_t row_begin, uint64_t row_end,
                              int32_t apply_silu, uint16_t* c, int32_t nthreads) {
  if (k == 0 || row_end > m || row_begin > row_end) return ORACLE_INVALID_APPLICATION;
  parallel_rows(row_end - row_begin, nthreads, [&](uint64_t rb, uint64_t re) {
    std::vector<float> af(k);
    for (uint64_t ii = rb; ii < re; ++ii) {
      uint64_t i = row_begin + ii;
      for (uint64_t d = 0; d < k; ++d) af[d] = oracle_bf16_to_f32(a[i * k + d]);
      for (uint64_t j = 0; j < n; ++j) {
        const uint16_t* br = b + j * k;
        float acc = af[0] * oracle_bf16_to_f32(br[0]);
        for (uint64_t d = 1; d < k; ++d) acc = acc + af[d] * oracle_bf16_to_f32(br[d]);
        float v = apply_silu ? oracle_silu(acc, nullptr) : canon(acc);
        c[ii * n + j] = oracle_f32_to_bf16(v);
      }
    }
  });
  return ORACLE_OK;
}

}  // extern "C"
