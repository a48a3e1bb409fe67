// Shared device numerics and PTX helpers for the tiler-cuda kernels (sm_100a).
//
// Numerical rules restated from moderately-ai/tiler's tiler-reference:
//  * every binary32 + - * / is one IEEE RNE operation, subnormals preserved
//    (the library is built with -fmad=false and without -ftz / fast-math, and
//    the kernels spell the reference's separate roundings with __fadd_rn /
//    __fmul_rn / __fdiv_rn so no contraction can fuse them);
//  * arithmetic NaN results are canonicalized to 0x7fc00000
//    (crates/tiler-reference/src/lib.rs:144-150);
//  * exp and 1/sqrt are correctly rounded (certified) binary32 values
//    (silu.rs:220-277, rms_norm.rs:238-293).
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/tiler_cuda.h"

namespace tc {

constexpr uint32_t kCanonicalNan = 0x7fc00000u;

__host__ __device__ __forceinline__ uint64_t umin64(uint64_t a, uint64_t b) { return a < b ? a : b; }

__device__ __forceinline__ bool is_nan_bits(float v) { return (__float_as_uint(v) & 0x7fffffffu) > 0x7f800000u; }

__device__ __forceinline__ bool is_positive_normal(float v) {
  const uint32_t b = __float_as_uint(v);
  return (b >> 31) == 0 && (b >> 23) != 0 && (b >> 23) != 0xffu;
}

__device__ __forceinline__ float canon(float v) {
  return isnan(v) ? __uint_as_float(kCanonicalNan) : v;
}

// maximum_f32 — crates/tiler-reference/src/softmax.rs:168-186.
__device__ __forceinline__ float maximum(float a, float b) {
  if (isnan(a) || isnan(b)) return __uint_as_float(kCanonicalNan);
  if (a == b) return __uint_as_float(__float_as_uint(a) & __float_as_uint(b));
  return a > b ? a : b;
}

// Bf16 RNE rounding of a binary32 value, canonical NaN 0x7fc0
// (crates/tiler-reference/src/bf16.rs:393-580).
__device__ __forceinline__ uint16_t f32_to_bf16(float v) {
  if (isnan(v)) return 0x7fc0;
  uint32_t b = __float_as_uint(v);
  b += 0x7fffu + ((b >> 16) & 1u);
  return (uint16_t)(b >> 16);
}
__device__ __forceinline__ float bf16_to_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

// ---- device status word --------------------------------------------------

// error_key = (position << 8) | code; the smallest position wins.
__device__ __forceinline__ void report_error(tiler_cuda_status* s, uint64_t position, uint32_t code) {
  if (s) atomicMin((unsigned long long*)&s->error_key, (unsigned long long)((position << 8) | code));
}
__device__ __forceinline__ void report_value(tiler_cuda_status* s, uint64_t position, uint32_t value) {
  if (s) atomicMin((unsigned long long*)&s->value_key, (unsigned long long)((position << 32) | value));
}
__device__ __forceinline__ void report_undecided(tiler_cuda_status* s) {
  if (s) atomicAdd(&s->undecided, 1u);
}

// ---- correctly rounded exp --------------------------------------------------
//
// Tang's table-driven method (P. T. P. Tang, "Table-driven implementation of
// the exponential function in IEEE floating-point arithmetic", ACM TOMS 15(2),
// 1989) carried out in binary64 and rounded once to binary32, then certified:
//   x = (256 m + j) ln2/256 + r,  |r| <= ln2/512,
//   e^x = 2^m * 2^(j/256) * e^r,  e^r - 1 by its Taylor polynomial.
// The binary64 value carries a relative error below 2^-51; it is accepted
// only when it lies farther than 2^-49 (relative) from every binary32
// rounding midpoint.  Otherwise the rare slow path re-evaluates in
// double-double (error below 2^-100) and decides against the midpoints; a
// value still undecided there is counted in the status word, mirroring the
// reference's UndecidedTranscendentalReference refusal.
//
// The 2^(j/256) table (hi + lo doubles) is written once per device by the
// host runtime (abi.cu, from __float128 exp2q) into g_exp2_table; the fast
// path reads its hi column from a shared-memory copy.

// C names, so a payload module's copies are found by name (cuModuleGetGlobal)
// and written the same way when the module is loaded.
extern "C" {
__device__ double g_exp2_table[256][2];
__device__ double g_exp2_hi[256];  // the hi column again, contiguous (read where no shared copy is kept)
// The C-ABI version the code was built for: a payload module must carry it.
__device__ uint32_t tiler_cuda_payload_abi = TILER_CUDA_ABI_VERSION;
}

// 256/ln2 and ln2/256 split so that n*kLn2By256Hi is exact for |n| < 2^17.
constexpr double kInvLn2x256 = 369.3299304675746271;            // 256 / ln 2 (rounded)
constexpr double kLn2By256Hi = 0x1.62e42fefa0000p-9;             // 36 significant bits
constexpr double kLn2By256Mid = 0x1.cf79abc9e3b3ap-48;           // next 53 bits
constexpr double kLn2By256Lo = -0x1.ff0342542fc33p-102;           // remainder

__device__ __forceinline__ double pow2_double(int m) {  // 2^m for -1022 <= m <= 1023
  return __longlong_as_double((long long)(m + 1023) << 52);
}

__device__ __forceinline__ float next_up(float f) {  // f >= 0 finite
  return f == 0.0f ? __uint_as_float(1u) : __uint_as_float(__float_as_uint(f) + 1u);
}
__device__ __forceinline__ float next_down(float f) {  // f > 0
  return __uint_as_float(__float_as_uint(f) - 1u);
}

// Midpoint between the largest finite binary32 and 2^128: everything at or
// above it rounds to +inf (silu.rs:246-249).
constexpr double kOverflowMidpoint = 340282356779733661637539395458142568448.0;  // 2^128 - 2^103

// Distance test of a positive binary64 approximation y (relative error bound
// tol) against the midpoints around f = rn32(y).  Returns true when decided.
__device__ __forceinline__ bool decided(double y, float f, double tol) {
  double t = tol * y;
  if (isinf(f)) return y - t > kOverflowMidpoint;
  double fd = f;
  double upper = (__float_as_uint(f) == 0x7f7fffffu) ? kOverflowMidpoint : 0.5 * (fd + (double)next_up(f));
  if (y + t >= upper) return false;
  if (f == 0.0f) return true;  // nothing below zero is reachable
  double lower = 0.5 * (fd + (double)next_down(f));
  return y - t > lower;
}

// Double-double helpers (Dekker / Knuth error-free transformations).
struct dd { double hi, lo; };
__device__ __forceinline__ dd two_sum(double a, double b) {
  double s = __dadd_rn(a, b);
  double bb = __dsub_rn(s, a);
  double e = __dadd_rn(__dsub_rn(a, __dsub_rn(s, bb)), __dsub_rn(b, bb));
  return {s, e};
}
__device__ __forceinline__ dd two_prod(double a, double b) {
  double p = __dmul_rn(a, b);
  return {p, __fma_rn(a, b, -p)};
}
__device__ __forceinline__ dd dd_add(dd a, dd b) {
  dd s = two_sum(a.hi, b.hi);
  double e = __dadd_rn(s.lo, __dadd_rn(a.lo, b.lo));
  return two_sum(s.hi, e);
}
__device__ __forceinline__ dd dd_mul(dd a, dd b) {
  dd p = two_prod(a.hi, b.hi);
  double e = __fma_rn(a.hi, b.lo, __fma_rn(a.lo, b.hi, p.lo));
  return two_sum(p.hi, e);
}
__device__ __forceinline__ dd dd_mul_d(dd a, double b) {
  dd p = two_prod(a.hi, b);
  return two_sum(p.hi, __fma_rn(a.lo, b, p.lo));
}

// Rounds the double-double Y = y.hi + y.lo (> 0, relative error <= 2^-100)
// to binary32, deciding against the midpoints; flags when it cannot decide.
__device__ __noinline__ float round_dd_to_f32(dd y, bool* undecided) {
  float f = __double2float_rn(y.hi);
  const double tol = 0x1p-98 * y.hi;
  if (isinf(f)) {
    double d = __dadd_rn(__dsub_rn(y.hi, kOverflowMidpoint), y.lo);
    if (fabs(d) <= tol) *undecided = true;
    return d > 0 ? f : 3.40282347e38f;
  }
  double fd = f;
  if (__float_as_uint(f) != 0x7f7fffffu) {
    double upper = 0.5 * (fd + (double)next_up(f));
    double du = __dadd_rn(__dsub_rn(y.hi, upper), y.lo);
    if (fabs(du) <= tol) *undecided = true;
    if (du > 0) return next_up(f);
  }
  if (f != 0.0f) {
    double lower = 0.5 * (fd + (double)next_down(f));
    double dl = __dadd_rn(__dsub_rn(y.hi, lower), y.lo);
    if (fabs(dl) <= tol) *undecided = true;
    if (dl < 0) return next_down(f);
  }
  return f;
}

// Slow path: e^x in double-double.
__device__ __noinline__ float exp_slow(float x, int n, bool* undecided) {
  double nd = (double)n;
  // r = x - n ln2/256 as a double-double: x - n*Hi is exact (Sterbenz).
  double r0 = __fma_rn(-nd, kLn2By256Hi, (double)x);
  dd nm = two_prod(nd, kLn2By256Mid);
  dd r = two_sum(r0, -nm.hi);
  r.lo = __dsub_rn(__dsub_rn(r.lo, nm.lo), nd * kLn2By256Lo);
  r = two_sum(r.hi, r.lo);
  // e^r - 1 = sum_{i=1..10} r^i / i!, terms formed in double-double
  // (|r| <= 2^-9.4, so the first omitted term is below 2^-110).
  dd term = r, em1 = r;
  for (int i = 2; i <= 10; ++i) {
    term = dd_mul(term, r);
    double q = term.hi / (double)i;
    dd qi = two_prod(q, (double)i);
    double rem = __dadd_rn(__dsub_rn(term.hi, qi.hi), __dsub_rn(term.lo, qi.lo));
    term = two_sum(q, rem / (double)i);
    em1 = dd_add(em1, term);
  }
  int j = n & 255, m = n >> 8;
  dd t = {g_exp2_table[j][0], g_exp2_table[j][1]};
  dd y = dd_add(t, dd_mul(t, em1));
  // scale by 2^m in two exact steps (m >= -152, and y.hi*2^m stays normal)
  double s = pow2_double(m);
  y.hi *= s;
  y.lo *= s;
  return round_dd_to_f32(y, undecided);
}

// Correctly rounded binary32 e^x (certified_exp_strict, silu.rs:220-277).
// `table_hi` is a shared-memory (or global) copy of g_exp2_table[.][0].
__device__ __forceinline__ float exp_cr(float x, const double* table_hi, tiler_cuda_status* st) {
  if (isnan(x)) return __uint_as_float(kCanonicalNan);
  if (x >= 89.0f) return __uint_as_float(0x7f800000u);
  if (x <= -104.0f) return 0.0f;
  if (x == 0.0f) return 1.0f;
  double xd = (double)x;
  double nd = rint(xd * kInvLn2x256);
  int n = (int)nd;
  double r = __fma_rn(-nd, kLn2By256Hi, xd);  // exact
  r = __fma_rn(-nd, kLn2By256Mid, r);
  // e^r - 1 ~ r + r^2 (1/2 + r (1/6 + r/24)); |r| <= 2^-9.4, remainder < 2^-56
  double q = __fma_rn(r, 1.0 / 24.0, 1.0 / 6.0);
  q = __fma_rn(r, q, 0.5);
  double p = __fma_rn(__dmul_rn(r, r), q, r);
  int j = n & 255, m = n >> 8;
  double t = table_hi[j];
  double y = __fma_rn(t, p, t) * pow2_double(m);
  float f = __double2float_rn(y);
  if (decided(y, f, 0x1p-49)) return f;
  bool und = false;
  f = exp_slow(x, n, &und);
  if (und) report_undecided(st);
  return f;
}

// Fast form of exp_cr for a finite argument in (-104, 89): the same Tang
// evaluation, with n taken by adding 1.5*2^52 (round to nearest in the
// addition) and the midpoint test done on the bits of the binary64 value:
// its 29 bits below binary32 precision must differ from the midpoint pattern
// 1 << 28 by more than 64 units (2^-46 relative, against an evaluation error
// below 2^-51).  Results outside the normal binary32 range, and undecided
// ones, go to exp_cr.
constexpr double kRoundShift = 6755399441055744.0;  // 1.5 * 2^52
__device__ __forceinline__ float exp_cr_fast(float x, const double* table_hi, tiler_cuda_status* st) {
  const double xd = (double)x;
  const double t = __fma_rn(xd, kInvLn2x256, kRoundShift);
  const int n = __double2loint(t);
  const double nd = __dsub_rn(t, kRoundShift);
  double r = __fma_rn(-nd, kLn2By256Hi, xd);
  r = __fma_rn(-nd, kLn2By256Mid, r);
  double q = __fma_rn(r, 1.0 / 24.0, 1.0 / 6.0);
  q = __fma_rn(r, q, 0.5);
  const double p = __fma_rn(__dmul_rn(r, r), q, r);
  const double tj = table_hi[n & 255];
  const double y0 = __fma_rn(tj, p, tj);
  const int hi = __double2hiint(y0) + ((n >> 8) << 20);
  const int lo = __double2loint(y0);
  const int d = (int)((uint32_t)lo & 0x1fffffffu) - 0x10000000;
  const bool ok = hi >= 0x38100000 && hi < 0x47f00000 && (d > 64 || d < -64);
  if (ok) return __double2float_rn(__hiloint2double(hi, lo));
  return exp_cr(x, table_hi, st);
}

// exp_cr_fast without its fallback, for callers that batch the rare
// undecided arguments into one warp-uniform branch: returns the binary32
// bits of e^x for x in (-104, 89) and sets *ok when they are certified;
// otherwise the caller must take exp_cr(x).  A leaner evaluation than
// exp_cr_fast's, with the certification window widened to match:
//   n = rint(x * 256/ln2) (one FMA against 1.5 * 2^52), j = n mod 256,
//   r = x - n * L with L = RN(ln2/256), one FMA (|r| <= ln2/512 + tiny);
//     |n| < 2^15.3 and |L - ln2/256| <= 2^-62 put r within 2^-46.7 of
//     x - n ln2/256;
//   e^r - 1 ~ r + r^2 (1/2 + r/6), truncation below |r|^4/24 < 2^-42.7;
//   y = 2^(j/256) (1 + p), the table entry and the FMA rounding add 2^-52;
// so y is within 2^-42.6 (relative) of e^x, i.e. within 2^10.4 units of
// its own last bit.  It is certified when it is a normal binary32 value
// (hi in [0x38100000, 0x47f00000)) and its 29 bits below binary32 precision
// lie more than 2048 units from the midpoint pattern 1 << 28; then bit 28
// of the low word rounds it.  A value within the window (about one in 2^17)
// takes the caller's exact path.
#ifndef TILER_EXP_LEAN
#define TILER_EXP_LEAN 1
#endif
constexpr double kLn2By256 = 0x1.62e42fefa39efp-9;  // RN(ln2 / 256)
// kRangeChecked: the caller keeps x inside (-87, 88), where e^x is a normal
// binary32 value, so only the midpoint window decides ok.
template <bool kRangeChecked = false>
__device__ __forceinline__ uint32_t exp_cr_bits(float x, const double* table_hi, bool* ok) {
  const double xd = (double)x;
  const double t = __fma_rn(xd, kInvLn2x256, kRoundShift);
  const int n = __double2loint(t);
  const double nd = __dsub_rn(t, kRoundShift);
#if TILER_EXP_LEAN
  const double r = __fma_rn(-nd, kLn2By256, xd);
  const double q = __fma_rn(r, 1.0 / 6.0, 0.5);
  const double p = __fma_rn(__dmul_rn(r, r), q, r);
  constexpr uint32_t kWindow = 2048;
#else
  double r = __fma_rn(-nd, kLn2By256Hi, xd);
  r = __fma_rn(-nd, kLn2By256Mid, r);
  double q = __fma_rn(r, 1.0 / 24.0, 1.0 / 6.0);
  q = __fma_rn(r, q, 0.5);
  const double p = __fma_rn(__dmul_rn(r, r), q, r);
  constexpr uint32_t kWindow = 64;
#endif
  const double tj = table_hi[n & 255];
  const double y0 = __fma_rn(tj, p, tj);
  const uint32_t hi = (uint32_t)__double2hiint(y0) + ((uint32_t)(n >> 8) << 20);
  const uint32_t lo = (uint32_t)__double2loint(y0);
  const bool window_ok = ((lo & 0x1fffffffu) - (0x10000000u - kWindow)) > 2 * kWindow;
  *ok = kRangeChecked ? window_ok : (hi - 0x38100000u) < (0x47f00000u - 0x38100000u) && window_ok;
  // binary32 bits: exponent rebased, 23 mantissa bits from hi:lo, rounded by bit 28
  return __funnelshift_l(lo, hi - 0x38000000u, 3) + ((lo >> 28) & 1u);
}

// Correctly rounded binary32 1/sqrt(t) (certified_rsqrt_strict,
// rms_norm.rs:238-293).  The binary64 candidate is checked exactly: f is the
// correctly rounded value iff mlo^2 t < 1 < mhi^2 t for the midpoints mlo,
// mhi around f; m^2 is exact in binary64 (25-bit m) and m^2 t is formed
// exactly as a double-double.
__device__ __forceinline__ int cmp_sq_times_one(double m, float t) {
  double m2 = m * m;  // exact
  double ph = m2 * (double)t;
  double pl = __fma_rn(m2, (double)t, -ph);
  if (ph > 1.0) return 1;
  if (ph < 1.0) return -1;
  return pl > 0 ? 1 : (pl < 0 ? -1 : 0);
}

__device__ __forceinline__ float rsqrt_cr(float t) {
  if (isnan(t)) return __uint_as_float(kCanonicalNan);
  if (isinf(t)) return t > 0 ? 0.0f : __uint_as_float(kCanonicalNan);
  if (t == 0.0f) return signbit(t) ? __uint_as_float(0xff800000u) : __uint_as_float(0x7f800000u);
  if (t < 0.0f) return __uint_as_float(kCanonicalNan);
  // candidate: the hardware reciprocal square root (relative error below
  // 2^-21) refined by one Newton step in binary64, r1 = r0 + (r0/2)(1 - t r0^2),
  // which leaves it within 2^-40 of 1/sqrt(t); a subnormal t is first scaled
  // by 2^64 (exact) and the result by 2^32.  The exact midpoint test below
  // decides the rounding whatever the candidate's error.
  const bool tiny = t < 0x1p-126f;
  const float ts = tiny ? t * 0x1p64f : t;
  const double r0 = (double)rsqrtf(ts);
  const double e = __fma_rn(-__dmul_rn((double)ts, r0), r0, 1.0);
  const double r1 = __fma_rn(__dmul_rn(0.5, r0), e, r0);
  float f = __double2float_rn(tiny ? r1 * 0x1p32 : r1);
  for (int it = 0; it < 4; ++it) {
    double fd = f;
    double mhi = 0.5 * (fd + (double)next_up(f));
    if (cmp_sq_times_one(mhi, t) <= 0) { f = next_up(f); continue; }  // root >= mhi
    double mlo = 0.5 * (fd + (double)next_down(f));
    if (cmp_sq_times_one(mlo, t) >= 0) { f = next_down(f); continue; }  // root <= mlo
    break;
  }
  return f;
}

// x / d rounded to nearest for the SiLU denominator, by Markstein's method
// (P. Markstein, "Computation of elementary functions on the IBM RISC
// System/6000 processor", IBM J. Res. Dev. 34(1), 1990): a reciprocal y
// within half an ulp of 1/d, a quotient q0 = RN(x y) within an ulp of x / d,
// its exact remainder r = x - q0 d (one FMA), and q = RN(q0 + r y) is the
// correctly rounded quotient.  y comes from the hardware reciprocal estimate
// refined by one FMA Newton step, y = y0 + y0 (1 - d y0), the correctly
// rounded reciprocal except possibly when d's significand is all ones.  The
// caller keeps d in [1, 2^126) (a reciprocal above the subnormal range) and
// |x| at or above 2^-60 (a quotient clear of the subnormal range, no signed
// zero).  For the SiLU map, where d = 1 + RN(exp(-x)), the quotient equals
// the IEEE division on every binary32 argument in that range, the
// all-ones-significand d included: a GPU test checks all 2^32 arguments.
__device__ __forceinline__ float div_rn_markstein(float x, float d) {
  float y0;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(y0) : "f"(d));
  const float e = __fmaf_rn(-d, y0, 1.0f);
  const float y = __fmaf_rn(e, y0, y0);
  const float q0 = __fmul_rn(x, y);
  const float r = __fmaf_rn(-q0, d, x);
  return __fmaf_rn(r, y, q0);
}

// SiLU — silu_f32_under, crates/tiler-reference/src/silu.rs:158-180.
__device__ __forceinline__ float silu_cr(float x, const double* table_hi, tiler_cuda_status* st) {
  if (isnan(x)) return __uint_as_float(kCanonicalNan);
  if (isinf(x)) return x > 0 ? x : __uint_as_float(kCanonicalNan);
  float e = exp_cr(-x, table_hi, st);
  float d = __fadd_rn(1.0f, e);
  return canon(__fdiv_rn(x, d));
}

// SiLU with the fast certified exp: the same value as silu_cr.  For x in
// (-89, 104) the exponential exp(-x) is finite and above the underflow guard;
// outside that range silu_cr's guards apply.
__device__ __forceinline__ float silu_cr_fast(float x, const double* table_hi, tiler_cuda_status* st) {
  if (x > -89.0f && x < 104.0f) {
    const float e = exp_cr_fast(-x, table_hi, st);
    return __fdiv_rn(x, __fadd_rn(1.0f, e));
  }
  return silu_cr(x, table_hi, st);
}

// bf16(SiLU(x)) for the contraction epilogue: the bf16 rounding of the
// certified binary32 SiLU, without evaluating the certified value in the
// common case.  An approximation y' = x / (1 + exp(-x)) from the hardware
// exp2 / fast division has, for |x| < 80, relative error below (|x| + 11) *
// 2^-24 (argument scaling of exp2 |x| * 2^-24, ex2 2^-22, the add 2^-24,
// the division 2^-22), i.e. fewer than |x| + 11 binary32 ulps of y.  The bf16
// rounding of a binary32 value changes only where its low 16 bits cross
// 0x8000, so when y' sits more than 2|x| + 24 ulps from that point the
// certified y rounds to the same bf16 as y'.  Otherwise, and outside
// |x| < 80, the certified path decides.
__device__ __forceinline__ uint16_t silu_bf16_epilogue(float x, const double* table_hi, tiler_cuda_status* st) {
  const float ax = fabsf(x);
  if (ax < 80.0f) {
    const float e = __expf(-x);
    const float y = __fdividef(x, __fadd_rn(1.0f, e));
    const uint32_t b = __float_as_uint(y);
    const int dist = abs((int)(b & 0xffffu) - 0x8000);
    const bool normal = ((b >> 23) & 0xffu) != 0;
    if (normal && (float)dist > 2.0f * ax + 24.0f) return (uint16_t)((b + 0x7fffu + ((b >> 16) & 1u)) >> 16);
  }
  return f32_to_bf16(silu_cr_fast(x, table_hi, st));
}

// The same decision split in two for a warp draining 32 accumulators per
// lane: silu_bf16_fast returns the bf16 bits of the approximation and sets
// *certain when they are provably those of the certified value; the rare
// uncertain elements are then redone by silu_bf16_certified in one
// warp-uniform branch, so the common path has no per-element branch.
__device__ __forceinline__ uint32_t silu_bf16_fast(float x, bool* certain) {
  const float ax = fabsf(x);
  const float y = __fdividef(x, __fadd_rn(1.0f, __expf(-x)));
  const uint32_t b = __float_as_uint(y);
  // the low 16 bits as a float without an int->float conversion: 2^23 + v - 2^23
  const float low = __fsub_rn(__uint_as_float(0x4b000000u | (b & 0xffffu)), 8388608.0f);
  const float dist = fabsf(__fsub_rn(low, 32768.0f));
  *certain = ax < 80.0f && (b & 0x7f800000u) != 0 && dist > __fadd_rn(__fmul_rn(2.0f, ax), 24.0f);
  return (b + 0x7fffu + ((b >> 16) & 1u)) >> 16;
}
__device__ __noinline__ uint32_t silu_bf16_certified(float x, const double* table_hi, tiler_cuda_status* st) {
  return f32_to_bf16(silu_cr_fast(x, table_hi, st));
}

// Copies the 2^(j/256) hi column into shared memory (call by all threads,
// followed by __syncthreads()).
__device__ __forceinline__ void load_exp_table(double* smem_table) {
  for (int i = threadIdx.x; i < 256; i += blockDim.x) smem_table[i] = g_exp2_table[i][0];
}

// ---- PTX wrappers: mbarrier, bulk copies, TMA ---------------------------------

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return (uint32_t)__cvta_generic_to_shared(p);
}

__device__ __forceinline__ uint4 lds_u4(uint32_t saddr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(saddr));
  return v;
}

// Programmatic dependent launch (launch.cuh launches with it): a kernel may
// start while the previous kernel on the stream finishes; it waits here,
// before its first access to global memory, until that kernel has completed
// and its writes are visible, then lets the next kernel start launching.
// Without a programmatic dependency both are no-ops.
__device__ __forceinline__ void grid_dependency_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

__device__ __forceinline__ void sts_u4(uint32_t saddr, const uint4& v) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(saddr), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.shared::cta.b64 st, [%0];\n}" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n .reg .b64 st;\n mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n}" ::"r"(smem_u32(bar)),
               "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_test_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: polls the barrier phase and gives up after about two seconds
// of %globaltimer time, recording a timeout in the status word instead of
// hanging the device.
constexpr uint64_t kWaitLimitNs = 2000000000ull;
__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, tiler_cuda_status* st,
                                          uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 255) == 0 && global_ns() - t0 > limit_ns) break;
  }
  if (st) atomicAdd(&st->timeouts, 1u);
  return false;
}

// 1D bulk copy global -> shared, completing on an mbarrier (16-byte aligned
// addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_g2s(void* smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(smem_dst)),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// The same with the destination as a shared-window address.
__device__ __forceinline__ void bulk_g2s_u32(uint32_t smem_dst, const void* gmem_src, uint32_t bytes, uint64_t* bar,
                                             uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_dst),
      "l"(gmem_src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// 2D tiled TMA load (no multicast) completing on an mbarrier.
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* tmap, int32_t x, int32_t y, uint64_t* bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
      "%3}], [%4], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(tmap), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ float4 ld_global_policy(const float4* p, uint64_t policy) {
  float4 v;
  asm volatile("ld.global.L2::cache_hint.v4.f32 {%0,%1,%2,%3}, [%4], %5;"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "l"(p), "l"(policy));
  return v;
}
__device__ __forceinline__ void st_global_stream(float4* p, float4 v) {
  asm volatile("st.global.cs.v4.f32 [%0], {%1,%2,%3,%4};" ::"l"(p), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ uint4 ld_global_nc_u4(const uint4* p) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}
__device__ __forceinline__ void st_global_stream_u4(uint4* p, uint4 v) {
  asm volatile("st.global.cs.v4.u32 [%0], {%1,%2,%3,%4};" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z), "r"(v.w)
               : "memory");
}

}  // namespace tc
