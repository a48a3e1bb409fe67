// Warp-cooperative strict left fold of NON-NEGATIVE binary32 terms.
//
// The reference folds the squares of an RMS row (rms_norm.rs:147-170) and the
// exponentials of a softmax row (softmax.rs:295-300) strictly left to right,
// every add rounded once (RNE): s_{i+1} = RN(s_i + a_i), seeded at a_0.  The
// chain is serial by definition, but for terms a_i >= +0 it has structure
// that lets a warp evaluate it exactly, 256 terms per step:
//
//  * s never decreases, so it stays inside one binade [2^e, 2^(e+1)) for long
//    runs.  Inside a binade every binary32 is an integer multiple of
//    u = 2^(e-23): s = S*u with S an integer in [2^23, 2^24).
//  * While the exact sum S*u + a stays below 2^(e+1), RN(S*u + a) is the
//    multiple of u nearest to it: (S + q)*u with q = a/u rounded to the
//    nearest integer.  When a/u = n + 1/2 exactly (a tie) the even one of
//    S + n and S + n + 1 is taken: S + n + ((S + n) & 1).
//  * So inside a binade the fold is an integer recurrence.  Without ties it is
//    a plain sum (S_{i+1} = S_i + q_i; integer addition is associative, so a
//    warp reduction computes it exactly).  A tie adds n plus one parity bit,
//    and the parity of a sum is the XOR of its terms' parities; after a tie the
//    running value is even.  So each tie's bit is the XOR of the low bits of
//    the terms since the previous tie (or since the running value S), which
//    two warp ballots give every lane.
//
// The binade ends where S + (the terms so far) reaches 2^24 (a CROSSING: the
// sum leaves the binade, or rounds up to its end).  A crossing, and a
// non-finite term (its q is clamped to 2^23, which always crosses), is
// resolved by one real binary32 add of the running value and the term, in
// order; the binade (e, u, S) is then re-read from the new running value and
// the chunk resumes at the next term.  Below 2^-103 (where 2^(23-e) is not a
// normal binary32) terms are folded one at a time instead.  A running value
// of +inf stays +inf unless a later term is NaN; NaN absorbs the rest.  The
// result is the bits of the reference's strict fold, NaN canonicalized.
//
// Layout: the caller hands the terms over in chunks of 256 (terms 8*l .. 8*l+7
// of a chunk in lane l, in order), masked terms as +0 (adding +0 to a
// non-negative running value is the identity, and a fold seeded at a_0 >= +0
// equals the same fold started from +0).
#pragma once

#include "common.cuh"

namespace tc {

struct NonnegFold {
  uint32_t S;  // fast mode: the running value in units of u (an integer in [2^23, 2^24))
  float p;     // 2^(23-e)
  float u;     // 2^(e-23)
  float s;     // other modes: the running value itself
  int mode;    // kFoldFast, kFoldSmall, kFoldInf, kFoldNan
  int serial;  // small mode leaves no earlier than this many terms into the chunk
};
constexpr int kFoldFast = 0, kFoldSmall = 1, kFoldInf = 2, kFoldNan = 3;
constexpr uint32_t kFoldTwo24 = 1u << 24;
// 2^-103: the smallest running value whose binade has a normal 2^(23-e)
constexpr float kFoldFastMin = 9.8607613e-32f;

// A fold starts in small mode at +0.  The first `serial_terms` terms of the
// first chunk are folded one at a time whatever their size: a fold crosses a
// binade boundary every time its running value doubles, so crossings are
// dense among the first terms (about log2 of the term count in all), and one
// at a time is cheaper there than a scan per crossing.
__device__ __forceinline__ NonnegFold fold_start(int serial_terms = 0) {
  return NonnegFold{0u, 0.f, 0.f, 0.f, kFoldSmall, serial_terms};
}

// Enter fast mode at a finite running value s >= 2^-103 (a normal binary32).
__device__ __forceinline__ void fold_enter_fast(NonnegFold& F, float s) {
  const uint32_t b = __float_as_uint(s);
  const uint32_t be = b >> 23;  // biased exponent, >= 24
  F.S = (b & 0x7fffffu) | 0x800000u;
  F.p = __uint_as_float((277u - be) << 23);  // 2^(150 - be) = 2^(23 - e)
  F.u = __uint_as_float((be - 23u) << 23);   // 2^(e - 23)
  F.mode = kFoldFast;
}

__device__ __forceinline__ float fold_value(const NonnegFold& F) {
  if (F.mode == kFoldFast) return __fmul_rn((float)F.S, F.u);
  if (F.mode == kFoldNan) return __uint_as_float(kCanonicalNan);
  return F.s;  // small (possibly +0 or subnormal) or +inf
}

// Warp-uniform: does any lane hold a NaN among its 8 terms?
__device__ __forceinline__ bool fold_any_nan(const float (&a)[8]) {
  bool n = false;
#pragma unroll
  for (int k = 0; k < 8; ++k) n |= isnan(a[k]);
  return __any_sync(0xffffffffu, n);
}

// Zero the terms at chunk positions <= j (position = 8 * lane + k).
__device__ __forceinline__ void fold_consume(float (&a)[8], uint32_t lane, int j) {
#pragma unroll
  for (int k = 0; k < 8; ++k)
    if ((int)(8 * lane + k) <= j) a[k] = 0.0f;
}

// Continue after a real add produced s at chunk position j.
__device__ __forceinline__ void fold_after_add(NonnegFold& F, float s, float (&a)[8], uint32_t lane, int j) {
  if (isnan(s)) { F.mode = kFoldNan; return; }
  fold_consume(a, lane, j);
  if (isinf(s)) {
    F.s = s;
    F.mode = fold_any_nan(a) ? kFoldNan : kFoldInf;
    return;
  }
  if (s < kFoldFastMin) { F.s = s; F.mode = kFoldSmall; return; }
  fold_enter_fast(F, s);
}

// Two binary32 operations at once on the f32x2 ALU; each half is the IEEE RN
// result of its own operands.
__device__ __forceinline__ void fold_mul2(float a0, float a1, float b0, float b1, float& r0, float& r1) {
  uint64_t x, y, r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(y) : "f"(b0), "f"(b1));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(x), "l"(y));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r0), "=f"(r1) : "l"(r));
}
__device__ __forceinline__ void fold_add2(float a0, float a1, float b0, float b1, float& r0, float& r1) {
  uint64_t x, y, r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(y) : "f"(b0), "f"(b1));
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(x), "l"(y));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r0), "=f"(r1) : "l"(r));
}
// a * b + c with one rounding per half (used only where the result is exact)
__device__ __forceinline__ void fold_fma2(float a0, float a1, float b0, float b1, float c0, float c1, float& r0,
                                          float& r1) {
  uint64_t x, y, z, r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(y) : "f"(b0), "f"(b1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(z) : "f"(c0), "f"(c1));
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(x), "l"(y), "l"(z));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r0), "=f"(r1) : "l"(r));
}

__device__ __forceinline__ uint32_t warp_sum_u32(uint32_t v) {
  uint32_t r;
  asm volatile("redux.sync.add.u32 %0, %1, 0xffffffff;" : "=r"(r) : "r"(v));
  return r;
}

// Folds one chunk of 256 terms (a: this lane's 8 terms, in order; modified).
// All 32 lanes must call it with the same F.
__device__ __forceinline__ void fold_chunk(NonnegFold& F, float (&a)[8], uint32_t lane) {
  for (;;) {
    if (F.mode == kFoldNan) return;
    if (F.mode == kFoldInf) {
      if (fold_any_nan(a)) F.mode = kFoldNan;
      return;
    }
    if (F.mode == kFoldSmall) {
      // one term at a time, until the running value reaches 2^-103 (and at
      // least the first F.serial terms)
      // (lane l's 8 terms are fetched at once and added in order; the running
      // value is kept at the term where small mode ends)
      float s = F.s;
      int j = -1;
      for (int l = 0; l < 32 && j < 0; ++l) {
        float t[8];
#pragma unroll
        for (int k = 0; k < 8; ++k) t[k] = __shfl_sync(0xffffffffu, a[k], l);
        float r = s;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
          r = __fadd_rn(r, t[k]);
          if (j < 0 && !(r < kFoldFastMin) && 8 * l + k + 1 >= F.serial) {  // also taken for NaN
            j = 8 * l + k;
            s = r;
          }
        }
        if (j < 0) s = r;
      }
      F.serial = 0;
      if (j < 0) { F.s = s; return; }  // the whole chunk stayed small
      fold_after_add(F, s, a, lane, j);
      continue;
    }
    // ---- fast mode ----------------------------------------------------------
    // t = a * 2^(23-e) exactly; q = rint(t); a tie where |t - q| = 1/2, whose
    // integer part n = floor(t) is kept in v.  t is clamped to 2^23 first:
    // S >= 2^23, so any term that large crosses, and NaN / inf terms clamp to
    // it too (min returns the non-NaN operand).  rint is one add: t + 2^23
    // lies in [2^23, 2^24], where the binary32 spacing is 1, so the add rounds
    // t to the nearest integer, ties to even (2^23 is even), and that integer
    // is the sum's bit pattern minus 2^23's (conversion instructions, which
    // issue at a quarter of the rate, are avoided).
    // Pairs of terms go through the f32x2 ALU (mul / add / fma .rn.f32x2,
    // each half one IEEE RN operation).  The sum of q is taken from the bit
    // patterns; the per-term values and tie bits are formed only where a tie
    // or a crossing needs them.
    float t[8], m[8], d[8];
    uint32_t bsum = 0;
    bool any_tie = false;
#pragma unroll
    for (int k = 0; k < 8; k += 2) {
      fold_mul2(a[k], a[k + 1], F.p, F.p, t[k], t[k + 1]);
      t[k] = fminf(t[k], 8388608.0f);
      t[k + 1] = fminf(t[k + 1], 8388608.0f);
      fold_add2(t[k], t[k + 1], 8388608.0f, 8388608.0f, m[k], m[k + 1]);
      float r0, r1;
      fold_add2(m[k], m[k + 1], -8388608.0f, -8388608.0f, r0, r1);
      fold_fma2(r0, r1, -1.0f, -1.0f, t[k], t[k + 1], d[k], d[k + 1]);  // t - r, exact
      any_tie |= fabsf(d[k]) == 0.5f;
      any_tie |= fabsf(d[k + 1]) == 0.5f;
      bsum += __float_as_uint(m[k]) + __float_as_uint(m[k + 1]);
    }
    uint32_t vsum = bsum - 8u * 0x4b000000u;
    uint32_t v[8];
    uint32_t ties = 0;  // bit k: term k is a tie
    auto exact_terms = [&]() {
      vsum = 0;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const bool tie = fabsf(d[k]) == 0.5f;
        v[k] = (__float_as_uint(m[k]) - 0x4b000000u) - (uint32_t)(tie && d[k] < 0.0f);
        ties |= (uint32_t)tie << k;
        vsum += v[k];
      }
    };
    const uint32_t tie_lanes = __ballot_sync(0xffffffffu, any_tie);
    uint32_t delta = 0;  // this lane's tie bits (0 without ties)
    uint32_t cin = 0;    // parity of the running value at this lane's first term
    if (tie_lanes) {
      exact_terms();
      // lane-local parity walk: `par` = parity of the terms since the lane's
      // start or its last tie; x0 = that parity through the first tie
      uint32_t par = 0, x0 = 0, later = 0;
      bool seen = false;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t pk = v[k] & 1u;
        if ((ties >> k) & 1u) {
          if (seen) later += par ^ pk; else x0 = par ^ pk;
          seen = true;
          par = 0;  // after a tie the running value is even
        } else {
          par ^= pk;
        }
      }
      // parity of the running value at each lane's end: `par` for a lane with
      // a tie, its carry-in XOR `par` otherwise; the carry-in of lane l is the
      // end parity of the last tie lane before it, XOR the parities of the
      // tie-free lanes in between (or S's parity XOR all lanes before l)
      const uint32_t outb = __ballot_sync(0xffffffffu, par != 0);
      const uint32_t lt = (1u << lane) - 1u;
      const uint32_t below = tie_lanes & lt;
      if (below) {
        const uint32_t lp = 31 - __clz(below);
        const uint32_t between = lt & ~((2u << lp) - 1u);
        cin = ((outb >> lp) & 1u) ^ (__popc(outb & between) & 1u);
      } else {
        cin = (F.S & 1u) ^ (__popc(outb & lt) & 1u);
      }
      delta = ties ? (cin ^ x0) + later : 0u;
    }
    const uint32_t inc = warp_sum_u32(vsum + delta);
    if (inc < kFoldTwo24 - F.S) {  // no crossing: the whole chunk stays in the binade
      F.S += inc;
      return;
    }
    // ---- a crossing: find its term (the running value is monotone) --------------
    if (!tie_lanes) exact_terms();
    uint32_t c[8];  // each term's increment of S
    {
      uint32_t par = cin;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        const uint32_t pk = v[k] & 1u;
        if ((ties >> k) & 1u) {
          c[k] = v[k] + (par ^ pk);
          par = 0;
        } else {
          c[k] = v[k];
          par ^= pk;
        }
      }
    }
    const uint32_t total = vsum + delta;
    uint32_t P = total;  // inclusive scan over lanes (saturating at 2^30, far past any crossing)
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const uint32_t o = __shfl_up_sync(0xffffffffu, P, d);
      if (lane >= (uint32_t)d) P = min(P + o, 0x40000000u);
    }
    const uint32_t E = P - min(total, P);  // exclusive prefix (exact below the saturation)
    const uint32_t L = __ffs(__ballot_sync(0xffffffffu, P >= kFoldTwo24 - F.S)) - 1;
    int kk = 7;
    uint32_t before = 0;
    float term = 0.0f;
    {
      uint32_t run = F.S + E;
      bool found = false;
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        if (!found && c[k] >= kFoldTwo24 - run) {
          found = true;
          kk = k;
          before = run;
          term = a[k];
        }
        if (!found) run += c[k];
      }
    }
    kk = __shfl_sync(0xffffffffu, kk, L);
    before = __shfl_sync(0xffffffffu, before, L);
    term = __shfl_sync(0xffffffffu, term, L);
    const float s = __fadd_rn(__fmul_rn((float)before, F.u), term);  // the reference's own add
    fold_after_add(F, s, a, lane, (int)(8 * L) + kk);
  }
}

}  // namespace tc
