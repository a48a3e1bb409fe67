// RMS normalization with every row resident in shared memory from its load
// to its normalize: x is read from HBM exactly once and never re-read.
//
// The reference fold (rms_norm.rs:147-170) is one strict chain of adds per
// row, so a row's sum of squares takes ~4 cycles per element however many
// lanes are free.  Keeping whole rows on chip for that long would need ~20
// rows per SM (320 KB for f32 rows of 4096); this kernel instead streams
// each row in as P column chunks and runs the rows of a block as a diagonal
// pipeline, so a row holds only the chunks it has loaded so far:
//
//   step b:  chain lane (k, r) folds chunk k of row r of group b - k
//            (a group = R consecutive rows), so P groups are in the fold at
//            once, each one chunk further along than the next; the running
//            sums move one lane group up (shfl_up by R) between steps, and
//            the lanes of chunk P-1 finish their rows' sums, form the scales
//            (mean = total / N, t = mean + eps, correctly rounded 1/sqrt(t),
//            rms_norm.rs:172-193) and hand the group to the normalize warps;
//   producer one warp: batch b = the bulk copies of the chunks step b reads,
//            issued up to c + 1 steps ahead on the batch's mbarrier;
//   normalize the warps form y = w * (x * s) (two roundings,
//            rms_norm.rs:479-485) from the staged chunks and write y with
//            streaming stores, then release the group's chunk slots.
//
// Chunk k of group t occupies slot t mod L_k of chunk k's slot ring, from
// its load (batch t + k) until group t is normalized (after step t + P - 1):
// L_k = P + c - k slots, so the rings hold sum_k (P + c - k) chunk buffers
// of R rows instead of 2 P full groups.  Before issuing batch b the
// producer waits until group b - P - c (the previous user of every slot that
// batch fills) is normalized.
//
// Shared-memory layout: buffer (k, slot, r) holds one row's chunk; lanes
// read their buffers at the same column offset at the same time, so each
// buffer starts 16 * (lane mod 8) bytes into a 128-byte-padded pitch and the
// eight lanes of a 16-byte load phase hit distinct banks.
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace tc {

template <int P_, int R_, int CB_, int C_, int PAD_ = 128>
struct RmsStreamCfg {
  static constexpr int P = P_;    // chunks per row (at most)
  static constexpr int R = R_;    // rows per group
  static constexpr int CB = CB_;  // chunk bytes (at most)
  static constexpr int C = C_;    // extra slot lifetime (steps of producer lead)
  // buffer pitch: a 128-byte pad lets each (chunk, row) ring start 16 * (lane
  // mod 8) bytes into it (conflict-free chain reads); a smaller pad spreads
  // the buffers over the banks by the pitch alone
  static constexpr bool kStagger = PAD_ >= 128;
  static constexpr int kPitch = (CB + 127) / 128 * 128 + PAD_;
  static constexpr int kBuffers = (P * (P + 1) / 2 + C * P) * R;
  // mbarrier rings (batches, groups): the producer issues the first P + C
  // batches before it waits for anything, so the batch ring must hold them all
  static constexpr int kRing = 16;
  static constexpr int kWarps = 12;
  static constexpr int kThreads = 32 * kWarps;
  static_assert(P * R <= 32, "one chain lane per (chunk, row)");
  static_assert(P <= 8 && CB <= 2048, "one normalize warp per chunk, at most four vectors per lane");
  static_assert(kRing >= P + C + 1, "barrier rings must cover the producer's lead");
};

// f32 rows of up to 16 KB: 8 chunks of 2 KB, groups of 2 rows (16 chain lanes).
using RmsStreamF32 = RmsStreamCfg<8, 2, 2048, 2>;
// bf16 rows of up to 8 KB: 8 chunks of 1 KB, groups of 4 rows (32 chain lanes;
// a bf16 row moves half the bytes of an f32 row for the same fold length),
// buffers 1072 bytes apart with no per-lane stagger so four rows fit (the
// chain does 8 adds per 16-byte load, so a 2-way bank conflict costs little):
// 40.6 us for [8192,4096] against 42.7 us with 3 rows and C = 3 and 44.2 us
// with 3 rows and C = 2.
using RmsStreamBF16 = RmsStreamCfg<8, 4, 1024, 2, 48>;

template <class Cfg>
struct RmsStreamSmem {
  uint64_t full[Cfg::kRing];       // batch b: its bulk copies landed
  uint64_t folded[Cfg::kRing];     // group t: its scales are known
  uint64_t normalized[Cfg::kRing]; // group t: its chunk slots are free
  float sum[Cfg::kRing][Cfg::R];  // group t's sums of squares
  // fused quantize: per row of group t, the largest |y| (magnitude bits) and
  // the first column whose y is NaN, combined over the normalize warps
  uint32_t ymax[Cfg::kRing][Cfg::R];
  uint32_t ynan[Cfg::kRing][Cfg::R];
  alignas(128) uint8_t buf[Cfg::kBuffers * Cfg::kPitch];
};
template <class Cfg>
constexpr size_t rms_stream_smem_bytes() {
  static_assert(sizeof(RmsStreamSmem<Cfg>) <= 227 * 1024, "one CTA's shared memory on sm_100a");
  return sizeof(RmsStreamSmem<Cfg>);
}

// Warp roles: warp 0 folds, alone on its scheduler (a warp's scheduler is its
// index mod 4, and warps 4 and 8 do nothing); warp 1 loads; warps 2, 3, 5, 6,
// 7, 9, 10, 11 normalize, normalize warp j owning chunk j of every row, so its
// slice of the weight row is loaded into registers once.
__device__ __forceinline__ int rms_stream_norm_index(int warp) {
  // warps 2, 3, 5, 6, 7, 9, 10, 11 -> 0 .. 7; else -1
  if (warp < 2 || (warp & 3) == 0) return -1;
  return warp - 2 - (warp >> 2);
}
constexpr int kRmsStreamNormWarps = 8;

// Folds the nvec 16-byte vectors at shared address p into acc in column
// order, with kAhead vectors of loads in flight ahead of the adds (a
// 16-entry register ring, indices fixed by unrolling), so the add chain
// does not wait on shared-memory latency.
#ifndef TILER_RMS_FOLD_FORM
#define TILER_RMS_FOLD_FORM 1
#endif
template <class E>
__device__ __forceinline__ float rms_fold_chunk(float acc, uint32_t p, uint32_t nvec) {
  constexpr uint32_t kRing = 16, kAhead = 12;
  constexpr int V = E::kPerVec;
  uint4 q[kRing];
#if TILER_RMS_FOLD_FORM == 0
  auto fold = [&](const uint4& v) {
    float e[V];
    E::unpack(v, e);
#pragma unroll
    for (int j = 0; j < V; j += 2) {
      float s0, s1;
      square2(e[j], e[j + 1], s0, s1);
      acc = __fadd_rn(acc, s0);
      acc = __fadd_rn(acc, s1);
    }
  };
#pragma unroll
  for (uint32_t u = 0; u < kAhead; ++u)
    if (u < nvec) q[u] = lds_u4_nv(p + u * 16);
  uint32_t v0 = 0;
  for (; v0 + kRing + kAhead <= nvec; v0 += kRing) {
#pragma unroll
    for (uint32_t u = 0; u < kRing; ++u) {
      q[(u + kAhead) % kRing] = lds_u4_nv(p + (v0 + u + kAhead) * 16);
      fold(q[u]);
    }
  }
  for (; v0 < nvec; v0 += kRing) {
#pragma unroll
    for (uint32_t u = 0; u < kRing; ++u) {
      if (v0 + u + kAhead < nvec) q[(u + kAhead) % kRing] = lds_u4_nv(p + (v0 + u + kAhead) * 16);
      if (v0 + u < nvec) fold(q[u]);
    }
  }
#else
  // the squares of vector v + 1 are formed before the adds of vector v, so
  // the adds run back to back on the chain
  float sq[2][V];
  auto square = [&](const uint4& v, float (&o)[V]) {
    float e[V];
    E::unpack(v, e);
#pragma unroll
    for (int j = 0; j < V; j += 2) square2(e[j], e[j + 1], o[j], o[j + 1]);
  };
  auto add = [&](const float (&o)[V]) {
#pragma unroll
    for (int j = 0; j < V; ++j) acc = __fadd_rn(acc, o[j]);
  };
#pragma unroll
  for (uint32_t u = 0; u < kAhead; ++u)
    if (u < nvec) q[u] = lds_u4_nv(p + u * 16);
  square(q[0], sq[0]);
  uint32_t v0 = 0;
  for (; v0 + kRing + kAhead <= nvec; v0 += kRing) {
#pragma unroll
    for (uint32_t u = 0; u < kRing; ++u) {
      q[(u + kAhead) % kRing] = lds_u4_nv(p + (v0 + u + kAhead) * 16);
      square(q[(u + 1) % kRing], sq[(u + 1) & 1]);
      add(sq[u & 1]);
    }
  }
  for (; v0 < nvec; v0 += kRing) {
#pragma unroll
    for (uint32_t u = 0; u < kRing; ++u) {
      if (v0 + u + kAhead < nvec) q[(u + kAhead) % kRing] = lds_u4_nv(p + (v0 + u + kAhead) * 16);
      if (v0 + u + 1 < nvec) square(q[(u + 1) % kRing], sq[(u + 1) & 1]);
      if (v0 + u < nvec) add(sq[u & 1]);
    }
  }
#endif
  return acc;
}

// A chunk shorter than the configured chunk (the last chunk of a row that is
// not a multiple of it), out of line: the full chunks call the fold with
// their length as a compile-time constant, which the compiler schedules
// better (f32 RMS [8192,4096] 59.2 -> 57.6 us, bf16 50.3 -> 44.0 us).
template <class E>
__device__ __noinline__ float rms_fold_chunk_partial(float acc, uint32_t p, uint32_t nvec) {
  return rms_fold_chunk<E>(acc, p, nvec);
}

// QUANT: the fused RMS norm -> per-row int8 quantize (f32 only): the
// normalize warps keep y in registers, combine each row's max |y| across
// the chunk owners (shared-memory atomics and one named barrier per group)
// and write the codes and scales; y never leaves the SM.
template <class E, class Cfg, bool QUANT = false>
__device__ __forceinline__ void rms_norm_stream(const uint8_t* __restrict__ x, const uint8_t* __restrict__ w,
                                                uint64_t rows, uint64_t extent, float eps, uint8_t* __restrict__ y,
                                                tiler_cuda_status* st, int8_t* __restrict__ codes = nullptr,
                                                float* __restrict__ scales = nullptr) {
  constexpr int P = Cfg::P, R = Cfg::R, C = Cfg::C, RING = Cfg::kRing, PITCH = Cfg::kPitch;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  RmsStreamSmem<Cfg>& S = *reinterpret_cast<RmsStreamSmem<Cfg>*>(smem_raw);
  const int warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  const uint64_t esize = sizeof(typename E::T);
  const uint64_t row_bytes = extent * esize;
  // chunk bytes: the row split into at most P chunks of 16-byte multiples
  const uint32_t cb = (uint32_t)(((row_bytes + P - 1) / P + 15) / 16 * 16);
  const int nch = (int)((row_bytes + cb - 1) / cb);
  const uint64_t rb = blockIdx.x * rows / gridDim.x, re = (blockIdx.x + 1) * rows / gridDim.x;
  const int my_rows = (int)(re - rb);  // the launcher bounds rows per CTA below 2^30
  const int G = (my_rows + R - 1) / R;  // groups
  const int nsteps = G + nch - 1;
  auto group_rows = [&](int t) { return min(R, my_rows - t * R); };
  auto chunk_bytes = [&](int k) { return (uint32_t)umin64(cb, row_bytes - (uint64_t)k * cb); };
  // buffer (k, slot, r): ring k has L_k = nch + C - k slots of R rows; the
  // buffer of row r of chunk k sits 16 * ((k R + r) mod 8) bytes into its pitch
  auto ring_base = [&](int k, int r) -> uint32_t {
    const int base = k * (nch + C) - k * (k - 1) / 2;  // sum_{j<k} L_j
    return smem_u32(S.buf) + (uint32_t)((base * R + r) * PITCH + (Cfg::kStagger ? 16 * ((k * R + r) & 7) : 0));
  };

  if (threadIdx.x == 0) {
    for (int i = 0; i < RING; ++i) {
      mbar_init(&S.full[i], 1);
      mbar_init(&S.folded[i], 1);
      mbar_init(&S.normalized[i], kRmsStreamNormWarps);
    }
    fence_barrier_init();
  }
  __syncthreads();
  if (G == 0) return;

  // chain and producer lanes: lane (k, r) = chunk k of row r, for group b - k
  // at step b, in slot (b - k) mod L_k of ring k (advanced by one per step)
  const int k = lane / R, r = lane % R;
  const bool lane_on = lane < P * R && k < nch;
  const int lk = nch + C - k;
  int slot = lane_on ? (lk - k % lk) % lk : 0;
  const uint32_t lane_ring = lane_on ? ring_base(k, r) : 0;
  const uint32_t lane_bytes = lane_on ? chunk_bytes(k) : 0;

  if (warp == 1) {
    // ---- producer ------------------------------------------------------------
    const uint64_t pol = policy_evict_first();  // x is read once
    for (int b = 0; b < nsteps; ++b) {
      const int prev = b - nch - C;  // the group whose slots batch b reuses
      if (prev >= 0 && !mbar_wait(&S.normalized[prev % RING], (uint32_t)((prev / RING) & 1), st)) break;
      const int t = b - k;
      const bool valid = lane_on && t >= 0 && t < G && r < group_rows(t);
      const uint32_t bytes = valid ? lane_bytes : 0;
      const uint32_t total = __reduce_add_sync(0xffffffffu, bytes);
      if (lane == 0) mbar_arrive_expect_tx(&S.full[b % RING], total);
      __syncwarp();
      if (valid) {
        const uint64_t row = rb + (uint64_t)t * R + r;
        bulk_g2s_u32(lane_ring + (uint32_t)(slot * R * PITCH), x + row * row_bytes + (uint64_t)k * cb, bytes,
                     &S.full[b % RING], pol);
      }
      slot = slot + 1 == lk ? 0 : slot + 1;
    }
  } else if (warp == 0) {
    // ---- chain ---------------------------------------------------------------
    float acc = 0.0f;
    for (int b = 0; b < nsteps; ++b) {
      const float prev_acc = __shfl_up_sync(0xffffffffu, acc, R);
      if (!mbar_wait(&S.full[b % RING], (uint32_t)((b / RING) & 1), st)) {
        // a wait that gave up: the producer runs at most nch + C batches
        // ahead, so let the copies of those land (each wait bounded at 1 ms)
        // before this CTA's shared memory is released
        for (int b2 = b; b2 < min(nsteps, b + nch + C); ++b2)
          mbar_wait(&S.full[b2 % RING], (uint32_t)((b2 / RING) & 1), nullptr, 1000000ull);
        break;
      }
      const int t = b - k;
      const bool valid = lane_on && t >= 0 && t < G && r < group_rows(t);
      // the fold starts from +0 at chunk 0: +0 + a_0 is a_0 exactly (squares
      // are never -0), the reference's seed at the first square
      if (valid) {
        const float a0 = k == 0 ? 0.0f : prev_acc;
        const uint32_t p = lane_ring + (uint32_t)(slot * R * PITCH);
        acc = lane_bytes == (uint32_t)Cfg::CB ? rms_fold_chunk<E>(a0, p, Cfg::CB / 16)
                                              : rms_fold_chunk_partial<E>(a0, p, lane_bytes / 16);
      }
      // the group that finished its last chunk this step: its sums go to the
      // normalize warps, which form the scales off the chain's path
      const int tf = b - (nch - 1);
      if (tf >= 0 && tf < G) {
        if (valid && k == nch - 1) {
          S.sum[tf % RING][r] = acc;
          if constexpr (QUANT) {
            S.ymax[tf % RING][r] = 0;
            S.ynan[tf % RING][r] = 0xffffffffu;
          }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.folded[tf % RING]);
      }
      slot = slot + 1 == lk ? 0 : slot + 1;
    }
  } else {
    const int nw = rms_stream_norm_index(warp);
    if (nw < 0) return;
    // ---- normalize -----------------------------------------------------------
    constexpr int U = 4;  // 16-byte vectors per lane: a chunk is at most 2 KB
    const int kk = nw;     // this warp's chunk
    const uint32_t nvec = kk < nch ? chunk_bytes(kk) / 16 : 0;
    const uint64_t off = (uint64_t)kk * cb;
    uint4 wq[U];
#pragma unroll
    for (int u = 0; u < U; ++u)
      if (lane + 32 * u < nvec) wq[u] = __ldg(reinterpret_cast<const uint4*>(w + off) + lane + 32 * u);
    const int lkk = nch + C - kk;
    for (int t = 0; t < G; ++t) {
      if (!mbar_wait(&S.folded[t % RING], (uint32_t)((t / RING) & 1), st)) break;
      const int gr = group_rows(t);
      const uint32_t slot_off = (uint32_t)((t % lkk) * R * PITCH);
      // rms_norm.rs:172-193: mean = total / N, t = mean + eps, certified rsqrt;
      // lane r forms row r's scale
      const float s_lane =
          lane < gr ? rsqrt_cr(__fadd_rn(__fdiv_rn(S.sum[t % RING][lane], (float)extent), eps)) : 0.0f;
      if constexpr (QUANT) {
        // quantize_i8_rows of each row's y (quantization.rs:188-247, :404-430
        // with the per-row scale max|y| / 127): y stays in registers between
        // the maximum and the codes; the group's rows are handled together
        // (unrolled) so their dependent steps overlap
        float yr[R][U][E::kPerVec];
        uint32_t mb[R], first[R];
#pragma unroll
        for (int rr = 0; rr < R; ++rr) {
          mb[rr] = 0;
          first[rr] = 0xffffffffu;
          if (kk < nch && rr < gr) {
            const float s = __shfl_sync(0xffffffffu, s_lane, rr);
            const uint32_t p = ring_base(kk, rr) + slot_off;
#pragma unroll
            for (int u = 0; u < U; ++u)
              if (lane + 32 * u < nvec) {
                float xe[E::kPerVec], we[E::kPerVec];
                E::unpack(lds_u4_nv(p + (lane + 32 * u) * 16), xe);
                E::unpack(wq[u], we);
#pragma unroll
                for (int j = 0; j < E::kPerVec; ++j) {
                  // a NaN y (any payload) has magnitude bits above +inf's
                  const float yv = __fmul_rn(we[j], __fmul_rn(xe[j], s));
                  yr[rr][u][j] = yv;
                  mb[rr] = max(mb[rr], __float_as_uint(yv) & 0x7fffffffu);
                }
              }
          }
        }
#pragma unroll
        for (int rr = 0; rr < R; ++rr) {
          const uint32_t m = __reduce_max_sync(0xffffffffu, mb[rr]);
          if (m > 0x7f800000u) {  // the chunk holds a NaN y: its first column
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
              for (int j = 0; j < E::kPerVec; ++j)
                if (lane + 32 * u < nvec && (__float_as_uint(yr[rr][u][j]) & 0x7fffffffu) > 0x7f800000u)
                  first[rr] = min(first[rr], (uint32_t)(off / sizeof(float)) + (lane + 32 * u) * E::kPerVec + j);
          }
          const uint32_t f = __reduce_min_sync(0xffffffffu, first[rr]);
          if (lane == 0 && kk < nch && rr < gr) {
            atomicMax(&S.ymax[t % RING][rr], m);
            if (f != 0xffffffffu) atomicMin(&S.ynan[t % RING][rr], f);
          }
        }
        // y is in registers: the group's chunk slots can be refilled while the
        // codes are formed
        __syncwarp();
        if (lane == 0) mbar_arrive(&S.normalized[t % RING]);
        // every normalize warp has combined its chunk of every row
        asm volatile("bar.sync 1, %0;" ::"r"(32 * kRmsStreamNormWarps) : "memory");
        // lane r forms row r's quantize scale max|y| / 127 and its reciprocal
        const uint32_t mb_lane = lane < gr ? S.ymax[t % RING][lane] : 0u;
        float scale_lane = 0.0f, inv_lane = 0.0f;
        if (lane < gr) {
          scale_lane = __fdiv_rn(__uint_as_float(mb_lane), 127.0f);
          if (is_positive_normal(scale_lane)) inv_lane = __frcp_rn(scale_lane);
        }
        if (nw == 0 && lane < gr) {
          const uint64_t row = rb + (uint64_t)t * R + lane;
          if (mb_lane > 0x7f800000u) {  // a NaN y: report its first column
            report_error(st, row * extent + S.ynan[t % RING][lane], TILER_CUDA_NAN_INPUT);
          } else {
            scales[row] = scale_lane;
            if (!is_positive_normal(scale_lane)) report_error(st, row * extent, TILER_CUDA_SCALE_DOMAIN);
          }
        }
        // code = rint(y / scale) clamped to [-127, 127]: y * (1/scale) decides
        // it unless the product lies within 3e-5 of a half-integer, where the
        // exact quotient is taken (one warp-uniform branch).  |q| <= 127, so
        // RN(q + 1.5 * 2^23) is 1.5 * 2^23 + rint(q) (ties to even), whose
        // low bits are the integer
        constexpr float kMagic = 12582912.0f;  // 1.5 * 2^23
        float scale[R], inv[R];
        bool live[R];
        float tv[R][U][4];
        bool near_half = false;
#pragma unroll
        for (int rr = 0; rr < R; ++rr) {
          const uint32_t m = __shfl_sync(0xffffffffu, mb_lane, rr);
          scale[rr] = __shfl_sync(0xffffffffu, scale_lane, rr);
          inv[rr] = __shfl_sync(0xffffffffu, inv_lane, rr);
          live[rr] = kk < nch && rr < gr && m <= 0x7f800000u && is_positive_normal(scale[rr]);
#pragma unroll
          for (int u = 0; u < U; ++u)
#pragma unroll
            for (int j = 0; j < 4; ++j) {
              const float q = __fmul_rn(yr[rr][u][j], inv[rr]);
              const float t1 = __fadd_rn(q, kMagic);
              near_half |= live[rr] && lane + 32 * u < nvec && fabsf(__fsub_rn(q, __fsub_rn(t1, kMagic))) > 0.49997f;
              tv[rr][u][j] = t1;
            }
        }
        if (__any_sync(0xffffffffu, near_half)) {
#pragma unroll
          for (int rr = 0; rr < R; ++rr)
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const float q = __fmul_rn(yr[rr][u][j], inv[rr]);
                if (live[rr] && fabsf(__fsub_rn(q, __fsub_rn(tv[rr][u][j], kMagic))) > 0.49997f)
                  tv[rr][u][j] = __fadd_rn(__fdiv_rn(yr[rr][u][j], scale[rr]), kMagic);
              }
        }
#pragma unroll
        for (int rr = 0; rr < R; ++rr) {
          if (!live[rr]) continue;
          int* crow = reinterpret_cast<int*>(codes + (rb + (uint64_t)t * R + rr) * extent + off / sizeof(float));
#pragma unroll
          for (int u = 0; u < U; ++u)
            if (lane + 32 * u < nvec) {
              int c[4];
#pragma unroll
              for (int j = 0; j < 4; ++j) c[j] = max(-127, min(127, (int)__float_as_uint(tv[rr][u][j]) - 0x4B400000));
              uint32_t hi, packed;  // cvt.pack d, a, b, c: d = c << 16 | sat8(a) << 8 | sat8(b)
              asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, 0;" : "=r"(hi) : "r"(c[3]), "r"(c[2]));
              asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(packed) : "r"(c[1]), "r"(c[0]), "r"(hi));
              __stcs(crow + lane + 32 * u, (int)packed);
            }
        }
        continue;  // the slots were released above
      } else {
        for (int rr = 0; kk < nch && rr < gr; ++rr) {
            const float s = __shfl_sync(0xffffffffu, s_lane, rr);
          const uint32_t p = ring_base(kk, rr) + slot_off;
          uint4* yk = reinterpret_cast<uint4*>(y + (rb + (uint64_t)t * R + rr) * row_bytes + off);
          uint4 xq[U];
  #pragma unroll
          for (int u = 0; u < U; ++u)
            if (lane + 32 * u < nvec) xq[u] = lds_u4_nv(p + (lane + 32 * u) * 16);
  #pragma unroll
          for (int u = 0; u < U; ++u)
            if (lane + 32 * u < nvec) {
              float xe[E::kPerVec], we[E::kPerVec], ye[E::kPerVec];
              E::unpack(xq[u], xe);
              E::unpack(wq[u], we);
  #pragma unroll
              for (int j = 0; j < E::kPerVec; ++j) {
                const float yv = __fmul_rn(we[j], __fmul_rn(xe[j], s));
                ye[j] = E::kPackCanonicalizes ? yv : canon(yv);
              }
              st_global_stream_u4(yk + lane + 32 * u, E::pack(ye));
            }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.normalized[t % RING]);
    }
  }
}

}  // namespace tc

#define TILER_RMS_STREAM_PARAMS                                                                             \
  const uint8_t *__restrict__ x, const uint8_t *__restrict__ w, uint64_t rows, uint64_t extent, float eps, \
      uint8_t *__restrict__ y, tiler_cuda_status *st
extern "C" __global__ void __launch_bounds__(tc::RmsStreamF32::kThreads, 1)
    tiler_rms_norm_stream_f32(TILER_RMS_STREAM_PARAMS) {
  tc::grid_dependency_wait();
  tc::rms_norm_stream<tc::RmsElem<false>, tc::RmsStreamF32>(x, w, rows, extent, eps, y, st);
}
extern "C" __global__ void __launch_bounds__(tc::RmsStreamBF16::kThreads, 1)
    tiler_rms_norm_stream_bf16(TILER_RMS_STREAM_PARAMS) {
  tc::grid_dependency_wait();
  tc::rms_norm_stream<tc::RmsElem<true>, tc::RmsStreamBF16>(x, w, rows, extent, eps, y, st);
}
extern "C" __global__ void __launch_bounds__(tc::RmsStreamF32::kThreads, 1)
    tiler_rms_norm_stream_quantize_i8(const uint8_t* __restrict__ x, const uint8_t* __restrict__ w, uint64_t rows,
                                      uint64_t extent, float eps, int8_t* __restrict__ codes,
                                      float* __restrict__ scales, tiler_cuda_status* st) {
  tc::grid_dependency_wait();
  tc::rms_norm_stream<tc::RmsElem<false>, tc::RmsStreamF32, true>(x, w, rows, extent, eps, nullptr, st, codes,
                                                                 scales);
}
#undef TILER_RMS_STREAM_PARAMS

namespace tc {

// The streamed form applies to 16-byte-aligned rows with a broadcast weight
// row that fit its chunk rings; it returns false where it does not.
bool rms_stream_launch(int bf16, const void* x, const void* w, int64_t w_row_stride, uint64_t rows, uint64_t extent,
                       float eps, void* y, tiler_cuda_status* st, int sm_count, cudaStream_t stream) {
  const uint64_t esize = bf16 ? 2 : 4;
  const uint64_t row_bytes = extent * esize;
  const uint64_t max_row = bf16 ? (uint64_t)RmsStreamBF16::P * RmsStreamBF16::CB
                                : (uint64_t)RmsStreamF32::P * RmsStreamF32::CB;
  if (w_row_stride != 0 || row_bytes % 16 || row_bytes > max_row) return false;
  const uint64_t grid = umin64((uint64_t)sm_count, rows);
  if (rows / grid >= (1ull << 30)) return false;
  const void* fn = bf16 ? (const void*)tiler_rms_norm_stream_bf16 : (const void*)tiler_rms_norm_stream_f32;
  const size_t smem = bf16 ? rms_stream_smem_bytes<RmsStreamBF16>() : rms_stream_smem_bytes<RmsStreamF32>();
  cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  launch_kernel(fn, bf16 ? "tiler_rms_norm_stream_bf16" : "tiler_rms_norm_stream_f32", dim3((unsigned)grid),
                dim3(RmsStreamF32::kThreads), smem, stream, (const uint8_t*)x, (const uint8_t*)w, rows, extent, eps,
                (uint8_t*)y, st);
  return true;
}

// The fused RMS -> int8 quantize in the streamed form (f32 rows of up to
// 16 KB, a broadcast weight row); false where it does not apply.
bool rms_stream_quant_launch(const float* x, const float* w, int64_t w_row_stride, uint64_t rows, uint64_t extent,
                             float eps, int8_t* codes, float* scales, tiler_cuda_status* st, int sm_count,
                             cudaStream_t stream) {
  const uint64_t row_bytes = extent * 4;
  if (w_row_stride != 0 || row_bytes % 16 || row_bytes > (uint64_t)RmsStreamF32::P * RmsStreamF32::CB) return false;
  const uint64_t grid = umin64((uint64_t)sm_count, rows);
  if (rows / grid >= (1ull << 30)) return false;
  const size_t smem = rms_stream_smem_bytes<RmsStreamF32>();
  cudaFuncSetAttribute(tiler_rms_norm_stream_quantize_i8, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  launch_kernel((const void*)tiler_rms_norm_stream_quantize_i8, "tiler_rms_norm_stream_quantize_i8",
                dim3((unsigned)grid), dim3(RmsStreamF32::kThreads), smem, stream, (const uint8_t*)x,
                (const uint8_t*)w, rows, extent, eps, codes, scales, st);
  return true;
}

}  // namespace tc
