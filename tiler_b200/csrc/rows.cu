// Row families: RMS normalization (f32 / bf16), max-shifted softmax with the
// causal block mask, and the per-row int8 strict-affine quantize / decode.
//
// Each row family's reference fold is a strict left fold along the row
// (rms_norm.rs:147-170 sum of squares, softmax.rs:295-300 denominator), a
// dependent chain of adds that no reassociation may shorten.  The kernels
// therefore give every row its own lane for the chain and keep the other
// warps busy moving bytes: the chain reads staged copies from shared memory
// while HBM traffic stays one read (plus an L2-resident re-read for RMS) and
// one write per element.
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "tmap.cuh"

namespace tc {

// ---------------------------------------------------------------------------
// RMS normalization
// ---------------------------------------------------------------------------
//
// Per CTA (one per SM): a contiguous block of rows, split into waves of up to
// kRmsWave rows.  The CTA runs kRmsPipes independent pipelines; pipeline p
// takes waves p, p + kRmsPipes, ... and pipeline p > 0 starts when pipeline
// p-1 has folded half of its first wave, so the pipelines' load, fold and
// store phases interleave instead of hitting HBM and L2 all at once.
//
// One pipeline = 1 producer warp + 1 chain warp + kRmsNormWarps warps:
//   producer   streams the wave's rows through a ring of shared-memory stages:
//              per stage, lane r issues one bulk copy (cp.async.bulk) of row
//              r's 2 KB column slab, completing on the stage's mbarrier; rows
//              are padded by 16 bytes so the chain lanes' 16-byte reads down
//              a column are bank-conflict-free.  (Bulk copies cost a roughly
//              fixed time each, so slabs are 2 KB rather than 1 KB: 1 KB
//              slabs halve the load rate; cp.async 16-byte copies, the
//              alternative, put 64 threads' worth of issue next to the chain.)
//   chain      lane r folds row r's squares strictly in column order
//              (rms_norm.rs:147-170), the shared-memory loads of the next 8
//              vectors issued before the adds of the current 8;
//   normalize  once the wave's scales are known (mean = total/N, t = mean +
//              eps, correctly rounded 1/sqrt(t)), re-read the wave's rows (an
//              L2 hit, evict_first) and write y = w*(x*s) with streaming
//              stores, while the producer and the chain move on.  A broadcast
//              weight row is staged in shared memory once per CTA.

// pipeline p > 0 starts once pipeline p - 1 has folded NUM/DEN of its first wave
#ifndef TILER_RMS_STAGGER_NUM
#define TILER_RMS_STAGGER_NUM 1
#endif
#ifndef TILER_RMS_STAGGER_DEN
#define TILER_RMS_STAGGER_DEN 2
#endif
#ifndef TILER_RMS_WAVE
#define TILER_RMS_WAVE 28
#endif
#ifndef TILER_RMS_STAGES
#define TILER_RMS_STAGES 3
#endif
#ifndef TILER_RMS_PIPES
#define TILER_RMS_PIPES 1
#endif
#ifndef TILER_RMS_NORM_WARPS
#define TILER_RMS_NORM_WARPS 14
#endif
#ifndef TILER_RMS_SLAB
#define TILER_RMS_SLAB 2048
#endif
constexpr int kRmsSlabBytes = TILER_RMS_SLAB;
constexpr int kRmsPitch = kRmsSlabBytes + 16;
constexpr int kRmsWave = TILER_RMS_WAVE;  // rows per wave (one chain lane per row), <= 32
constexpr int kRmsStages = TILER_RMS_STAGES;
constexpr int kRmsPipes = TILER_RMS_PIPES;
constexpr int kRmsLoadWarps = 1;
constexpr int kRmsNormWarps = TILER_RMS_NORM_WARPS;
constexpr int kRmsPipeWarps = kRmsLoadWarps + 1 + kRmsNormWarps;
// x is loaded with evict_last so it stays in L2 until the normalize pass
// re-reads it (with evict_first).
#ifndef TILER_RMS_KEEP_X
#define TILER_RMS_KEEP_X 1
#endif
constexpr int kRmsThreads = 32 * kRmsPipeWarps * kRmsPipes;

struct RmsPipeSmem {
  alignas(128) uint8_t stage[kRmsStages][kRmsWave * kRmsPitch];
  uint64_t full[kRmsStages];
  uint64_t empty[kRmsStages];
  uint64_t scale_full[2];
  uint64_t scale_empty[2];
  uint64_t started;  // arrived once this pipeline has folded half of its first wave
  float scale[2][kRmsWave];
};
// The broadcast weight row is staged once per CTA when it fits.
#ifndef TILER_RMS_W_STAGE
#define TILER_RMS_W_STAGE 1
#endif
constexpr int kRmsWeightBytes = TILER_RMS_W_STAGE ? 16384 : 16;
#ifndef TILER_RMS_NORM_U
#define TILER_RMS_NORM_U 8
#endif
struct RmsSmem {
  RmsPipeSmem pipe[kRmsPipes];
  alignas(16) uint8_t wrow[kRmsWeightBytes];
  int abort;
};
constexpr size_t kRmsSmemBytes = sizeof(RmsSmem);

// Shared-memory 16-byte load.  Volatile so the compiler cannot speculate it
// above the lane predicate that keeps its address inside the allocation.
__device__ __forceinline__ uint4 lds_u4_nv(uint32_t saddr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(saddr));
  return v;
}

template <bool BF16>
struct RmsElem;
template <>
struct RmsElem<false> {
  using T = float;
  static constexpr int kPerVec = 4;
  __device__ static void unpack(const uint4& v, float* o) {
    o[0] = __uint_as_float(v.x); o[1] = __uint_as_float(v.y); o[2] = __uint_as_float(v.z); o[3] = __uint_as_float(v.w);
  }
  __device__ static uint4 pack(const float* o) {
    return make_uint4(__float_as_uint(o[0]), __float_as_uint(o[1]), __float_as_uint(o[2]), __float_as_uint(o[3]));
  }
  static constexpr bool kPackCanonicalizes = false;
};
template <>
struct RmsElem<true> {
  using T = uint16_t;
  static constexpr int kPerVec = 8;
  __device__ static void unpack(const uint4& v, float* o) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      o[2 * i] = __uint_as_float(w[i] << 16);
      o[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  }
  // RNE to bf16 two at a time (cvt.rn.bf16x2.f32: a to the upper half, b to
  // the lower), then NaN halves set to the canonical 0x7fc0
  __device__ static uint4 pack(const float* o) {
    uint32_t w[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      uint32_t p;
      asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(p) : "f"(o[2 * i + 1]), "f"(o[2 * i]));
      const uint32_t nan_halves = __vcmpgtu2(p & 0x7fff7fffu, 0x7f807f80u);
      w[i] = (p & ~nan_halves) | (0x7fc07fc0u & nan_halves);
    }
    return make_uint4(w[0], w[1], w[2], w[3]);
  }
  static constexpr bool kPackCanonicalizes = true;
};

__device__ __forceinline__ uint4 ld_u4_policy(const void* p, uint64_t policy) {
  uint4 v;
  asm volatile("ld.global.L2::cache_hint.v4.u32 {%0,%1,%2,%3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(policy));
  return v;
}

// 32-byte global load (with an L2 policy) and streaming store, sm_100.
__device__ __forceinline__ void ld_v8_policy(const void* p, uint64_t policy, uint4& a, uint4& b) {
  asm volatile("ld.global.L2::cache_hint.v8.u32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8], %9;"
               : "=r"(a.x), "=r"(a.y), "=r"(a.z), "=r"(a.w), "=r"(b.x), "=r"(b.y), "=r"(b.z), "=r"(b.w)
               : "l"(p), "l"(policy));
}
__device__ __forceinline__ void st_v8_stream(void* p, const uint4& a, const uint4& b) {
  asm volatile("st.global.cs.v8.u32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"l"(p), "r"(a.x), "r"(a.y), "r"(a.z),
               "r"(a.w), "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
               : "memory");
}

// Folds `n` 16-byte vectors of one staged row into acc (strict order).
// Software-pipelined: the shared-memory loads of batch k + 1 are issued
// before the adds of batch k, so the dependent add chain never waits on a
// load's latency (the warp issues in order).
// Two binary32 squares with one mul.rn.f32x2 (each lane an IEEE RN product,
// the same bits as two mul.rn.f32).
__device__ __forceinline__ void square2(float a, float b, float& ra, float& rb) {
  uint64_t in, out;
  asm("mov.b64 %0, {%1, %2};" : "=l"(in) : "f"(a), "f"(b));
  asm("mul.rn.f32x2 %0, %1, %1;" : "=l"(out) : "l"(in));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(ra), "=f"(rb) : "l"(out));
}

template <class E>
__device__ __forceinline__ void rms_fold_batch(float& acc, const uint4 (&q)[8]) {
#pragma unroll
  for (uint32_t b = 0; b < 8; ++b) {
    float e[E::kPerVec];
    E::unpack(q[b], e);
#pragma unroll
    for (int j = 0; j < E::kPerVec; j += 2) {
      float s0, s1;
      square2(e[j], e[j + 1], s0, s1);
      acc = __fadd_rn(acc, s0);
      acc = __fadd_rn(acc, s1);
    }
  }
}
template <class E>
__device__ __forceinline__ float rms_fold_vectors(float acc, uint32_t rowp, uint32_t v, uint32_t n) {
  constexpr uint32_t B = 8;
  if (v + B <= n) {
    uint4 q[B], qn[B];
#pragma unroll
    for (uint32_t b = 0; b < B; ++b) q[b] = lds_u4_nv(rowp + (v + b) * 16);
    v += B;
    for (; v + B <= n; v += B) {
#pragma unroll
      for (uint32_t b = 0; b < B; ++b) qn[b] = lds_u4_nv(rowp + (v + b) * 16);
      rms_fold_batch<E>(acc, q);
#pragma unroll
      for (uint32_t b = 0; b < B; ++b) q[b] = qn[b];
    }
    rms_fold_batch<E>(acc, q);
  }
  for (; v < n; ++v) {
    float e[E::kPerVec];
    E::unpack(lds_u4_nv(rowp + v * 16), e);
#pragma unroll
    for (int j = 0; j < E::kPerVec; ++j) acc = __fadd_rn(acc, __fmul_rn(e[j], e[j]));
  }
  return acc;
}

__device__ __forceinline__ int code_of_bounded(float xv, float scale, float inv);

// QUANT: the fused RMS norm -> per-row int8 quantize (f32 only): instead of
// writing y, each normalize warp forms its row's y twice from the L2-resident
// x (max|y| first, then the codes), so y never reaches HBM.
template <bool BF16, bool QUANT = false>
__device__ __forceinline__ void rms_norm_wave(const uint8_t* __restrict__ x, const uint8_t* __restrict__ w,
                                              int64_t w_row_stride, uint64_t rows, uint64_t extent, float eps,
                                              uint8_t* __restrict__ y, uint32_t wave_rows, tiler_cuda_status* st,
                                              int8_t* __restrict__ codes, float* __restrict__ scales) {
  using E = RmsElem<BF16>;
  extern __shared__ __align__(128) uint8_t smem_raw[];
  RmsSmem& SS = *reinterpret_cast<RmsSmem*>(smem_raw);
  const uint32_t pipe = threadIdx.x / (32 * kRmsPipeWarps);
  const uint32_t pwarp = (threadIdx.x / 32) % kRmsPipeWarps, lane = threadIdx.x & 31;
  RmsPipeSmem& S = SS.pipe[pipe];
  const uint64_t esize = sizeof(typename E::T);
  const uint64_t row_bytes = extent * esize;
  const uint64_t rb = blockIdx.x * rows / gridDim.x, re = (blockIdx.x + 1) * rows / gridDim.x;
  const uint64_t my_rows = re - rb;
  const uint32_t WR = wave_rows;
  const uint64_t nwaves_all = (my_rows + WR - 1) / WR;
  // this pipeline's waves: pipe, pipe + kRmsPipes, ...
  const uint64_t nwaves = nwaves_all > pipe ? (nwaves_all - pipe + kRmsPipes - 1) / kRmsPipes : 0;
  const uint64_t nslabs = (row_bytes + kRmsSlabBytes - 1) / kRmsSlabBytes;
  const uint64_t total = nwaves * nslabs;
  auto wave_first_row = [&](uint64_t wv) { return (pipe + wv * kRmsPipes) * (uint64_t)WR; };
  auto wave_rows_of = [&](uint64_t wv) { return (uint32_t)umin64(WR, my_rows - wave_first_row(wv)); };

  if (threadIdx.x == 0) {
    for (int p = 0; p < kRmsPipes; ++p) {
      RmsPipeSmem& Q = SS.pipe[p];
      for (int s = 0; s < kRmsStages; ++s) { mbar_init(&Q.full[s], kRmsLoadWarps); mbar_init(&Q.empty[s], 1); }
      for (int s = 0; s < 2; ++s) { mbar_init(&Q.scale_full[s], 1); mbar_init(&Q.scale_empty[s], kRmsNormWarps); }
      mbar_init(&Q.started, 1);
    }
    SS.abort = 0;
    fence_barrier_init();
  }
  const bool w_staged = w_row_stride == 0 && row_bytes <= (uint64_t)kRmsWeightBytes;
  if (w_staged)
    for (uint32_t i = threadIdx.x; i < row_bytes / 16; i += blockDim.x)
      reinterpret_cast<uint4*>(SS.wrow)[i] = __ldg(reinterpret_cast<const uint4*>(w) + i);
  __syncthreads();
  volatile int* abort_flag = &SS.abort;
  if (nwaves == 0) return;

  if (pwarp < kRmsLoadWarps) {
    // ---- producers -----------------------------------------------------------
    // x stays in L2 until the normalize pass re-reads it (with evict_first)
    const uint64_t keep = TILER_RMS_KEEP_X ? policy_evict_last() : policy_evict_normal();
    if (pipe > 0 && !mbar_wait(&SS.pipe[pipe - 1].started, 0, st))
      *abort_flag = 1;
    // one warp: per stage, lane r issues one bulk copy of row r's slab
    // (padded pitch), completing on the stage's mbarrier
    if (pwarp == 0) {
      for (uint64_t i = 0; i < total && !*abort_flag; ++i) {
        const uint32_t stage = i % kRmsStages;
        const uint64_t use = i / kRmsStages;
        if (use > 0 && !mbar_wait(&S.empty[stage], (uint32_t)((use - 1) & 1), st)) { *abort_flag = 1; break; }
        const uint64_t wv = i / nslabs, c = i % nslabs;
        const uint32_t wr = wave_rows_of(wv);
        const uint32_t bytes = (uint32_t)umin64(kRmsSlabBytes, row_bytes - c * kRmsSlabBytes);
        const uint8_t* gbase = x + (rb + wave_first_row(wv)) * row_bytes + c * kRmsSlabBytes;
        if (lane == 0) mbar_arrive_expect_tx(&S.full[stage], bytes * wr);
        __syncwarp();
        if (lane < wr) bulk_g2s(&S.stage[stage][lane * kRmsPitch], gbase + lane * row_bytes, bytes, &S.full[stage], keep);
      }
    }
  } else if (pwarp == kRmsLoadWarps) {
    // ---- chain warp ------------------------------------------------------------
    bool signalled = false;
    for (uint64_t wv = 0; wv < nwaves; ++wv) {
      const uint32_t wr = wave_rows_of(wv);
      float acc = 0.0f;
      for (uint64_t c = 0; c < nslabs; ++c) {
        const uint64_t i = wv * nslabs + c;
        const uint32_t stage = i % kRmsStages;
        if (!mbar_wait(&S.full[stage], (uint32_t)((i / kRmsStages) & 1), st)) *abort_flag = 1;
        if (*abort_flag) break;
        const uint32_t nvec = (uint32_t)umin64(kRmsSlabBytes, row_bytes - c * kRmsSlabBytes) / 16;
        if (lane < wr) {
          const uint32_t rowp = smem_u32(&S.stage[stage][lane * kRmsPitch]);
          uint32_t v = 0;
          if (c == 0) {  // the fold is seeded at the first square
            float e[E::kPerVec];
            E::unpack(lds_u4_nv(rowp), e);
            acc = __fmul_rn(e[0], e[0]);
#pragma unroll
            for (int j = 1; j < E::kPerVec; ++j) acc = __fadd_rn(acc, __fmul_rn(e[j], e[j]));
            v = 1;
          }
          acc = rms_fold_vectors<E>(acc, rowp, v, nvec);
        }
        __syncwarp();
        if (lane == 0) {
          mbar_arrive(&S.empty[stage]);
          if (!signalled && (c + 1) * TILER_RMS_STAGGER_DEN >= nslabs * TILER_RMS_STAGGER_NUM) { mbar_arrive(&S.started); signalled = true; }
        }
      }
      if (*abort_flag) break;
      // rms_norm.rs:172-193: mean = total / N, t = mean + eps, certified rsqrt
      const float mean = __fdiv_rn(acc, (float)extent);
      const float s = rsqrt_cr(__fadd_rn(mean, eps));
      const uint32_t slot = wv & 1;
      const uint64_t use = wv >> 1;
      if (use > 0 && !mbar_wait(&S.scale_empty[slot], (uint32_t)((use - 1) & 1), st)) { *abort_flag = 1; break; }
      if (lane < wr) S.scale[slot][lane] = s;
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.scale_full[slot]);
    }
  } else {
    // ---- normalize warps: y = w * (x * s), two roundings (rms_norm.rs:479-485)
    const uint32_t nw = pwarp - kRmsLoadWarps - 1;
    const uint64_t drop = policy_evict_first();
    const bool wide = (uintptr_t)x % 32 == 0 && (uintptr_t)y % 32 == 0 && row_bytes % 32 == 0;
    const uint64_t nvec = row_bytes / 16;
    for (uint64_t wv = 0; wv < nwaves; ++wv) {
      const uint32_t wr = wave_rows_of(wv);
      const uint32_t slot = wv & 1;
      if (!mbar_wait(&S.scale_full[slot], (uint32_t)((wv >> 1) & 1), st)) *abort_flag = 1;
      if (*abort_flag) break;
      for (uint32_t r = nw; r < wr; r += kRmsNormWarps) {
        const float s = S.scale[slot][r];
        const uint64_t row = rb + wave_first_row(wv) + r;
        const uint8_t* xr = x + row * row_bytes;
        const uint8_t* wrow = w + (int64_t)row * w_row_stride * (int64_t)esize;
        uint8_t* yr = y + row * row_bytes;
        auto norm_vec = [&](const uint4& xq, uint64_t v) {  // y for the 16-byte vector v of the row
          const uint4 wq = w_staged ? reinterpret_cast<const uint4*>(SS.wrow)[v]
                                    : __ldg(reinterpret_cast<const uint4*>(wrow + v * 16));
          float xe[E::kPerVec], we[E::kPerVec], ye[E::kPerVec];
          E::unpack(xq, xe);
          E::unpack(wq, we);
#pragma unroll
          for (int j = 0; j < E::kPerVec; ++j) {
            // bf16 output: the packing maps every NaN to the canonical one
            const float yv = __fmul_rn(we[j], __fmul_rn(xe[j], s));
            ye[j] = E::kPackCanonicalizes ? yv : canon(yv);
          }
          return E::pack(ye);
        };
        if constexpr (QUANT) {
          // quantize_i8_rows of this row's y (quantization.rs:188-247, :404-430 with the
          // per-row scale max|y| / 127): max over the magnitude bits, then the codes
          constexpr int UQ = TILER_RMS_NORM_U;
          uint32_t mb = 0;
          for (uint64_t v0 = lane; v0 < nvec; v0 += 32 * UQ) {
            uint4 xv[UQ];
#pragma unroll
            for (int u = 0; u < UQ; ++u)
              if (v0 + 32 * u < nvec) xv[u] = ld_u4_policy(xr + (v0 + 32 * u) * 16, drop);
#pragma unroll
            for (int u = 0; u < UQ; ++u)
              if (v0 + 32 * u < nvec) {
                const uint4 q = norm_vec(xv[u], v0 + 32 * u);
                mb = max(mb, max(max(q.x & 0x7fffffffu, q.y & 0x7fffffffu), max(q.z & 0x7fffffffu, q.w & 0x7fffffffu)));
              }
          }
          mb = __reduce_max_sync(0xffffffffu, mb);
          if (mb > 0x7f800000u) {  // a NaN y: report its first column
            uint32_t first = 0xffffffffu;
            for (uint64_t v = lane; v < nvec; v += 32) {
              const uint4 q = norm_vec(ld_u4_policy(xr + v * 16, drop), v);
              const uint32_t b[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
              for (int j = 0; j < 4; ++j)
                if ((b[j] & 0x7fffffffu) > 0x7f800000u) first = min(first, (uint32_t)(v * 4 + j));
            }
            first = __reduce_min_sync(0xffffffffu, first);
            if (lane == 0) report_error(st, row * extent + first, TILER_CUDA_NAN_INPUT);
            continue;
          }
          const float scale = __fdiv_rn(__uint_as_float(mb), 127.0f);
          if (lane == 0) scales[row] = scale;
          if (!is_positive_normal(scale)) {
            if (lane == 0) report_error(st, row * extent, TILER_CUDA_SCALE_DOMAIN);
            continue;
          }
          const float inv = __frcp_rn(scale);
          int* crow = reinterpret_cast<int*>(codes + row * extent);
          for (uint64_t v0 = lane; v0 < nvec; v0 += 32 * UQ) {
            uint4 xv[UQ];
#pragma unroll
            for (int u = 0; u < UQ; ++u)
              if (v0 + 32 * u < nvec) xv[u] = ld_u4_policy(xr + (v0 + 32 * u) * 16, drop);
#pragma unroll
            for (int u = 0; u < UQ; ++u)
              if (v0 + 32 * u < nvec) {
                const uint4 q = norm_vec(xv[u], v0 + 32 * u);
                const int c0 = code_of_bounded(__uint_as_float(q.x), scale, inv);
                const int c1 = code_of_bounded(__uint_as_float(q.y), scale, inv);
                const int c2 = code_of_bounded(__uint_as_float(q.z), scale, inv);
                const int c3 = code_of_bounded(__uint_as_float(q.w), scale, inv);
                uint32_t hi, packed;  // cvt.pack d, a, b, c: d = c << 16 | sat8(a) << 8 | sat8(b)
                asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, 0;" : "=r"(hi) : "r"(c3), "r"(c2));
                asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(packed) : "r"(c1), "r"(c0), "r"(hi));
                __stcs(crow + v0 + 32 * u, (int)packed);
              }
          }
          continue;
        }
        if (wide) {
          // 32-byte loads and stores (half the memory instructions)
          constexpr int U2 = TILER_RMS_NORM_U / 2;
          const uint64_t npair = nvec / 2;
          for (uint64_t p0 = lane; p0 < npair; p0 += 32 * U2) {
            uint4 xa[U2], xb[U2];
#pragma unroll
            for (int u = 0; u < U2; ++u) {
              const uint64_t pp = p0 + 32 * u;
              if (pp < npair) ld_v8_policy(xr + pp * 32, drop, xa[u], xb[u]);
            }
#pragma unroll
            for (int u = 0; u < U2; ++u) {
              const uint64_t pp = p0 + 32 * u;
              if (pp < npair) st_v8_stream(yr + pp * 32, norm_vec(xa[u], 2 * pp), norm_vec(xb[u], 2 * pp + 1));
            }
          }
          continue;
        }
        constexpr int U = TILER_RMS_NORM_U;  // 16-byte loads of x in flight per lane
        for (uint64_t v0 = lane; v0 < nvec; v0 += 32 * U) {
          uint4 xv[U];
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const uint64_t v = v0 + 32 * u;
            if (v < nvec) xv[u] = ld_u4_policy(xr + v * 16, drop);
          }
#pragma unroll
          for (int u = 0; u < U; ++u) {
            const uint64_t v = v0 + 32 * u;
            if (v < nvec) st_global_stream_u4(reinterpret_cast<uint4*>(yr + v * 16), norm_vec(xv[u], v));
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&S.scale_empty[slot]);
    }
  }
}

}  // namespace tc

#define TILER_RMS_WAVE_PARAMS                                                                                  \
  const uint8_t *__restrict__ x, const uint8_t *__restrict__ w, int64_t w_row_stride, uint64_t rows,          \
      uint64_t extent, float eps, uint8_t *__restrict__ y, uint32_t wave_rows, tiler_cuda_status *st,          \
      int8_t *__restrict__ codes, float *__restrict__ scales
extern "C" __global__ void __launch_bounds__(tc::kRmsThreads, 1) tiler_rms_norm_wave_f32(TILER_RMS_WAVE_PARAMS) {
  tc::grid_dependency_wait();
  tc::rms_norm_wave<false, false>(x, w, w_row_stride, rows, extent, eps, y, wave_rows, st, codes, scales);
}
extern "C" __global__ void __launch_bounds__(tc::kRmsThreads, 1) tiler_rms_norm_wave_bf16(TILER_RMS_WAVE_PARAMS) {
  tc::grid_dependency_wait();
  tc::rms_norm_wave<true, false>(x, w, w_row_stride, rows, extent, eps, y, wave_rows, st, codes, scales);
}
extern "C" __global__ void __launch_bounds__(tc::kRmsThreads, 1)
    tiler_rms_norm_wave_quantize_i8(TILER_RMS_WAVE_PARAMS) {
  tc::grid_dependency_wait();
  tc::rms_norm_wave<false, true>(x, w, w_row_stride, rows, extent, eps, y, wave_rows, st, codes, scales);
}
#undef TILER_RMS_WAVE_PARAMS

namespace tc {

// Any-shape path (unaligned rows or extents not a multiple of 16 bytes): one
// warp per row, lane 0 folds the squares straight from global memory.
template <bool BF16>
__global__ void rms_norm_generic_kernel(const void* __restrict__ xv, const void* __restrict__ wv,
                                        int64_t w_row_stride, uint64_t rows, uint64_t extent, float eps,
                                        void* __restrict__ yv) {
  using T = typename RmsElem<BF16>::T;
  const T* x = (const T*)xv;
  const T* w = (const T*)wv;
  T* y = (T*)yv;
  const uint64_t row = blockIdx.x * (uint64_t)(blockDim.x / 32) + threadIdx.x / 32;
  const uint32_t lane = threadIdx.x & 31;
  if (row >= rows) return;
  auto ld = [](const T* p, uint64_t i) -> float {
    if constexpr (BF16) return bf16_to_f32(p[i]); else return p[i];
  };
  float s = 0.0f;
  if (lane == 0) {
    float acc = 0.0f;
    for (uint64_t i = 0; i < extent; ++i) {
      const float v = ld(x + row * extent, i);
      const float sq = __fmul_rn(v, v);
      acc = i == 0 ? sq : __fadd_rn(acc, sq);
    }
    s = rsqrt_cr(__fadd_rn(__fdiv_rn(acc, (float)extent), eps));
  }
  s = __shfl_sync(0xffffffffu, s, 0);
  for (uint64_t i = lane; i < extent; i += 32) {
    const float v = canon(__fmul_rn(ld(w + (int64_t)row * w_row_stride, i), __fmul_rn(ld(x + row * extent, i), s)));
    if constexpr (BF16) y[row * extent + i] = f32_to_bf16(v); else y[row * extent + i] = v;
  }
}

// TILER_RMS_FORM in the environment (read once per process) selects the RMS
// kernel where it applies: "scan" the warp-per-row kernel (rms_scan.cu),
// "stream" the chunk-streamed kernel (rms_stream.cu), "wave" the wave kernel.
// All are exact.  Unset, each family takes the form measured fastest on the
// BASELINE shapes: the streamed kernel for f32 and bf16 RMS (it reads x
// once), the wave kernel for the fused int8 quantize.
enum RmsForm { kRmsFormAuto = 0, kRmsFormWave = 1, kRmsFormScan = 2, kRmsFormStream = 3 };
static int rms_form_selected() {
  static const int form = [] {
    const char* v = getenv("TILER_RMS_FORM");
    if (v && strcmp(v, "scan") == 0) return (int)kRmsFormScan;
    if (v && strcmp(v, "stream") == 0) return (int)kRmsFormStream;
    if (v && strcmp(v, "wave") == 0) return (int)kRmsFormWave;
    return (int)kRmsFormAuto;
  }();
  return form;
}
static bool rms_scan_form_selected() { return rms_form_selected() == kRmsFormScan; }

int launch_rms_norm_quantize_i8(const float* x, const float* w, int64_t w_row_stride, uint64_t rows,
                                uint64_t extent, float eps, int8_t* codes, float* scales, tiler_cuda_status* st,
                                int sm_count, cudaStream_t stream) {
  if (rows == 0 || extent == 0) return 0;
  const bool aligned = ((uintptr_t)x % 16 == 0) && ((uintptr_t)w % 16 == 0) && ((uintptr_t)codes % 4 == 0) &&
                       extent % 4 == 0;
  if (!aligned) return TILER_CUDA_UNSUPPORTED;
  if (rms_scan_form_selected() &&
      rms_scan_launch(0, 1, x, w, w_row_stride, rows, extent, eps, nullptr, codes, scales, st, sm_count, stream))
    return 0;
  if (rms_form_selected() == kRmsFormStream &&
      rms_stream_quant_launch(x, w, w_row_stride, rows, extent, eps, codes, scales, st, sm_count, stream))
    return 0;
  const uint64_t grid = umin64((uint64_t)sm_count, rows);
  cudaFuncSetAttribute(tiler_rms_norm_wave_quantize_i8, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       (int)kRmsSmemBytes);
  launch_kernel((const void*)tiler_rms_norm_wave_quantize_i8, "tiler_rms_norm_wave_quantize_i8", dim3((unsigned)grid),
                dim3(kRmsThreads), kRmsSmemBytes, stream, (const uint8_t*)x, (const uint8_t*)w, w_row_stride, rows,
                extent, eps, (uint8_t*)nullptr, (uint32_t)kRmsWave, st, codes, scales);
  return 0;
}

int launch_rms_norm(int bf16, const void* x, const void* w, int64_t w_row_stride, uint64_t rows, uint64_t extent,
                    float eps, void* y, tiler_cuda_status* st, int sm_count, cudaStream_t stream) {
  if (rows == 0 || extent == 0) return 0;
  const uint64_t esize = bf16 ? 2 : 4;
  const bool aligned = ((uintptr_t)x % 16 == 0) && ((uintptr_t)y % 16 == 0) && ((uintptr_t)w % 16 == 0) &&
                       ((extent * esize) % 16 == 0);
  if (!aligned) {
    const unsigned wpb = 8;
    const unsigned blocks = (unsigned)((rows + wpb - 1) / wpb);
    if (bf16)
      rms_norm_generic_kernel<true><<<blocks, wpb * 32, 0, stream>>>(x, w, w_row_stride, rows, extent, eps, y);
    else
      rms_norm_generic_kernel<false><<<blocks, wpb * 32, 0, stream>>>(x, w, w_row_stride, rows, extent, eps, y);
    return 0;
  }
  // The warp-per-row form when selected and where it applies (broadcast
  // weights, rows up to 16 KB)
  if (rms_scan_form_selected() &&
      rms_scan_launch(bf16, 0, x, w, w_row_stride, rows, extent, eps, y, nullptr, nullptr, st, sm_count, stream))
    return 0;
  const int form = rms_form_selected();
  if ((form == kRmsFormStream || form == kRmsFormAuto) &&
      rms_stream_launch(bf16, x, w, w_row_stride, rows, extent, eps, y, st, sm_count, stream))
    return 0;
  // One CTA per SM; each takes rows/grid consecutive rows in waves.
  const uint64_t grid = umin64((uint64_t)sm_count, rows);
  const void* fn = bf16 ? (const void*)tiler_rms_norm_wave_bf16 : (const void*)tiler_rms_norm_wave_f32;
  cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRmsSmemBytes);
  launch_kernel(fn, bf16 ? "tiler_rms_norm_wave_bf16" : "tiler_rms_norm_wave_f32", dim3((unsigned)grid),
                dim3(kRmsThreads), kRmsSmemBytes, stream, (const uint8_t*)x, (const uint8_t*)w, w_row_stride, rows,
                extent, eps, (uint8_t*)y, (uint32_t)kRmsWave, st, (int8_t*)nullptr, (float*)nullptr);
  return 0;
}

// ---------------------------------------------------------------------------
// Softmax (softmax.rs:260-315) with the in-kernel causal block mask.
// ---------------------------------------------------------------------------
//
// Each CTA owns G row buffers in shared memory (a buffer is one whole row)
// and walks its groups of G consecutive rows:
//   1. row warp w bulk-copies row w in (one mbarrier per row buffer), once
//      its previous row's bulk store has read the buffer;
//   2. warp w takes row w: with a mask tensor, t = x + mask first (in
//      place); the row maximum over the unmasked columns (order-free,
//      NaN-propagating), then e_i = exp(x_i - m) in place (certified exp,
//      branch-free with one warp-uniform branch for flagged arguments); with
//      the causal mask, columns past the diagonal hold e = +0 exactly
//      (x + -inf = -inf), so they are zero-filled without evaluating exp,
//      and a masked x that is NaN or +inf (which makes that e NaN) is
//      recorded as a poisoned row;
//   3. the chain warp folds all G denominators at once, lane w folding row
//      w strictly, d = (((e_0 + e_1) + e_2) + ...), up to the diagonal only
//      with the causal mask, up to the last nonzero e with a mask tensor
//      (adding +0.0 to a positive running sum is the identity), r = 1/d;
//   4. warp w forms out_i = e_i * r in place over the live columns and
//      writes the row back with one bulk store.
// Four CTAs share an SM, so one CTA's loads and folds overlap the others'
// exponentials and stores.

#ifndef TILER_SMX_CTAS_PER_SM
#define TILER_SMX_CTAS_PER_SM 4
#endif
#ifndef TILER_SMX_MAX_GROUP
#define TILER_SMX_MAX_GROUP 6
#endif
#ifndef TILER_SMX_EXP_VECS
#define TILER_SMX_EXP_VECS 1
#endif
constexpr int kSmxMaxGroup = TILER_SMX_MAX_GROUP;  // rows per CTA group
constexpr uint64_t kSmxMaxExtent = 8192;

__device__ __forceinline__ float max_nan(float a, float b) {
  float d;
  asm("max.NaN.f32 %0, %1, %2;" : "=f"(d) : "f"(a), "f"(b));
  return d;
}

// e^sh for the group kernel's flagged arguments (out of the fast path's
// range, NaN, or near a rounding midpoint); kept out of line so the fast
// path's registers are not sized for it.
__device__ __noinline__ float softmax_exp_slow(float sh, const double* table, tiler_cuda_status* st) {
  return sh > -104.0f ? exp_cr(sh, table, st) : (is_nan_bits(sh) ? __uint_as_float(kCanonicalNan) : 0.0f);
}

// Step 2 of the softmax kernels for one row: with a mask tensor, t = x + mask
// in place; the row maximum over the unmasked columns; e_i = exp(x_i - m) in
// place (masked columns zero-filled); the row's poison flag and the end of its
// denominator fold go to *poisoned_out and *fold_end_out (lane 0).
__device__ __forceinline__ void softmax_row_exp(float* b, uint64_t row, uint32_t lane, uint64_t extent, bool causal,
                                                uint64_t period, uint64_t row_offset, const float* __restrict__ mask,
                                                uint64_t mask_rows, const double* table, tiler_cuda_status* st,
                                                uint32_t* poisoned_out, uint32_t* fold_end_out) {
  const uint32_t ext = (uint32_t)extent;
  const uint32_t live = causal ? (uint32_t)umin64((row_offset + row) % period + 1, extent) : ext;
  float4* b4 = reinterpret_cast<float4*>(b);
  float m = __uint_as_float(0xff800000u);
  const uint32_t live4 = live / 4;
  if (mask) {
    // the program's additive mask (an add-f32 of a broadcast mask tensor,
    // standard.rs:211-221): t = x + mask[row mod mask_rows], one rounding,
    // NaN canonicalized, written back in place before the maximum
    const float4* m4 = reinterpret_cast<const float4*>(mask + ((row_offset + row) % mask_rows) * extent);
    for (uint32_t v = lane; v < live4; v += 32) {
      const float4 q = b4[v], a = __ldg(m4 + v);
      const float4 t = make_float4(canon(__fadd_rn(q.x, a.x)), canon(__fadd_rn(q.y, a.y)),
                                   canon(__fadd_rn(q.z, a.z)), canon(__fadd_rn(q.w, a.w)));
      b4[v] = t;
      m = max_nan(max_nan(m, t.x), max_nan(t.y, max_nan(t.z, t.w)));
    }
  } else {
    for (uint32_t v = lane; v < live4; v += 32) {
      const float4 q = b4[v];
      m = max_nan(max_nan(m, q.x), max_nan(q.y, max_nan(q.z, q.w)));
    }
  }
  for (uint32_t c = live4 * 4 + lane; c < live; c += 32) m = max_nan(m, b[c]);
  uint32_t bad = 0;  // a masked x that is NaN or +inf poisons the row
  const uint32_t mask4 = (live + 3) / 4;  // first whole masked vector
  auto poison = [](uint32_t xb) { return (uint32_t)(((xb & 0x7fffffffu) > 0x7f800000u) | (xb == 0x7f800000u)); };
  for (uint32_t c = live + lane; c < mask4 * 4 && c < ext; c += 32) bad |= poison(__float_as_uint(b[c]));
  for (uint32_t v = mask4 + lane; v < ext / 4; v += 32) {
    const uint4 q = reinterpret_cast<const uint4*>(b)[v];
    bad |= poison(q.x) | poison(q.y) | poison(q.z) | poison(q.w);
  }
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) m = max_nan(m, __shfl_xor_sync(0xffffffffu, m, o));
  bad = __any_sync(0xffffffffu, bad != 0);
  // m is -inf only if every unmasked x is -inf: x - m is then NaN
  auto exp_of = [&](float xv) {
    const float sh = __fsub_rn(xv, m);
    return sh > -104.0f ? exp_cr_fast(sh, table, st) : (is_nan_bits(sh) ? __uint_as_float(kCanonicalNan) : 0.0f);
  };
  uint32_t last_nz = 0;  // one past this lane's last nonzero e (mask tensor only)
  // TRACK (a mask tensor): arguments at or below -104 give +0 without
  // certification and the last nonzero e is tracked, so the fold can stop
  // there; the in-kernel causal mask already stops at the diagonal
  auto exp_pass = [&](auto track) {
    constexpr bool TRACK = decltype(track)::value;
    constexpr int EV = TILER_SMX_EXP_VECS;  // float4s per lane per step: 4 * EV independent exps
    for (uint32_t v0 = lane; v0 < live4; v0 += 32 * EV) {
      float xs[4 * EV];
      uint32_t e[4 * EV], flagged = 0;
#pragma unroll
      for (int h = 0; h < EV; ++h) {
        const uint32_t v = v0 + 32 * h;
        const float4 q = v < live4 ? b4[v] : make_float4(0.f, 0.f, 0.f, 0.f);
        xs[4 * h] = q.x; xs[4 * h + 1] = q.y; xs[4 * h + 2] = q.z; xs[4 * h + 3] = q.w;
      }
      if (TRACK) {
        // a step whose arguments are all at or below -104 (a masked stretch)
        // is +0 throughout: skip the evaluation when the whole warp agrees
        bool low = true;
#pragma unroll
        for (int i = 0; i < 4 * EV; ++i) {
          const float sh = __fsub_rn(xs[i], m);
          low = low && !(sh > -104.0f) && !is_nan_bits(sh);
        }
        if (__all_sync(__activemask(), low)) {
#pragma unroll
          for (int h = 0; h < EV; ++h) {
            const uint32_t v = v0 + 32 * h;
            if (v < live4) b4[v] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
          }
          continue;
        }
      }
#pragma unroll
      for (int i = 0; i < 4 * EV; ++i) {
        const float sh = __fsub_rn(xs[i], m);
        bool ok;
        e[i] = exp_cr_bits(sh, table, &ok);
        if (TRACK) {
          // e^sh = +0 for sh <= -104 (silu.rs:224-235 guards): no certification needed
          const bool zero = !(sh > -104.0f) && !is_nan_bits(sh);
          if (zero) e[i] = 0u;
          flagged |= ((ok && sh > -104.0f) || zero ? 0u : 1u) << i;
        } else {
          flagged |= ((ok && sh > -104.0f) ? 0u : 1u) << i;
        }
      }
      if (__any_sync(__activemask(), flagged != 0)) {  // rare: certify or special-case the flagged ones
#pragma unroll
        for (int i = 0; i < 4 * EV; ++i)
          if ((flagged >> i) & 1u) e[i] = __float_as_uint(softmax_exp_slow(__fsub_rn(xs[i], m), table, st));
      }
#pragma unroll
      for (int h = 0; h < EV; ++h) {
        const uint32_t v = v0 + 32 * h;
        if (v < live4) {
          b4[v] = make_float4(__uint_as_float(e[4 * h]), __uint_as_float(e[4 * h + 1]),
                              __uint_as_float(e[4 * h + 2]), __uint_as_float(e[4 * h + 3]));
          if (TRACK) {
#pragma unroll
            for (int i = 0; i < 4; ++i)
              if (e[4 * h + i] != 0u) last_nz = max(last_nz, v * 4 + i + 1);
          }
        }
      }
    }
  };
  if (mask) exp_pass(std::true_type{});
  else exp_pass(std::false_type{});
  for (uint32_t c = live4 * 4 + lane; c < live; c += 32) {
    b[c] = exp_of(b[c]);
    if (mask && __float_as_uint(b[c]) != 0u) last_nz = max(last_nz, c + 1);
  }
  for (uint32_t c = live + lane; c < mask4 * 4 && c < ext; c += 32) b[c] = 0.0f;
  for (uint32_t v = mask4 + lane; v < ext / 4; v += 32) b4[v] = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
  if (mask) last_nz = __reduce_max_sync(0xffffffffu, last_nz);
  if (lane == 0) {
    *poisoned_out = bad;
    *fold_end_out = mask ? max(last_nz, 1u) : live;  // at least e_0, the seed
  }
}

// Step 3: lane r < n folds row r's denominator strictly,
// d = (((e_0 + e_1) + e_2) + ...) up to fold_end[r], and stores r = 1/d (NaN
// for a poisoned row) in rcp[r].
__device__ __forceinline__ void softmax_chain_fold(uint32_t lane, uint32_t n, const float* bufs, uint32_t ext,
                                                   const uint32_t* fold_end, const uint32_t* poisoned, float* rcp) {
  if (lane < n) {
    const uint32_t live = fold_end[lane];  // the unmasked columns up to the last nonzero e
    const uint32_t base = smem_u32(bufs + (uint64_t)lane * ext);
    const float* b = bufs + (uint64_t)lane * ext;
    float acc = b[0];
    uint32_t c = 1;
    for (; c < live && (c & 3); ++c) acc = __fadd_rn(acc, b[c]);
    const uint32_t nv = (live - c) / 4;
    uint32_t v = 0;
    for (; v + 8 <= nv; v += 8) {
      uint4 q[8];
#pragma unroll
      for (int k = 0; k < 8; ++k) q[k] = lds_u4(base + (c + 4 * (v + k)) * 4);
#pragma unroll
      for (int k = 0; k < 8; ++k) {
        acc = __fadd_rn(acc, __uint_as_float(q[k].x));
        acc = __fadd_rn(acc, __uint_as_float(q[k].y));
        acc = __fadd_rn(acc, __uint_as_float(q[k].z));
        acc = __fadd_rn(acc, __uint_as_float(q[k].w));
      }
    }
    for (; v < nv; ++v) {
      const uint4 q = lds_u4(base + (c + 4 * v) * 4);
      acc = __fadd_rn(acc, __uint_as_float(q.x));
      acc = __fadd_rn(acc, __uint_as_float(q.y));
      acc = __fadd_rn(acc, __uint_as_float(q.z));
      acc = __fadd_rn(acc, __uint_as_float(q.w));
    }
    for (c += 4 * nv; c < live; ++c) acc = __fadd_rn(acc, b[c]);
    const float r = __fdiv_rn(1.0f, acc);
    rcp[lane] = (poisoned[lane] || is_nan_bits(r)) ? __uint_as_float(kCanonicalNan) : r;
  }
}

// Step 4: out = e * r (softmax.rs:306-312) in place over the row's live
// columns, then one bulk store of the row (committed as a bulk group of the
// calling lane 0).
__device__ __forceinline__ void softmax_row_store(float* rowbuf, uint64_t row, uint32_t lane, float r, bool causal,
                                                  uint64_t period, uint64_t row_offset, uint64_t extent,
                                                  float* __restrict__ y) {
  const uint32_t ext = (uint32_t)extent, row_bytes = ext * 4;
  float4* b4 = reinterpret_cast<float4*>(rowbuf);
  if (is_nan_bits(r)) {
    const float nanv = __uint_as_float(kCanonicalNan);
    for (uint32_t v = lane; v < ext / 4; v += 32) b4[v] = make_float4(nanv, nanv, nanv, nanv);
  } else {
    // e is finite and >= 0 and r finite: the product is never NaN; the
    // masked tail already holds zeros (0 * r = +0)
    const uint64_t row_live = causal ? umin64((row_offset + row) % period + 1, extent) : extent;
    const uint32_t nv = (uint32_t)((row_live + 3) / 4);
    for (uint32_t v = lane; v < nv; v += 32) {
      const float4 q = b4[v];
      b4[v] = make_float4(__fmul_rn(q.x, r), __fmul_rn(q.y, r), __fmul_rn(q.z, r), __fmul_rn(q.w, r));
    }
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  __syncwarp();
  if (lane == 0) {
    asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(y + row * extent),
                 "r"(smem_u32(b4)), "r"(row_bytes)
                 : "memory");
    asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  }
}

__global__ void __launch_bounds__(32 * (kSmxMaxGroup + 1), TILER_SMX_CTAS_PER_SM)
    softmax_group_kernel(const float* __restrict__ x, uint64_t rows, uint64_t extent, uint64_t period,
                         uint64_t row_offset, float* __restrict__ y, uint32_t group, tiler_cuda_status* st,
                         const float* __restrict__ mask = nullptr, uint64_t mask_rows = 0) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  double* table = reinterpret_cast<double*>(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + 2048);  // one per row buffer
  float* rcp = reinterpret_cast<float*>(smem_raw + 2048 + 128);
  uint32_t* poisoned = reinterpret_cast<uint32_t*>(smem_raw + 2048 + 192);
  // fold_end[w]: the denominator fold of row w stops here; past it every e is
  // +0 exactly, and adding +0 to the positive running sum is the identity
  uint32_t* fold_end = reinterpret_cast<uint32_t*>(smem_raw + 2048 + 224);
  float* bufs = reinterpret_cast<float*>(smem_raw + 2048 + 256);
  // warp 0 folds the denominators (the oldest warp, so the scheduler tends to
  // favour its dependent chain); warp w + 1 handles row w of each group.
  const uint32_t lane = threadIdx.x & 31;
  const bool chain_warp = (threadIdx.x >> 5) == 0;
  const uint32_t warp = (threadIdx.x >> 5) - 1;  // row index for the row warps
  const uint32_t G = group;
  const uint32_t ext = (uint32_t)extent, row_bytes = ext * 4;
  // Groups are G consecutive rows (similar causal lengths, so the lockstep
  // fold of a group wastes little); CTA b takes groups b, b + grid, ... so
  // every CTA gets a mix of short and long groups.
  const uint64_t total_groups = (rows + G - 1) / G;
  const uint64_t ngroups = total_groups > blockIdx.x ? (total_groups - blockIdx.x + gridDim.x - 1) / gridDim.x : 0;
  auto group_row0 = [&](uint64_t g) { return (blockIdx.x + g * (uint64_t)gridDim.x) * G; };
  const bool causal = period != 0;
  const uint64_t drop = policy_evict_first();

  load_exp_table(table);
  if (threadIdx.x < kSmxMaxGroup) mbar_init(&full[threadIdx.x], 1);
  fence_barrier_init();
  __syncthreads();

  for (uint64_t g = 0; g < ngroups; ++g) {
    const uint64_t row0 = group_row0(g);
    const uint32_t n = (uint32_t)umin64(G, rows - row0);
    // each row warp loads its own row; its previous bulk store must have
    // finished reading the buffer first
    bool ok = true;
    if (!chain_warp && warp < n) {
      if (lane == 0) {
        asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
        mbar_arrive_expect_tx(&full[warp], row_bytes);
        bulk_g2s(bufs + (uint64_t)warp * ext, x + (row0 + warp) * extent, row_bytes, &full[warp], drop);
      }
      ok = mbar_wait(&full[warp], (uint32_t)(g & 1), st);
    }

    if (!chain_warp && warp < n) {
      softmax_row_exp(bufs + (uint64_t)warp * ext, row0 + warp, lane, extent, causal, period, row_offset, mask,
                      mask_rows, table, st, &poisoned[warp], &fold_end[warp]);
    }
    if (!__syncthreads_and(ok)) {
      if (lane == 0 && !chain_warp) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
      return;
    }

    if (chain_warp) {
      softmax_chain_fold(lane, n, bufs, ext, fold_end, poisoned, rcp);
    }
    __syncthreads();

    if (!chain_warp && warp < n) {
      softmax_row_store(bufs + (uint64_t)warp * ext, row0 + warp, lane, rcp[warp], causal, period, row_offset, extent,
                        y);
    }
    // no barrier here: a row warp reloads only its own buffer, after its store
  }
  if (lane == 0 && !chain_warp) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");  // stores complete
}

__device__ __forceinline__ float masked_value(float v, uint64_t col, uint64_t diag, bool causal) {
  return (causal && col > diag) ? __fadd_rn(v, __uint_as_float(0xff800000u)) : v;
}

// Any-shape path: one warp per row, y doubles as the exponential scratch.
__global__ void softmax_generic_kernel(const float* __restrict__ x, uint64_t rows, uint64_t extent, uint64_t period,
                                       uint64_t row_offset, float* __restrict__ y, tiler_cuda_status* st) {
  __shared__ double table[256];
  load_exp_table(table);
  __syncthreads();
  const uint64_t row = blockIdx.x * (uint64_t)(blockDim.x / 32) + threadIdx.x / 32;
  const uint32_t lane = threadIdx.x & 31;
  if (row >= rows) return;
  const float* xr = x + row * extent;
  float* yr = y + row * extent;
  const bool causal = period != 0;
  const uint64_t diag = causal ? (row_offset + row) % period : 0;
  float m = __uint_as_float(0xff800000u);
  for (uint64_t i = lane; i < extent; i += 32) m = maximum(m, masked_value(xr[i], i, diag, causal));
#pragma unroll
  for (int k = 1; k < 32; k <<= 1) m = maximum(m, __shfl_xor_sync(0xffffffffu, m, k));
  for (uint64_t i = lane; i < extent; i += 32) yr[i] = exp_cr(__fsub_rn(masked_value(xr[i], i, diag, causal), m), table, st);
  __syncwarp();
  float rcp = 0.0f;
  if (lane == 0) {
    float d = yr[0];
    for (uint64_t i = 1; i < extent; ++i) d = __fadd_rn(d, yr[i]);
    rcp = __fdiv_rn(1.0f, d);
  }
  rcp = __shfl_sync(0xffffffffu, rcp, 0);
  __syncwarp();
  for (uint64_t i = lane; i < extent; i += 32) yr[i] = canon(__fmul_rn(yr[i], rcp));
}

int launch_softmax(const float* x, uint64_t rows, uint64_t extent, uint64_t causal_period, uint64_t row_offset,
                   float* y, tiler_cuda_status* st, int sm_count, cudaStream_t stream, const float* mask,
                   uint64_t mask_rows) {
  if (rows == 0 || extent == 0) return 0;
  // G rows per CTA, sized so three CTAs share an SM's shared memory.
  const size_t fixed = 2048 + 256, row_bytes = extent * 4;
  const uint64_t g3 = ((224 * 1024) / TILER_SMX_CTAS_PER_SM - 1024 - fixed) / row_bytes;
  const uint64_t g1 = (220 * 1024 - fixed) / row_bytes;
  const uint64_t G = umin64(kSmxMaxGroup, umin64(rows, g3 >= 4 ? g3 : g1));
  const bool staged = (extent % 4 == 0) && extent <= kSmxMaxExtent && ((uintptr_t)x % 16 == 0) &&
                      ((uintptr_t)y % 16 == 0) && G >= 1;
  if (mask && (!staged || causal_period != 0 || (uintptr_t)mask % 16 != 0 || mask_rows == 0))
    return TILER_CUDA_UNSUPPORTED;  // the masked form runs on the staged kernel only
  if (!staged) {
    const unsigned wpb = 8;
    softmax_generic_kernel<<<(unsigned)((rows + wpb - 1) / wpb), wpb * 32, 0, stream>>>(x, rows, extent,
                                                                                       causal_period, row_offset, y, st);
    return 0;
  }
  const size_t smem = fixed + G * row_bytes;
  cudaFuncSetAttribute(softmax_group_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  // all of the SM's unified L1/shared storage as shared memory, so three CTAs fit
  cudaFuncSetAttribute(softmax_group_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  const int per_sm = std::max<int>(1, (int)((228 * 1024) / (smem + 1024)));
  const unsigned grid = (unsigned)umin64((rows + G - 1) / G, (uint64_t)sm_count * per_sm);
  softmax_group_kernel<<<grid, (unsigned)(32 * (G + 1)), smem, stream>>>(x, rows, extent, causal_period,
                                                                          row_offset, y, (uint32_t)G, st, mask,
                                                                          mask_rows);
  return 0;
}

// ---------------------------------------------------------------------------
// Per-row int8 strict-affine quantize and decode.
// ---------------------------------------------------------------------------
//
// One CTA per row.  Pass 1 folds max|x| (order-free maximum) and finds the
// first NaN; scale = max/127 (one division), refused unless positive-normal;
// pass 2 (an L1/L2-resident re-read) forms code = RNE(clamp(x/scale)).  The
// quotient is formed as x * (1/scale) and taken only when it is provably on
// the same side of every half-integer as the correctly rounded x/scale
// (|error| < 2^-16 below 128); within 2.5e-5 of a half-integer the exact
// IEEE division decides, so codes equal the oracle's bit for bit.

constexpr int kQThreads = 256;

__device__ __forceinline__ int8_t code_of(float xv, float scale, float inv) {
  float q = __fmul_rn(xv, inv);
  const float frac = fabsf(q - truncf(q));
  if (fabsf(frac - 0.5f) < 2.5e-5f || !isfinite(q)) q = __fdiv_rn(xv, scale);
  q = __fadd_rn(q, 0.0f);
  q = fminf(fmaxf(q, -127.0f), 127.0f);
  return (int8_t)__float2int_rn(q);
}

// code_of for |x| <= max|x| of a NaN-free row: then |x * (1/scale)| stays
// below 127 * (1 + 2^-21), so its rounding to an integer needs no clamp and
// the value is finite.  The product is taken unless it lies within 2.5e-5 of
// a half-integer; there the exact IEEE quotient decides (as in code_of).
__device__ __forceinline__ int code_of_bounded(float xv, float scale, float inv) {
  float q = __fmul_rn(xv, inv);
  float r = rintf(q);
  if (fabsf(__fsub_rn(q, r)) > 0.49997f) {
    q = __fdiv_rn(xv, scale);
    r = rintf(q);
  }
  return max(-127, min(127, __float2int_rn(r)));
}

// Row values are held in registers (up to kQMaxVec float4 per thread, rows of
// up to 4096 f32 with 256 threads), so x is read from HBM exactly once: all
// of a thread's loads are issued before the maximum consumes them.
constexpr int kQMaxVec = 4;

__device__ __forceinline__ void quantize_load_row(const float* xr, uint32_t nvec, float4 (&q)[kQMaxVec]) {
  const float4* x4 = reinterpret_cast<const float4*>(xr);
#pragma unroll
  for (int k = 0; k < kQMaxVec; ++k) {
    const uint32_t v = threadIdx.x + k * kQThreads;
    q[k] = v < nvec ? __ldcs(x4 + v) : make_float4(0.f, 0.f, 0.f, 0.f);
  }
}

// CTA b codes rows b, b + grid, ... (the launch uses one CTA per row).
__global__ void __launch_bounds__(kQThreads) quantize_i8_rows_kernel(const float* __restrict__ x, uint64_t rows,
                                                                    uint64_t extent, int8_t* __restrict__ codes,
                                                                    float* __restrict__ scales,
                                                                    tiler_cuda_status* st) {
  __shared__ float red[2][kQThreads / 32];
  __shared__ uint32_t nan_at[2][kQThreads / 32];
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t nvec = (uint32_t)(extent / 4);
  const bool regs = (extent % 4 == 0) && ((uintptr_t)x % 16 == 0) && nvec <= kQMaxVec * kQThreads &&
                    ((uintptr_t)codes % 4 == 0);
  float4 q[kQMaxVec], nq[kQMaxVec];
  uint64_t row = blockIdx.x;
  if (regs && row < rows) quantize_load_row(x + row * extent, nvec, nq);
  for (uint32_t it = 0; row < rows; row += gridDim.x, ++it) {
    const float* xr = x + row * extent;
    const uint32_t par = it & 1;
    float m = 0.0f;
    uint32_t first_nan = 0xffffffffu;  // column of the first NaN (extent < 2^32)
    if (regs) {
#pragma unroll
      for (int k = 0; k < kQMaxVec; ++k) q[k] = nq[k];
      if (row + gridDim.x < rows) quantize_load_row(x + (row + gridDim.x) * extent, nvec, nq);
#pragma unroll
      for (int k = 0; k < kQMaxVec; ++k) {
        const uint32_t v = threadIdx.x + k * kQThreads;
        if (v < nvec) {
          const float e[4] = {q[k].x, q[k].y, q[k].z, q[k].w};
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            if (is_nan_bits(e[j])) first_nan = min(first_nan, v * 4 + j);
            m = maximum(m, fabsf(e[j]));
          }
        }
      }
    } else {
      for (uint32_t i = threadIdx.x; i < (uint32_t)extent; i += kQThreads) {
        const float e = xr[i];
        if (is_nan_bits(e)) first_nan = min(first_nan, i);
        m = maximum(m, fabsf(e));
      }
    }
#pragma unroll
    for (int k = 1; k < 32; k <<= 1) {
      m = maximum(m, __shfl_xor_sync(0xffffffffu, m, k));
      first_nan = min(first_nan, __shfl_xor_sync(0xffffffffu, first_nan, k));
    }
    if (lane == 0) { red[par][warp] = m; nan_at[par][warp] = first_nan; }
    __syncthreads();  // double-buffered slots: the next row writes the other half
    m = red[par][0];
    first_nan = nan_at[par][0];
    for (int i = 1; i < kQThreads / 32; ++i) {
      m = maximum(m, red[par][i]);
      first_nan = min(first_nan, nan_at[par][i]);
    }
    if (first_nan != 0xffffffffu) {
      if (threadIdx.x == 0) report_error(st, row * extent + first_nan, TILER_CUDA_NAN_INPUT);
      continue;
    }
    // maximum|x| over a NaN-free row; 0 stays +0 (all |x| are non-negative)
    const float scale = __fdiv_rn(m, 127.0f);
    if (threadIdx.x == 0) scales[row] = scale;
    if (!is_positive_normal(scale)) {
      if (threadIdx.x == 0) report_error(st, row * extent, TILER_CUDA_SCALE_DOMAIN);
      continue;
    }
    const float inv = __frcp_rn(scale);
    int8_t* cr = codes + row * extent;
    if (regs) {
      char4* c4 = reinterpret_cast<char4*>(cr);
#pragma unroll
      for (int k = 0; k < kQMaxVec; ++k) {
        const uint32_t v = threadIdx.x + k * kQThreads;
        if (v < nvec)
          __stcs(reinterpret_cast<int*>(c4 + v),
                 (int)(uint8_t)code_of(q[k].x, scale, inv) | ((int)(uint8_t)code_of(q[k].y, scale, inv) << 8) |
                     ((int)(uint8_t)code_of(q[k].z, scale, inv) << 16) |
                     ((int)(uint8_t)code_of(q[k].w, scale, inv) << 24));
      }
    } else {
      for (uint32_t i = threadIdx.x; i < (uint32_t)extent; i += kQThreads) cr[i] = code_of(xr[i], scale, inv);
    }
  }
}

// Staged variant for rows of up to 16 KB (16-byte aligned, extent a multiple
// of 4): a persistent CTA double-buffers rows in shared memory, thread 0
// bringing row i + 2 * grid in with one bulk copy while the CTA codes row i,
// so every SM keeps 2 rows per CTA in flight at no register cost.  Same
// numerics and error rules as the kernel above.
constexpr int kQbThreads = 256;
constexpr int kQbCtasPerSm = 6;
constexpr uint32_t kQbMaxRowBytes = 16384;

__global__ void __launch_bounds__(kQbThreads, kQbCtasPerSm)
    quantize_i8_rows_bulk_kernel(const float* __restrict__ x, uint64_t rows, uint64_t extent,
                                 int8_t* __restrict__ codes, float* __restrict__ scales, tiler_cuda_status* st) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  float* buf = reinterpret_cast<float*>(smem_raw);  // [2][kQbMaxRowBytes / 4]
  uint64_t* full = reinterpret_cast<uint64_t*>(smem_raw + 2 * kQbMaxRowBytes);
  __shared__ uint32_t nan_at[kQbThreads / 32];
  __shared__ int abort_flag;
  const uint32_t lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const uint32_t row_bytes = (uint32_t)extent * 4, nvec = (uint32_t)(extent / 4);
  const uint64_t pol = policy_evict_first();
  auto issue = [&](uint64_t row, uint32_t b) {
    mbar_arrive_expect_tx(&full[b], row_bytes);
    bulk_g2s(buf + b * (kQbMaxRowBytes / 4), x + row * extent, row_bytes, &full[b], pol);
  };
  if (threadIdx.x == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    abort_flag = 0;
    fence_barrier_init();
    if (blockIdx.x < rows) issue(blockIdx.x, 0);
    if (blockIdx.x + gridDim.x < rows) issue(blockIdx.x + gridDim.x, 1);
  }
  __syncthreads();
  uint32_t it = 0;
  for (uint64_t row = blockIdx.x; row < rows; row += gridDim.x, ++it) {
    const uint32_t b = it & 1;
    if (!mbar_wait(&full[b], (it >> 1) & 1, st)) abort_flag = 1;
    const float4* b4 = reinterpret_cast<const float4*>(buf + b * (kQbMaxRowBytes / 4));
    // max|x| as an unsigned maximum of the magnitude bits: for non-NaN
    // values it orders like the float maximum (all magnitudes are >= +0);
    // a NaN shows as a maximum above 0x7f800000 and is then located exactly.
    uint32_t mb = 0;
    for (uint32_t v = threadIdx.x; v < nvec; v += kQbThreads) {
      const uint4 q = *reinterpret_cast<const uint4*>(b4 + v);
      mb = max(mb, max(max(q.x & 0x7fffffffu, q.y & 0x7fffffffu), max(q.z & 0x7fffffffu, q.w & 0x7fffffffu)));
    }
    mb = __reduce_max_sync(0xffffffffu, mb);
    if (lane == 0) nan_at[warp] = mb;
    __syncthreads();
    if (abort_flag) break;
    mb = nan_at[0];
    for (int i = 1; i < kQbThreads / 32; ++i) mb = max(mb, nan_at[i]);
    if (mb > 0x7f800000u) {
      // rare: the row holds a NaN; report its first column
      uint32_t first_nan = 0xffffffffu;
      for (uint32_t v = threadIdx.x; v < nvec; v += kQbThreads) {
        const float4 q = b4[v];
        const float e[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
        for (int j = 0; j < 4; ++j)
          if (is_nan_bits(e[j])) first_nan = min(first_nan, v * 4 + j);
      }
      first_nan = __reduce_min_sync(0xffffffffu, first_nan);
      __syncthreads();  // everyone has read nan_at
      if (lane == 0) nan_at[warp] = first_nan;
      __syncthreads();
      if (threadIdx.x == 0) {
        for (int i = 1; i < kQbThreads / 32; ++i) first_nan = min(first_nan, nan_at[i]);
        first_nan = min(first_nan, nan_at[0]);
        report_error(st, row * extent + first_nan, TILER_CUDA_NAN_INPUT);
      }
    } else {
      const float m = __uint_as_float(mb);
      const float scale = __fdiv_rn(m, 127.0f);
      if (threadIdx.x == 0) scales[row] = scale;
      if (!is_positive_normal(scale)) {
        if (threadIdx.x == 0) report_error(st, row * extent, TILER_CUDA_SCALE_DOMAIN);
      } else {
        const float inv = __frcp_rn(scale);
        int* c4 = reinterpret_cast<int*>(codes + row * extent);
        for (uint32_t v = threadIdx.x; v < nvec; v += kQbThreads) {
          const float4 q = b4[v];
          const float e[4] = {q.x, q.y, q.z, q.w};
          int c[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) c[j] = code_of_bounded(e[j], scale, inv);
          // cvt.pack d, a, b, c: d = c << 16 | sat8(a) << 8 | sat8(b)
          uint32_t hi, packed;
          asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, 0;" : "=r"(hi) : "r"(c[3]), "r"(c[2]));
          asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(packed) : "r"(c[1]), "r"(c[0]), "r"(hi));
          __stcs(c4 + v, (int)packed);
        }
      }
    }
    __syncthreads();  // buffer b and the reduction slots are free again
    if (threadIdx.x == 0 && row + 2 * (uint64_t)gridDim.x < rows) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      issue(row + 2 * (uint64_t)gridDim.x, b);
    }
  }
  // a copy still in flight (abort) must land before the CTA's shared memory is released
  if (threadIdx.x == 0 && abort_flag) {
    for (uint32_t k = 0; k < 2; ++k) (void)mbar_wait(&full[(it + k) & 1], ((it + k) >> 1) & 1, nullptr);
  }
}

void launch_quantize_i8_rows(const float* x, uint64_t rows, uint64_t extent, int8_t* codes, float* scales,
                             tiler_cuda_status* st, int sm_count, cudaStream_t stream) {
  if (rows == 0) return;
  const bool staged = extent > 0 && extent % 4 == 0 && extent * 4 <= kQbMaxRowBytes && (uintptr_t)x % 16 == 0 &&
                      (uintptr_t)codes % 4 == 0;
  if (staged) {
    const size_t smem = 2 * kQbMaxRowBytes + 16;
    cudaFuncSetAttribute(quantize_i8_rows_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(quantize_i8_rows_bulk_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    const unsigned grid = (unsigned)umin64(rows, (uint64_t)sm_count * kQbCtasPerSm);
    quantize_i8_rows_bulk_kernel<<<grid, kQbThreads, smem, stream>>>(x, rows, extent, codes, scales, st);
    return;
  }
  // one CTA per row measured fastest here (short-lived CTAs keep many rows' loads in flight)
  const unsigned grid = (unsigned)rows;
  quantize_i8_rows_kernel<<<grid, kQThreads, 0, stream>>>(x, rows, extent, codes, scales, st);
}

__global__ void __launch_bounds__(256) dequantize_i8_rows_kernel(const int8_t* __restrict__ codes,
                                                                  const float* __restrict__ scales, uint64_t rows,
                                                                  uint64_t extent, float* __restrict__ y) {
  const bool vec = (extent % 16 == 0) && ((uintptr_t)codes % 16 == 0) && ((uintptr_t)y % 16 == 0);
  for (uint64_t row = blockIdx.x; row < rows; row += gridDim.x) {
  const float s = __ldg(scales + row);
  const int8_t* cr = codes + row * extent;
  float* yr = y + row * extent;
  auto dec = [s](uint32_t w, int j) {
    const int8_t code = (int8_t)((w >> (8 * j)) & 0xff);
    return code == 0 ? 0.0f : __fmul_rn((float)code, s);
  };
  if (vec) {
    const uint4* c16 = reinterpret_cast<const uint4*>(cr);
    float4* y4 = reinterpret_cast<float4*>(yr);
    const uint32_t nv = (uint32_t)(extent / 16);
    constexpr int U = 2;
    for (uint32_t v0 = threadIdx.x; v0 < nv; v0 += blockDim.x * U) {
      uint4 c[U];
#pragma unroll
      for (int u = 0; u < U; ++u)
        if (v0 + u * blockDim.x < nv) c[u] = ld_global_nc_u4(c16 + v0 + u * blockDim.x);
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const uint32_t v = v0 + u * blockDim.x;
        if (v < nv) {
          const uint32_t w[4] = {c[u].x, c[u].y, c[u].z, c[u].w};
#pragma unroll
          for (int q = 0; q < 4; ++q)
            st_global_stream(y4 + v * 4 + q, make_float4(dec(w[q], 0), dec(w[q], 1), dec(w[q], 2), dec(w[q], 3)));
        }
      }
    }
  } else {
    for (uint64_t i = threadIdx.x; i < extent; i += blockDim.x) {
      const int8_t code = cr[i];
      yr[i] = code == 0 ? 0.0f : __fmul_rn((float)code, s);
    }
  }
  }
}

// Staged decode for rows whose codes and output are 16-byte aligned, extent
// a multiple of 16 and at most 4096: a persistent CTA double-buffers a row's
// codes (one bulk load), decodes them into a shared-memory output row and
// writes it back with one bulk store, so the 4x larger output stream goes
// through the copy engine instead of per-thread stores.
constexpr int kDqThreads = 256;
constexpr int kDqCtasPerSm = 4;
constexpr uint32_t kDqMaxExtent = 4096;

__global__ void __launch_bounds__(kDqThreads, kDqCtasPerSm)
    dequantize_i8_rows_bulk_kernel(const int8_t* __restrict__ codes, const float* __restrict__ scales, uint64_t rows,
                                   uint64_t extent, float* __restrict__ y, tiler_cuda_status* st) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  float* out = reinterpret_cast<float*>(smem_raw);                          // [2][kDqMaxExtent]
  uint8_t* in = smem_raw + 2 * kDqMaxExtent * 4;                           // [2][kDqMaxExtent]
  uint64_t* full = reinterpret_cast<uint64_t*>(in + 2 * kDqMaxExtent);     // [2]
  __shared__ int abort_flag;
  const uint32_t ext = (uint32_t)extent, nw = ext / 4;
  const uint64_t pol = policy_evict_first();
  auto issue = [&](uint64_t row, uint32_t b) {
    mbar_arrive_expect_tx(&full[b], ext);
    bulk_g2s(in + b * kDqMaxExtent, codes + row * extent, ext, &full[b], pol);
  };
  if (threadIdx.x == 0) {
    mbar_init(&full[0], 1);
    mbar_init(&full[1], 1);
    abort_flag = 0;
    fence_barrier_init();
    if (blockIdx.x < rows) issue(blockIdx.x, 0);
    if (blockIdx.x + gridDim.x < rows) issue(blockIdx.x + gridDim.x, 1);
  }
  __syncthreads();
  uint32_t it = 0;
  for (uint64_t row = blockIdx.x; row < rows; row += gridDim.x, ++it) {
    const uint32_t b = it & 1;
    if (threadIdx.x == 0) {
      // the store that last read out[b] (two rows ago) has finished reading
      asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
    }
    if (!mbar_wait(&full[b], (it >> 1) & 1, st)) abort_flag = 1;
    __syncthreads();
    if (abort_flag) break;
    const float s = __ldg(scales + row);
    const uint32_t* c32 = reinterpret_cast<const uint32_t*>(in + b * kDqMaxExtent);
    float4* o4 = reinterpret_cast<float4*>(out + b * kDqMaxExtent);
    for (uint32_t v = threadIdx.x; v < nw; v += kDqThreads) {
      const uint32_t w = c32[v];
      float d[4];
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const int8_t code = (int8_t)((w >> (8 * j)) & 0xff);
        d[j] = code == 0 ? 0.0f : __fmul_rn((float)code, s);
      }
      o4[v] = make_float4(d[0], d[1], d[2], d[3]);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0) {
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(y + row * extent),
                   "r"(smem_u32(out + b * kDqMaxExtent)), "r"(ext * 4)
                   : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      if (row + 2 * (uint64_t)gridDim.x < rows) issue(row + 2 * (uint64_t)gridDim.x, b);
    }
  }
  if (threadIdx.x == 0) {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    // a load still in flight (abort) must land before shared memory is released
    if (abort_flag)
      for (uint32_t k = 0; k < 2; ++k) (void)mbar_wait(&full[(it + k) & 1], ((it + k) >> 1) & 1, nullptr);
  }
}

void launch_dequantize_i8_rows(const int8_t* codes, const float* scales, uint64_t rows, uint64_t extent, float* y,
                               int sm_count, cudaStream_t stream, tiler_cuda_status* st) {
  if (rows == 0 || extent == 0) return;
  const bool staged = extent % 16 == 0 && extent <= kDqMaxExtent && (uintptr_t)codes % 16 == 0 &&
                      (uintptr_t)y % 16 == 0;
  if (staged) {
    const size_t smem = 2 * kDqMaxExtent * 5 + 16;
    cudaFuncSetAttribute(dequantize_i8_rows_bulk_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    cudaFuncSetAttribute(dequantize_i8_rows_bulk_kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
    const unsigned grid = (unsigned)umin64(rows, (uint64_t)sm_count * kDqCtasPerSm);
    dequantize_i8_rows_bulk_kernel<<<grid, kDqThreads, smem, stream>>>(codes, scales, rows, extent, y, st);
    return;
  }
  const unsigned threads = (unsigned)umin64(256, std::max<uint64_t>(32, (extent / 16 + 31) / 32 * 32));
  const unsigned grid = (unsigned)rows;
  dequantize_i8_rows_kernel<<<grid, threads, 0, stream>>>(codes, scales, rows, extent, y);
}

}  // namespace tc
