// RMS normalization, one warp per row, the row held in shared memory once.
//
// rms_norm.rs:136-194 and :453-489 per row: a strict left fold of x_i*x_i
// seeded at the first square, mean = total / N, t = mean + eps, s = the
// correctly rounded 1/sqrt(t), y_i = w_i * (x_i * s) (two roundings), NaN
// canonicalized.  The squares are non-negative, so the strict fold runs as the
// warp-cooperative scan of strict_fold.cuh -- exact, and with no serial chain
// -- and a warp can take a whole row by itself:
//
//   1. lane 0 bulk-copies the row into the warp's shared-memory slot (one
//      cp.async.bulk completing on the slot's mbarrier), up to two rows ahead;
//   2. the warp folds the squares 256 at a time (lane l: terms 8l .. 8l+7);
//   3. the warp forms y from the same staged row and the staged weight row and
//      writes it with 32-byte streaming stores (the fused quantize form
//      instead takes max|y| and then the int8 codes from the same staged row).
//
// HBM traffic is one read of x and one write of y: nothing is re-read.
// Rows go round-robin over all warps of the grid (one CTA per SM).
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"
#include "strict_fold.cuh"

namespace tc {

#ifndef TILER_RS_WARPS
#define TILER_RS_WARPS 12
#endif
#ifndef TILER_RS_SLOT
#define TILER_RS_SLOT 16384
#endif
#ifndef TILER_RS_SERIAL
#define TILER_RS_SERIAL 64
#endif
constexpr int kRsWarps = TILER_RS_WARPS;
constexpr uint32_t kRsSlotBytes = TILER_RS_SLOT;  // per warp: e.g. one f32 row of 4096, or two bf16 rows
constexpr uint32_t kRsWeightBytes = 16384;
constexpr int kRsThreads = 32 * kRsWarps;

struct RsSmem {
  alignas(128) uint8_t slot[kRsWarps][kRsSlotBytes];
  alignas(16) uint8_t wrow[kRsWeightBytes];
  uint64_t full[kRsWarps][2];
};
constexpr size_t kRsSmemBytes = sizeof(RsSmem);

// Rows this kernel takes: a broadcast weight row, a row of at most 16 KB that
// is a multiple of 16 bytes, 16-byte aligned operands.
__host__ __device__ __forceinline__ bool rms_scan_applies(uint64_t row_bytes, int64_t w_row_stride) {
  return w_row_stride == 0 && row_bytes > 0 && row_bytes <= kRsSlotBytes && row_bytes <= kRsWeightBytes &&
         row_bytes % 16 == 0;
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mul2(float a0, float a1, float b0, float b1, float& r0, float& r1) {
  uint64_t x, y, r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(x) : "f"(a0), "f"(a1));
  asm("mov.b64 %0, {%1, %2};" : "=l"(y) : "f"(b0), "f"(b1));
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(x), "l"(y));
  asm("mov.b64 {%0, %1}, %2;" : "=f"(r0), "=f"(r1) : "l"(r));
}

// This lane's 8 consecutive elements of chunk c (elements 256c + 8*lane ..)
// from a staged row at shared address `base`, widened to f32.
template <bool BF16>
__device__ __forceinline__ void rs_load8(uint32_t base, uint32_t c, uint32_t lane, float (&v)[8]) {
  if constexpr (BF16) {
    const uint4 q = lds_u4(base + c * 512 + lane * 16);
    const uint32_t w[4] = {q.x, q.y, q.z, q.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      v[2 * i] = __uint_as_float(w[i] << 16);
      v[2 * i + 1] = __uint_as_float(w[i] & 0xffff0000u);
    }
  } else {
    const uint4 q0 = lds_u4(base + c * 1024 + lane * 32);
    const uint4 q1 = lds_u4(base + c * 1024 + lane * 32 + 16);
    v[0] = __uint_as_float(q0.x); v[1] = __uint_as_float(q0.y); v[2] = __uint_as_float(q0.z); v[3] = __uint_as_float(q0.w);
    v[4] = __uint_as_float(q1.x); v[5] = __uint_as_float(q1.y); v[6] = __uint_as_float(q1.z); v[7] = __uint_as_float(q1.w);
  }
}

template <bool BF16, bool QUANT>
__device__ __forceinline__ void rms_norm_scan(const uint8_t* __restrict__ x, const uint8_t* __restrict__ w,
                                              uint64_t rows, uint32_t extent, float eps, uint8_t* __restrict__ y,
                                              tiler_cuda_status* st, int8_t* __restrict__ codes,
                                              float* __restrict__ scales) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  RsSmem& SS = *reinterpret_cast<RsSmem*>(smem_raw);
  const uint32_t warp = threadIdx.x / 32, lane = threadIdx.x & 31;
  constexpr uint32_t esize = BF16 ? 2 : 4;
  const uint32_t row_bytes = extent * esize;
  const uint32_t chunk_bytes = 256 * esize;
  const uint32_t nchunks = (extent + 255) / 256;
  // slot pitch: whole chunks, so a chunk's loads never leave the slot
  const uint32_t pitch = (row_bytes + chunk_bytes - 1) / chunk_bytes * chunk_bytes;
  const uint32_t nbuf = pitch * 2 <= kRsSlotBytes ? 2 : 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kRsWarps; ++i) { mbar_init(&SS.full[i][0], 1); mbar_init(&SS.full[i][1], 1); }
    fence_barrier_init();
  }
  for (uint32_t i = threadIdx.x; i < row_bytes / 16; i += blockDim.x)
    reinterpret_cast<uint4*>(SS.wrow)[i] = __ldg(reinterpret_cast<const uint4*>(w) + i);
  __syncthreads();

  // the weight row has no NaN / infinity: then y = w * (x * s) needs no NaN
  // check for rows whose x and s are finite
  bool w_finite = true;
  for (uint32_t i = lane; i < extent; i += 32) {
    const float wv = BF16 ? bf16_to_f32(reinterpret_cast<const uint16_t*>(SS.wrow)[i])
                          : reinterpret_cast<const float*>(SS.wrow)[i];
    w_finite &= isfinite(wv);
  }
  w_finite = __all_sync(0xffffffffu, w_finite);

  const uint64_t gw = (uint64_t)blockIdx.x * kRsWarps + warp, G = (uint64_t)gridDim.x * kRsWarps;
  if (gw >= rows) return;
  const uint64_t nmine = (rows - gw + G - 1) / G;
  const uint64_t keep = policy_evict_first();
  uint8_t* slot = SS.slot[warp];
  auto issue = [&](uint64_t k) {  // lane 0: row k of this warp into slot k % nbuf
    const uint32_t b = (uint32_t)(k % nbuf);
    mbar_arrive_expect_tx(&SS.full[warp][b], row_bytes);
    bulk_g2s(slot + b * pitch, x + (gw + k * G) * row_bytes, row_bytes, &SS.full[warp][b], keep);
  };
  if (lane == 0)
    for (uint64_t k = 0; k < nbuf && k < nmine; ++k) issue(k);
  const uint32_t wbase = smem_u32(SS.wrow);
  const bool y_wide = ((uintptr_t)y % 32 == 0) && row_bytes % 32 == 0;
  const bool codes8 = ((uintptr_t)codes % 8 == 0) && extent % 8 == 0;

  for (uint64_t k = 0; k < nmine; ++k) {
    const uint64_t row = gw + k * G;
    const uint32_t b = (uint32_t)(k % nbuf);
    if (!mbar_wait(&SS.full[warp][b], (uint32_t)((k / nbuf) & 1), st)) return;  // timeout recorded
    const uint32_t base = smem_u32(slot + b * pitch);

    // ---- the strict fold of the squares -------------------------------------
    NonnegFold F = fold_start(TILER_RS_SERIAL);
    float vn[8];  // the next chunk, loaded a chunk ahead
    rs_load8<BF16>(base, 0, lane, vn);
    for (uint32_t c = 0; c < nchunks; ++c) {
      float v[8], a[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) v[i] = vn[i];
      if (c + 1 < nchunks) rs_load8<BF16>(base, c + 1, lane, vn);
      const bool tail = (c + 1) * 256 > extent;
#pragma unroll
      for (int i = 0; i < 8; i += 2) mul2(v[i], v[i + 1], v[i], v[i + 1], a[i], a[i + 1]);
      if (tail) {
#pragma unroll
        for (int i = 0; i < 8; ++i)
          if (c * 256 + 8 * lane + i >= extent) a[i] = 0.0f;  // past the row's end
      }
      fold_chunk(F, a, lane);
    }
    const float total = fold_value(F);
    const float mean = __fdiv_rn(total, (float)extent);
    const float s = rsqrt_cr(__fadd_rn(mean, eps));
    // A finite total means every square, so every x, is finite; then with w
    // finite, x * s finite and w * (x * s) free of 0 * inf: no NaN can arise.
    const bool plain = w_finite && isfinite(total) && isfinite(s);

    if constexpr (!QUANT) {
      // ---- y = w * (x * s) ------------------------------------------------------
      uint8_t* yr = y + row * row_bytes;
      float vn[8], wn[8];  // the next chunk of x and w, loaded a chunk ahead
      rs_load8<BF16>(base, 0, lane, vn);
      rs_load8<BF16>(wbase, 0, lane, wn);
      for (uint32_t c = 0; c < nchunks; ++c) {
        float v[8], wv[8], o[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          v[i] = vn[i];
          wv[i] = wn[i];
        }
        if (c + 1 < nchunks) {
          rs_load8<BF16>(base, c + 1, lane, vn);
          rs_load8<BF16>(wbase, c + 1, lane, wn);
        }
        if (c * 256 + 8 * lane >= extent) continue;  // lanes past a short row's end
#pragma unroll
        for (int i = 0; i < 8; i += 2) {
          float t0, t1;
          mul2(v[i], v[i + 1], s, s, t0, t1);
          mul2(wv[i], wv[i + 1], t0, t1, o[i], o[i + 1]);
        }
        if (!plain) {
#pragma unroll
          for (int i = 0; i < 8; ++i) o[i] = canon(o[i]);
        }
        const uint32_t off = c * chunk_bytes + lane * 8 * esize;
        if constexpr (BF16) {
          // 16-byte rows hold a multiple of 8 bf16 elements: all 8 are inside the row
          st_global_stream_u4(reinterpret_cast<uint4*>(yr + off), RmsElem<true>::pack(o));
        } else {
          const uint32_t left = extent - (c * 256 + 8 * lane);  // this lane's elements inside the row
          const uint4 q0 = make_uint4(__float_as_uint(o[0]), __float_as_uint(o[1]), __float_as_uint(o[2]),
                                      __float_as_uint(o[3]));
          const uint4 q1 = make_uint4(__float_as_uint(o[4]), __float_as_uint(o[5]), __float_as_uint(o[6]),
                                      __float_as_uint(o[7]));
          if (left >= 8 && y_wide) {
            st_v8_stream(yr + off, q0, q1);
          } else {  // 16-byte rows: left is 4 or a multiple of 8
            st_global_stream_u4(reinterpret_cast<uint4*>(yr + off), q0);
            if (left >= 8) st_global_stream_u4(reinterpret_cast<uint4*>(yr + off + 16), q1);
          }
        }
      }
    } else {
      // ---- fused per-row int8 quantize of y (quantization.rs:188-247, :404-430,
      // per-row scale max|y| / 127): max over the magnitude bits, then the codes
      uint32_t mb = 0;
      for (uint32_t c = 0; c < nchunks; ++c) {
        float v[8], wv[8];
        rs_load8<BF16>(base, c, lane, v);
        rs_load8<BF16>(wbase, c, lane, wv);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          if (c * 256 + 8 * lane + i < extent)
            mb = max(mb, __float_as_uint(__fmul_rn(wv[i], __fmul_rn(v[i], s))) & 0x7fffffffu);
        }
      }
      mb = __reduce_max_sync(0xffffffffu, mb);
      if (mb > 0x7f800000u) {  // a NaN y: report its first column
        uint32_t first = 0xffffffffu;
        for (uint32_t c = 0; c < nchunks; ++c) {
          float v[8], wv[8];
          rs_load8<BF16>(base, c, lane, v);
          rs_load8<BF16>(wbase, c, lane, wv);
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const uint32_t col = c * 256 + 8 * lane + i;
            if (col < extent && isnan(__fmul_rn(wv[i], __fmul_rn(v[i], s)))) first = min(first, col);
          }
        }
        first = __reduce_min_sync(0xffffffffu, first);
        if (lane == 0) report_error(st, row * extent + first, TILER_CUDA_NAN_INPUT);
      } else {
        const float scale = __fdiv_rn(__uint_as_float(mb), 127.0f);
        if (lane == 0) scales[row] = scale;
        if (!is_positive_normal(scale)) {
          if (lane == 0) report_error(st, row * extent, TILER_CUDA_SCALE_DOMAIN);
        } else {
          const float inv = __frcp_rn(scale);
          int8_t* crow = codes + row * extent;
          for (uint32_t c = 0; c < nchunks; ++c) {
            if (c * 256 + 8 * lane >= extent) continue;
            float v[8], wv[8];
            rs_load8<BF16>(base, c, lane, v);
            rs_load8<BF16>(wbase, c, lane, wv);
            int q[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) q[i] = code_of_bounded(__fmul_rn(wv[i], __fmul_rn(v[i], s)), scale, inv);
            uint32_t hi, lo, packed0, packed1;  // cvt.pack d, a, b, c: d = c << 16 | sat8(a) << 8 | sat8(b)
            asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, 0;" : "=r"(hi) : "r"(q[3]), "r"(q[2]));
            asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(packed0) : "r"(q[1]), "r"(q[0]), "r"(hi));
            asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, 0;" : "=r"(lo) : "r"(q[7]), "r"(q[6]));
            asm("cvt.pack.sat.s8.s32.b32 %0, %1, %2, %3;" : "=r"(packed1) : "r"(q[5]), "r"(q[4]), "r"(lo));
            const uint32_t col = c * 256 + 8 * lane;
            if (codes8) {
              asm volatile("st.global.cs.v2.u32 [%0], {%1, %2};" ::"l"(crow + col), "r"(packed0), "r"(packed1)
                           : "memory");
            } else {  // extent % 4 == 0: 4-byte stores, the second only inside the row
              __stcs(reinterpret_cast<int*>(crow + col), (int)packed0);
              if (extent - col >= 8) __stcs(reinterpret_cast<int*>(crow + col + 4), (int)packed1);
            }
          }
        }
      }
    }

    // the slot is refilled only after every lane's reads of this row
    __syncwarp();
    if (lane == 0 && k + nbuf < nmine) {
      fence_proxy_async_smem();
      issue(k + nbuf);
    }
  }
}

}  // namespace tc

#define TILER_RS_PARAMS                                                                                 \
  const uint8_t *__restrict__ x, const uint8_t *__restrict__ w, uint64_t rows, uint32_t extent, float eps,     \
      uint8_t *__restrict__ y, tiler_cuda_status *st, int8_t *__restrict__ codes, float *__restrict__ scales
extern "C" __global__ void __launch_bounds__(tc::kRsThreads, 1) tiler_rms_norm_f32(TILER_RS_PARAMS) {
  tc::grid_dependency_wait();
  tc::rms_norm_scan<false, false>(x, w, rows, extent, eps, y, st, codes, scales);
}
extern "C" __global__ void __launch_bounds__(tc::kRsThreads, 1) tiler_rms_norm_bf16(TILER_RS_PARAMS) {
  tc::grid_dependency_wait();
  tc::rms_norm_scan<true, false>(x, w, rows, extent, eps, y, st, codes, scales);
}
extern "C" __global__ void __launch_bounds__(tc::kRsThreads, 1) tiler_rms_norm_quantize_i8(TILER_RS_PARAMS) {
  tc::grid_dependency_wait();
  tc::rms_norm_scan<false, true>(x, w, rows, extent, eps, y, st, codes, scales);
}
#undef TILER_RS_PARAMS

namespace tc {

bool rms_scan_launch(int bf16, int quant, const void* x, const void* w, int64_t w_row_stride, uint64_t rows,
                     uint64_t extent, float eps, void* y, int8_t* codes, float* scales, tiler_cuda_status* st,
                     int sm_count, cudaStream_t stream) {
  const uint64_t row_bytes = extent * (bf16 ? 2 : 4);
  if (!rms_scan_applies(row_bytes, w_row_stride)) return false;
  if ((uintptr_t)x % 16 || (uintptr_t)w % 16 || (!quant && (uintptr_t)y % 16) || (quant && (uintptr_t)codes % 4))
    return false;
  const unsigned grid = (unsigned)umin64((uint64_t)sm_count, (rows + kRsWarps - 1) / kRsWarps);
  const void* fn = quant ? (const void*)tiler_rms_norm_quantize_i8
                         : bf16 ? (const void*)tiler_rms_norm_bf16 : (const void*)tiler_rms_norm_f32;
  const char* name = quant ? "tiler_rms_norm_quantize_i8" : bf16 ? "tiler_rms_norm_bf16" : "tiler_rms_norm_f32";
  cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kRsSmemBytes);
  launch_kernel(fn, name, dim3(grid), dim3(kRsThreads), kRsSmemBytes, stream, (const uint8_t*)x, (const uint8_t*)w,
                rows, (uint32_t)extent, eps, (uint8_t*)y, st, codes, scales);
  return true;
}

}  // namespace tc
