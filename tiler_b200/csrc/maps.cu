// Elementwise maps (SiLU, scale-bias), the row gather, the reference's own
// per-tensor unsigned strict-affine quantize / decode, and the status-word
// reset.  All are grid-stride kernels sized to a multiple of the SM count,
// with 16-byte vector access where the pointers allow.
#include "common.cuh"
#include "kernels.h"

namespace tc {

__global__ void status_reset_kernel(tiler_cuda_status* st) {
  st->error_key = ~0ull;
  st->value_key = ~0ull;
  st->undecided = 0;
  st->timeouts = 0;
  st->reserved = 0;
}

void launch_status_reset(tiler_cuda_status* st, cudaStream_t stream) { status_reset_kernel<<<1, 1, 0, stream>>>(st); }

// The bounded wait every kernel uses, made to run out: an mbarrier phase that
// nothing completes (one expected arrival, none made), waited on with a short
// limit.  The wait gives up, counts a timeout in the status word and the
// kernel returns; nothing is in flight, so the context stays usable.
__global__ void bounded_wait_selftest_kernel(tiler_cuda_status* st, uint64_t limit_ns) {
  __shared__ uint64_t bar;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    fence_barrier_init();
  }
  __syncthreads();
  if (threadIdx.x == 0) (void)mbar_wait(&bar, 0, st, limit_ns);
}

void launch_bounded_wait_selftest(tiler_cuda_status* st, uint64_t limit_ns, cudaStream_t stream) {
  bounded_wait_selftest_kernel<<<1, 32, 0, stream>>>(st, limit_ns);
}

// silu_cr out of line, so the rare flagged arguments cost the common path no
// registers
__device__ __noinline__ float silu_cr_outlined(float x, const double* table, tiler_cuda_status* st) {
  return silu_cr(x, table, st);
}

// SiLU of four values: for 2^-60 <= |x| < 87, where exp(-x) is a normal
// binary32 value below 2^126 and x / d clear of the subnormal range, the
// certified exp and Markstein's division run branch-free; a lane holding any
// other value (out of range, NaN, an exp near a rounding midpoint) redoes its
// four values with silu_cr, the exact path, in one warp-uniform branch.
struct SiluOp {
  const double* table;
  tiler_cuda_status* st;
  __device__ __forceinline__ float4 operator()(float4 q) const {
    const float xs[4] = {q.x, q.y, q.z, q.w};
    float r[4];
    bool all_ok = true;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      bool ok;
      const float e = __uint_as_float(exp_cr_bits<true>(-xs[i], table, &ok));
      r[i] = div_rn_markstein(xs[i], __fadd_rn(1.0f, e));
      // 2^-60 <= |x| < 87 (0x21800000 and 0x42ae0000 as magnitude bits; NaN above)
      all_ok = all_ok && ok && ((__float_as_uint(xs[i]) & 0x7fffffffu) - 0x21800000u) < 0x212e0000u;
    }
    if (__any_sync(__activemask(), !all_ok) && !all_ok) {
#pragma unroll
      for (int i = 0; i < 4; ++i) r[i] = silu_cr_outlined(xs[i], table, st);
    }
    return make_float4(r[0], r[1], r[2], r[3]);
  }
  __device__ __forceinline__ float operator()(float x) const { return silu_cr(x, table, st); }
};

// multiply-f32 then add-f32, two roundings (standard.rs:105-120,
// evaluate.rs:448-485), NaN canonicalized after each operation.
__device__ __forceinline__ float scale_bias1(float x, float a, float b) {
  return canon(__fadd_rn(canon(__fmul_rn(x, a)), b));
}

struct ScaleBiasOp {
  float a, b;
  __device__ __forceinline__ float4 operator()(float4 q) const {
    return make_float4(scale_bias1(q.x, a, b), scale_bias1(q.y, a, b), scale_bias1(q.z, a, b),
                       scale_bias1(q.w, a, b));
  }
  __device__ __forceinline__ float operator()(float x) const { return scale_bias1(x, a, b); }
};

// Staged elementwise map over a flat f32 array whose input and output are
// 16-byte aligned.  A persistent CTA walks tiles of kMapTile floats with a
// ring of kMapStages shared-memory buffers: one bulk load per tile (issued
// kMapStages - 1 tiles ahead), the map applied in place, one bulk store per
// tile.  The reads in flight are the copy engine's, so they do not depend on
// the map's register footprint.  The last n % 4 elements are done by block 0
// with plain accesses.
constexpr int kMapThreads = 256;
// 16 KB tiles in a ring of 3: per thread four float4 per tile between the
// tile's barriers (8 KB tiles in a ring of 4 measured SiLU 59.8 us and
// scale-bias 46.1 us at [8192,4096], against 57.0 and 45.5 us)
constexpr uint32_t kMapTile = 4096;  // floats (16 KB)
constexpr uint32_t kMapStages = 3;
constexpr int kMapCtasPerSm = 6;
constexpr size_t kMapSmem = (size_t)kMapStages * kMapTile * 4 + kMapStages * 8;

template <class Op>
__device__ __forceinline__ void staged_map(const float* __restrict__ x, uint64_t n, float* __restrict__ y, Op op,
                                           float* buf, uint64_t* full, tiler_cuda_status* st) {
  __shared__ int abort_flag;
  const uint64_t n4 = n / 4 * 4;
  const uint64_t tiles = (n4 + kMapTile - 1) / kMapTile;
  const uint64_t pol = policy_evict_first();
  auto tile_floats = [&](uint64_t t) -> uint32_t {
    return (uint32_t)umin64(kMapTile, n4 - t * kMapTile);
  };
  auto issue = [&](uint64_t t, uint32_t b) {
    const uint32_t bytes = tile_floats(t) * 4;
    mbar_arrive_expect_tx(&full[b], bytes);
    bulk_g2s(buf + b * kMapTile, x + t * kMapTile, bytes, &full[b], pol);
  };
  if (threadIdx.x == 0) {
    for (uint32_t b = 0; b < kMapStages; ++b) mbar_init(&full[b], 1);
    abort_flag = 0;
    fence_barrier_init();
    for (uint32_t b = 0; b + 1 < kMapStages; ++b)
      if (blockIdx.x + (uint64_t)b * gridDim.x < tiles) issue(blockIdx.x + (uint64_t)b * gridDim.x, b);
  }
  __syncthreads();
  uint32_t k = 0;
  for (uint64_t t = blockIdx.x; t < tiles; t += gridDim.x, ++k) {
    const uint32_t b = k % kMapStages;
    if (!mbar_wait(&full[b], (k / kMapStages) & 1, st)) abort_flag = 1;
    __syncthreads();
    if (abort_flag) break;
    const uint32_t nf = tile_floats(t);
    float4* v = reinterpret_cast<float4*>(buf + b * kMapTile);
    if (nf == kMapTile) {
      // a full tile: a fixed number of vectors per thread, unrolled (SiLU
      // 56.5 -> 55.5 us at [8192,4096])
#pragma unroll
      for (uint32_t j = 0; j < kMapTile / 4 / kMapThreads; ++j)
        v[threadIdx.x + j * kMapThreads] = op(v[threadIdx.x + j * kMapThreads]);
    } else {
      for (uint32_t i = threadIdx.x; i < nf / 4; i += kMapThreads) v[i] = op(v[i]);
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncthreads();
    if (threadIdx.x == 0) {
      asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(y + t * kMapTile),
                   "r"(smem_u32(buf + b * kMapTile)), "r"(nf * 4)
                   : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
      // refill the buffer stored one tile ago once that store has read it
      // (this tile's store stays in flight)
      const uint64_t nt = t + (uint64_t)(kMapStages - 1) * gridDim.x;
      if (nt < tiles) {
        asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory");
        issue(nt, (k + kMapStages - 1) % kMapStages);
      }
    }
  }
  if (threadIdx.x == 0) {
    asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    // loads still in flight (abort) must land before shared memory is released
    if (abort_flag)
      for (uint32_t j = 0; j + 1 < kMapStages; ++j) {
        const uint32_t kk = k + j;
        if (blockIdx.x + (uint64_t)kk * gridDim.x < tiles)
          (void)mbar_wait(&full[kk % kMapStages], (kk / kMapStages) & 1, nullptr);
      }
  }
  if (blockIdx.x == 0)
    for (uint64_t i = n4 + threadIdx.x; i < n; i += kMapThreads) y[i] = op(x[i]);
}

// SiluF32Reference — silu.rs:78-110 (map) and :158-180 (scalar).
__global__ void __launch_bounds__(kMapThreads) silu_staged_kernel(const float* __restrict__ x, uint64_t n,
                                                                  float* __restrict__ y, tiler_cuda_status* st) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  __shared__ double table[256];
  load_exp_table(table);
  staged_map(x, n, y, SiluOp{table, st}, reinterpret_cast<float*>(smem_raw),
             reinterpret_cast<uint64_t*>(smem_raw + (size_t)kMapStages * kMapTile * 4), st);
}

__global__ void scale_bias_staged_kernel(const float* __restrict__ x, uint64_t n, const float* __restrict__ a,
                                         const float* __restrict__ b, float* __restrict__ y, tiler_cuda_status* st) {
  extern __shared__ __align__(128) uint8_t smem_raw[];
  staged_map(x, n, y, ScaleBiasOp{__ldg(a), __ldg(b)}, reinterpret_cast<float*>(smem_raw),
             reinterpret_cast<uint64_t*>(smem_raw + (size_t)kMapStages * kMapTile * 4), st);
}

template <class K>
static unsigned staged_map_grid(K kernel, uint64_t n, int sm_count) {
  cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kMapSmem);
  cudaFuncSetAttribute(kernel, cudaFuncAttributePreferredSharedMemoryCarveout, 100);
  int resident = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&resident, kernel, kMapThreads, kMapSmem) != cudaSuccess ||
      resident < 1)
    resident = 1;
  const uint64_t tiles = (n / 4 * 4 + kMapTile - 1) / kMapTile;
  return (unsigned)std::max<uint64_t>(1, umin64(tiles, (uint64_t)sm_count * std::min(resident, kMapCtasPerSm)));
}

// The unaligned form: grid-stride over single elements.
__global__ void silu_kernel(const float* __restrict__ x, uint64_t n, float* __restrict__ y, tiler_cuda_status* st) {
  __shared__ double table[256];
  load_exp_table(table);
  __syncthreads();
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += stride) y[i] = silu_cr(x[i], table, st);
}

void launch_silu(const float* x, uint64_t n, float* y, tiler_cuda_status* st, int sm_count, cudaStream_t stream) {
  if (n == 0) return;
  if ((uintptr_t)x % 16 == 0 && (uintptr_t)y % 16 == 0) {
    silu_staged_kernel<<<staged_map_grid(silu_staged_kernel, n, sm_count), kMapThreads, kMapSmem, stream>>>(x, n, y,
                                                                                                           st);
    return;
  }
  const uint64_t want = (n + 255) / 256;
  silu_kernel<<<(unsigned)std::min<uint64_t>(want, (uint64_t)sm_count * 8), 256, 0, stream>>>(x, n, y, st);
}

// The general form (tensor a / b, or unaligned): grid-stride, float4 where
// the pointers allow.
__global__ void scale_bias_kernel(const float* __restrict__ x, uint64_t n, const float* __restrict__ a, int a_scalar,
                                  const float* __restrict__ b, int b_scalar, float* __restrict__ y) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  const uint64_t tid = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x;
  const bool vec = ((uintptr_t)x % 16 == 0) && ((uintptr_t)y % 16 == 0) && (a_scalar || (uintptr_t)a % 16 == 0) &&
                   (b_scalar || (uintptr_t)b % 16 == 0);
  const float as = a_scalar ? __ldg(a) : 0.0f, bs = b_scalar ? __ldg(b) : 0.0f;
  uint64_t done = 0;
  if (vec) {
    const float4* x4 = reinterpret_cast<const float4*>(x);
    float4* y4 = reinterpret_cast<float4*>(y);
    const uint64_t nv = n / 4;
    for (uint64_t v = tid; v < nv; v += stride) {
      const float4 q = __ldcs(x4 + v);
      const float4 av = a_scalar ? make_float4(as, as, as, as) : __ldcs(reinterpret_cast<const float4*>(a) + v);
      const float4 bv = b_scalar ? make_float4(bs, bs, bs, bs) : __ldcs(reinterpret_cast<const float4*>(b) + v);
      st_global_stream(y4 + v, make_float4(scale_bias1(q.x, av.x, bv.x), scale_bias1(q.y, av.y, bv.y),
                                           scale_bias1(q.z, av.z, bv.z), scale_bias1(q.w, av.w, bv.w)));
    }
    done = n / 4 * 4;
  }
  for (uint64_t i = done + tid; i < n; i += stride)
    y[i] = scale_bias1(x[i], a_scalar ? as : a[i], b_scalar ? bs : b[i]);
}

void launch_scale_bias(const float* x, uint64_t n, const float* a, int a_scalar, const float* b, int b_scalar,
                       float* y, int sm_count, cudaStream_t stream) {
  if (n == 0) return;
  if (a_scalar && b_scalar && (uintptr_t)x % 16 == 0 && (uintptr_t)y % 16 == 0) {
    // the broadcast form through the staged map (a wait that runs out ends the
    // kernel early; this entry has no status word to report it in)
    scale_bias_staged_kernel<<<staged_map_grid(scale_bias_staged_kernel, n, sm_count), kMapThreads, kMapSmem,
                               stream>>>(x, n, a, b, y, nullptr);
    return;
  }
  const uint64_t want = (n / 4 + 255) / 256 + 1;
  scale_bias_kernel<<<(unsigned)std::min<uint64_t>(want, (uint64_t)sm_count * 8), 256, 0, stream>>>(
      x, n, a, a_scalar, b, b_scalar, y);
}

// GatherF32Reference (structural.rs:513-606): bit-exact row copies; an
// out-of-range id is reported with its position and value (the smallest
// position wins, as the reference refuses at the first one in order) and
// its row is not written.
__global__ void gather_rows_kernel(const uint8_t* __restrict__ table, uint64_t table_rows, uint64_t row_bytes,
                                   const void* __restrict__ ids, int ids_unsigned, uint64_t n_ids,
                                   uint8_t* __restrict__ out, tiler_cuda_status* st) {
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t warps = (uint64_t)gridDim.x * (blockDim.x / 32);
  const bool vec = (row_bytes % 16 == 0) && ((uintptr_t)table % 16 == 0) && ((uintptr_t)out % 16 == 0);
  for (uint64_t i = blockIdx.x * (uint64_t)(blockDim.x / 32) + threadIdx.x / 32; i < n_ids; i += warps) {
    int64_t v = ids_unsigned ? (int64_t)__ldg((const uint32_t*)ids + i) : (int64_t)__ldg((const int32_t*)ids + i);
    if (v < 0 || (uint64_t)v >= table_rows) {
      if (lane == 0) {
        report_error(st, i, TILER_CUDA_GATHER_INDEX_OUT_OF_BOUNDS);
        report_value(st, i, (uint32_t)v);
      }
      continue;
    }
    const uint8_t* src = table + (uint64_t)v * row_bytes;
    uint8_t* dst = out + i * row_bytes;
    if (vec) {
      const uint4* s4 = reinterpret_cast<const uint4*>(src);
      uint4* d4 = reinterpret_cast<uint4*>(dst);
      const uint64_t nv = row_bytes / 16;
      uint64_t k = lane;
      // 16 vectors per lane in flight (a whole 8 KB row per warp): 23.6 ->
      // 22.8 us for [8192] rows of bf16 [128256,4096] against 4 at a time
      for (; k + 32 * 15 < nv; k += 32 * 16) {
        uint4 a[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) a[j] = ld_global_nc_u4(s4 + k + 32 * j);
#pragma unroll
        for (int j = 0; j < 16; ++j) st_global_stream_u4(d4 + k + 32 * j, a[j]);
      }
      for (; k + 32 * 3 < nv; k += 32 * 4) {
        const uint4 a0 = ld_global_nc_u4(s4 + k), a1 = ld_global_nc_u4(s4 + k + 32);
        const uint4 a2 = ld_global_nc_u4(s4 + k + 64), a3 = ld_global_nc_u4(s4 + k + 96);
        st_global_stream_u4(d4 + k, a0);
        st_global_stream_u4(d4 + k + 32, a1);
        st_global_stream_u4(d4 + k + 64, a2);
        st_global_stream_u4(d4 + k + 96, a3);
      }
      for (; k < nv; k += 32) st_global_stream_u4(d4 + k, ld_global_nc_u4(s4 + k));
    } else {
      for (uint64_t k = lane; k < row_bytes; k += 32) dst[k] = src[k];
    }
  }
}

void launch_gather_rows(const void* table, uint64_t table_rows, uint64_t row_bytes, const void* ids,
                        int ids_unsigned, uint64_t n_ids, void* out, tiler_cuda_status* st, int sm_count,
                        cudaStream_t stream) {
  if (n_ids == 0 || row_bytes == 0) return;
  const unsigned wpb = 8;
  const uint64_t want = (n_ids + wpb - 1) / wpb;
  gather_rows_kernel<<<(unsigned)std::min<uint64_t>(want, (uint64_t)sm_count * 16), wpb * 32, 0, stream>>>(
      (const uint8_t*)table, table_rows, row_bytes, ids, ids_unsigned, n_ids, (uint8_t*)out, st);
}

// quantize_one / dequantize_one — quantization.rs:404-451 (per-tensor scale,
// unsigned codes, maximum 15 or 255).
__global__ void quantize_affine_u8_kernel(const float* __restrict__ x, uint64_t n, float scale, uint32_t zp,
                                          uint32_t maximum, uint8_t* __restrict__ codes, tiler_cuda_status* st) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    const float v = x[i];
    if (isnan(v)) {
      report_error(st, i, TILER_CUDA_NAN_INPUT);
      continue;
    }
    const float s = __fdiv_rn(v, scale);
    const float t = __fadd_rn(s, (float)zp);
    const float c = fminf(fmaxf(t, 0.0f), (float)maximum);
    codes[i] = (uint8_t)__float2uint_rn(c);
  }
}

__global__ void dequantize_affine_u8_kernel(const uint8_t* __restrict__ codes, uint64_t n, float scale, uint32_t zp,
                                            uint32_t maximum, float* __restrict__ y, tiler_cuda_status* st) {
  const uint64_t stride = (uint64_t)gridDim.x * blockDim.x;
  for (uint64_t i = blockIdx.x * (uint64_t)blockDim.x + threadIdx.x; i < n; i += stride) {
    const uint32_t c = codes[i];
    if (c > maximum) {  // the code domain check of dense_code_bytes (quantization.rs:308-327)
      report_error(st, i, TILER_CUDA_INVALID_APPLICATION);
      continue;
    }
    y[i] = c == zp ? 0.0f : __fmul_rn((float)((int32_t)c - (int32_t)zp), scale);
  }
}

void launch_quantize_affine_u8(const float* x, uint64_t n, float scale, uint32_t zp, uint32_t maximum,
                               uint8_t* codes, tiler_cuda_status* st, int sm_count, cudaStream_t stream) {
  if (n == 0) return;
  quantize_affine_u8_kernel<<<(unsigned)std::min<uint64_t>((n + 255) / 256, (uint64_t)sm_count * 8), 256, 0,
                              stream>>>(x, n, scale, zp, maximum, codes, st);
}

void launch_dequantize_affine_u8(const uint8_t* codes, uint64_t n, float scale, uint32_t zp, uint32_t maximum,
                                 float* y, tiler_cuda_status* st, int sm_count, cudaStream_t stream) {
  if (n == 0) return;
  dequantize_affine_u8_kernel<<<(unsigned)std::min<uint64_t>((n + 255) / 256, (uint64_t)sm_count * 8), 256, 0,
                                stream>>>(codes, n, scale, zp, maximum, y, st);
}

}  // namespace tc
