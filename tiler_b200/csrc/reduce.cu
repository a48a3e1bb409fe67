// Reduction families: the grouped fold (sum / governed maximum) under the
// backend's declared grouping, plus the reference-vocabulary groupings
// (strict serial, strict partitioned, cooperative) for drop-in parity.
//
// Declared grouping of the grouped fold (tiler_cuda_grouping, oracle
// oracle_grid_fold restates the same order):
//   level 1  exact contiguous partitions, one CTA each
//            (strict_partial_sums, crates/tiler-reference/src/evaluate.rs:612-832);
//   level 2  the ADR-0100 composition inside the CTA: block (r, g, l) owns the
//            k contributors at (r*T + g*32 + l)*k, folded strictly; an
//            ascending-mask XOR butterfly over the 32 lanes (result lane 0);
//            a strict fold over the G warp slots; round totals in ascending
//            order, round 0 peeled (docs/decisions/0100-...md decisions 1-5);
//            tail padding with the two-sided identity (-0.0 / -inf);
//   level 3  the last CTA of a row folds the partials: strictly (the second
//            pass of strict_partitioned_sum) or by a second composition.
// The data path reads each contributor once with 16-byte loads, all rounds'
// loads issued before the folds consume them.
#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

namespace tc {

template <int OP>
__device__ __forceinline__ float fold2(float a, float b) {
  if (OP == 0) return __fadd_rn(a, b);
  return maximum(a, b);
}

template <int OP>
__device__ __forceinline__ float identity_value() {
  return OP == 0 ? __uint_as_float(0x80000000u) : __uint_as_float(0xff800000u);
}

// Ascending-mask butterfly (docs/decisions/0094-...md decision 4).
template <int OP>
__device__ __forceinline__ float butterfly(float v) {
#pragma unroll
  for (int m = 1; m < 32; m <<= 1) v = fold2<OP>(v, __shfl_xor_sync(0xffffffffu, v, m));
  return v;
}

// Folds one sequence seq[0, n) under the composition (T = blockDim.x, k, R)
// and returns the result in thread 0 (unCanonicalized).  `slots` is
// shared scratch of R*G floats plus R floats.  All threads must call it.
#ifndef TILER_SUM_CHUNK_ROUNDS
#define TILER_SUM_CHUNK_ROUNDS 4
#endif

template <int OP, int K>
__device__ float compose_block(const float* __restrict__ seq, uint64_t n, uint32_t R, float* slots,
                               bool vec_ok) {
  const uint32_t T = blockDim.x, G = T >> 5, tid = threadIdx.x;
  const uint32_t warp = tid >> 5, lane = tid & 31;
  const float ident = identity_value<OP>();
  // Software-pipelined in chunks of CH rounds: the loads of chunk c + 1 are
  // issued before the folds of chunk c, so no chunk waits on a full memory
  // latency after the previous one's arithmetic.
  constexpr uint32_t CH = TILER_SUM_CHUNK_ROUNDS;
  auto load_chunk = [&](uint32_t r0, float (&vals)[CH][K]) {
#pragma unroll
    for (uint32_t c = 0; c < CH; ++c) {
      const uint64_t base = ((uint64_t)(r0 + c) * T + tid) * K;
      if constexpr (K == 4) {
        if (r0 + c < R && base + K <= n && vec_ok) {
          const float4 v = __ldcs(reinterpret_cast<const float4*>(seq + base));
          vals[c][0] = v.x; vals[c][1] = v.y; vals[c][2] = v.z; vals[c][3] = v.w;
          continue;
        }
      }
#pragma unroll
      for (int i = 0; i < K; ++i) vals[c][i] = (r0 + c < R && base + i < n) ? __ldcs(seq + base + i) : ident;
    }
  };
  auto fold_chunk = [&](uint32_t r0, const float (&vals)[CH][K]) {
#pragma unroll
    for (uint32_t c = 0; c < CH; ++c) {
      if (r0 + c >= R) break;
      float v = vals[c][0];
#pragma unroll
      for (int i = 1; i < K; ++i) v = fold2<OP>(v, vals[c][i]);
      v = butterfly<OP>(v);
      if (lane == 0) slots[(r0 + c) * G + warp] = v;
    }
  };
  float cur[CH][K], nxt[CH][K];
  load_chunk(0, cur);
  for (uint32_t r0 = 0; r0 < R; r0 += CH) {
    if (r0 + CH < R) load_chunk(r0 + CH, nxt);
    fold_chunk(r0, cur);
#pragma unroll
    for (uint32_t c = 0; c < CH; ++c)
#pragma unroll
      for (int i = 0; i < K; ++i) cur[c][i] = nxt[c][i];
  }
  __syncthreads();
  float* staged = slots + R * G;
  for (uint32_t r = tid; r < R; r += T) {
    float s = slots[r * G];
    for (uint32_t g = 1; g < G; ++g) s = fold2<OP>(s, slots[r * G + g]);
    staged[r] = s;
  }
  __syncthreads();
  float total = 0.0f;
  if (tid == 0) {
    total = staged[0];
    for (uint32_t r = 1; r < R; ++r) total = fold2<OP>(total, staged[r]);
  }
  __syncthreads();  // slots may be reused by the caller
  return total;
}

// Runtime-k variant for the level-3 combine and small partitions.
template <int OP>
__device__ float compose_block_generic(const float* seq, uint64_t n, uint32_t T, uint32_t k, uint32_t R,
                                       float* slots, bool use_cg) {
  const uint32_t G = T >> 5, tid = threadIdx.x;
  const uint32_t warp = tid >> 5, lane = tid & 31;
  const float ident = identity_value<OP>();
  if (tid < T) {
    for (uint32_t r = 0; r < R; ++r) {
      uint64_t base = ((uint64_t)r * T + tid) * k;
      float v = ident;
      for (uint32_t i = 0; i < k; ++i) {
        float c = base + i < n ? (use_cg ? __ldcg(seq + base + i) : seq[base + i]) : ident;
        v = i == 0 ? c : fold2<OP>(v, c);
      }
      v = butterfly<OP>(v);
      if (lane == 0) slots[r * G + warp] = v;
    }
  }
  __syncthreads();
  float* staged = slots + R * G;
  for (uint32_t r = tid; r < R; r += blockDim.x) {
    float s = slots[r * G];
    for (uint32_t g = 1; g < G; ++g) s = fold2<OP>(s, slots[r * G + g]);
    staged[r] = s;
  }
  __syncthreads();
  float total = 0.0f;
  if (tid == 0) {
    total = staged[0];
    for (uint32_t r = 1; r < R; ++r) total = fold2<OP>(total, staged[r]);
  }
  __syncthreads();
  return total;
}

template <int OP, int K>
__device__ __forceinline__ void grouped_fold(const float* __restrict__ x, uint64_t count, GroupedParams gp,
                                             float* __restrict__ partials, unsigned int* __restrict__ tickets,
                                             float* __restrict__ out) {
  extern __shared__ float slots[];
  const uint64_t P = gp.partitions;
  const uint64_t row = blockIdx.x / P, p = blockIdx.x % P;
  const uint64_t per = count / P;
  const float* seq = x + row * count + p * per;
  const bool vec_ok = ((reinterpret_cast<uintptr_t>(seq) & 15u) == 0);
  float partial = compose_block<OP, K>(seq, per, gp.rounds, slots, vec_ok);
  if (P == 1) {
    if (threadIdx.x == 0) out[row] = canon(partial);
    return;
  }
  __shared__ unsigned int is_last;
  if (threadIdx.x == 0) {
    partials[row * P + p] = partial;
    __threadfence();
    unsigned int ticket = atomicAdd(&tickets[row], 1u);
    is_last = (ticket == P - 1);
  }
  __syncthreads();
  if (!is_last) return;
  __threadfence();
  const float* pr = partials + row * P;
  float total;
  if (gp.combine_threads == 0) {
    total = 0.0f;
    if (threadIdx.x == 0) {
      total = __ldcg(pr);
      for (uint64_t i = 1; i < P; ++i) total = fold2<OP>(total, __ldcg(pr + i));
    }
  } else {
    total = compose_block_generic<OP>(pr, P, gp.combine_threads, gp.combine_k, gp.combine_rounds, slots, true);
  }
  if (threadIdx.x == 0) {
    out[row] = canon(total);
    tickets[row] = 0;  // leaves the workspace ready for the next launch
  }
}

}  // namespace tc

#define TILER_GROUPED_KERNEL(NAME, OP, K)                                                                   \
  extern "C" __global__ void __launch_bounds__(1024)                                                       \
      NAME(const float* __restrict__ x, uint64_t count, tc::GroupedParams gp, float* __restrict__ partials, \
           unsigned int* __restrict__ tickets, float* __restrict__ out) {                                  \
    tc::grid_dependency_wait();                                                                            \
    tc::grouped_fold<OP, K>(x, count, gp, partials, tickets, out);                                         \
  }
TILER_GROUPED_KERNEL(tiler_grouped_sum_k1, 0, 1)
TILER_GROUPED_KERNEL(tiler_grouped_sum_k2, 0, 2)
TILER_GROUPED_KERNEL(tiler_grouped_sum_k4, 0, 4)
TILER_GROUPED_KERNEL(tiler_grouped_max_k1, 1, 1)
TILER_GROUPED_KERNEL(tiler_grouped_max_k2, 1, 2)
TILER_GROUPED_KERNEL(tiler_grouped_max_k4, 1, 4)
#undef TILER_GROUPED_KERNEL

namespace tc {

void launch_grouped_fold(int op, const float* x, uint64_t rows, uint64_t count, const GroupedParams& gp,
                         float* partials, unsigned int* tickets, float* out, cudaStream_t stream) {
  const uint32_t G = gp.threads / 32;
  uint32_t R = gp.rounds;
  uint32_t cR = gp.combine_threads ? gp.combine_rounds : 0;
  uint32_t cG = gp.combine_threads / 32;
  size_t smem = sizeof(float) * (size_t)std::max<uint64_t>((uint64_t)R * G + R, (uint64_t)cR * cG + cR);
  dim3 grid((unsigned)(rows * gp.partitions));
  const int ki = gp.k == 4 ? 2 : gp.k == 2 ? 1 : 0;
  static const void* const fns[2][3] = {{(const void*)tiler_grouped_sum_k1, (const void*)tiler_grouped_sum_k2,
                                         (const void*)tiler_grouped_sum_k4},
                                        {(const void*)tiler_grouped_max_k1, (const void*)tiler_grouped_max_k2,
                                         (const void*)tiler_grouped_max_k4}};
  static const char* const names[2][3] = {{"tiler_grouped_sum_k1", "tiler_grouped_sum_k2", "tiler_grouped_sum_k4"},
                                          {"tiler_grouped_max_k1", "tiler_grouped_max_k2", "tiler_grouped_max_k4"}};
  launch_kernel(fns[op][ki], names[op][ki], grid, dim3(gp.threads), smem, stream, x, count, gp, partials, tickets,
                out);
}

// ---- reference-vocabulary groupings ------------------------------------------

// A strict left fold of s[0..n) seeded at s[0] (n >= 1), by one warp: each
// 32-element batch is loaded coalesced (lane j holds element j) and folded in
// order by broadcasting lane j's value at step j, every lane carrying the
// same accumulator.  kFoldAhead batches are loaded ahead of the one being
// folded, so the chain of dependent adds, not the load latency, sets the
// pace.  The result is returned in every lane.
constexpr int kFoldAhead = 8;
__device__ __forceinline__ float warp_serial_fold(const float* __restrict__ s, uint64_t n, uint32_t lane) {
  const uint64_t nb = (n + 31) / 32;
  float pf[kFoldAhead];
#pragma unroll
  for (int d = 0; d < kFoldAhead; ++d) {
    const uint64_t idx = (uint64_t)d * 32 + lane;
    pf[d] = idx < n ? __ldcg(s + idx) : 0.0f;
  }
  float acc = __shfl_sync(0xffffffffu, pf[0], 0);
  for (uint64_t b0 = 0; b0 < nb; b0 += kFoldAhead) {
#pragma unroll
    for (int d = 0; d < kFoldAhead; ++d) {
      const uint64_t b = b0 + d;
      const float v = pf[d];
      const uint64_t nidx = (b + kFoldAhead) * 32 + lane;
      pf[d] = nidx < n ? __ldcg(s + nidx) : 0.0f;
      if (b < nb) {
        const uint32_t first = b == 0 ? 1u : 0u;  // element 0 seeds the fold
        const uint32_t m = (uint32_t)umin64(32, n - b * 32);
        if (first == 0 && m == 32) {
#pragma unroll
          for (int j = 0; j < 32; ++j) acc = __fadd_rn(acc, __shfl_sync(0xffffffffu, v, j));
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            const float e = __shfl_sync(0xffffffffu, v, j);
            if ((uint32_t)j >= first && (uint32_t)j < m) acc = __fadd_rn(acc, e);
          }
        }
      }
    }
  }
  return acc;
}

// A thread's strict left fold of s[0..n) seeded at s[0] (n >= 1), for short
// folds where a warp per fold would leave most lanes idle.
__device__ __forceinline__ float thread_serial_fold(const float* __restrict__ s, uint64_t n) {
  float acc = s[0];
  for (uint64_t i = 1; i < n; ++i) acc = __fadd_rn(acc, s[i]);
  return acc;
}

constexpr int kSerialFoldThreads = 128;
// folds at least this long get a warp each (warp_serial_fold), shorter ones a
// thread each
constexpr uint64_t kWarpFoldMin = 256;

// One strict fold per unit u < units: unit u covers s = x + (u / per_row) *
// row_stride + (u % per_row) * len, len elements.  WARP selects a warp per
// unit, else a thread per unit.
template <bool WARP>
__global__ void __launch_bounds__(kSerialFoldThreads)
    serial_folds_kernel(const float* __restrict__ x, uint64_t units, uint64_t per_row, uint64_t row_stride,
                        uint64_t len, float* __restrict__ out) {
  const uint32_t lane = threadIdx.x & 31;
  const uint64_t u = WARP ? blockIdx.x * (uint64_t)(kSerialFoldThreads / 32) + (threadIdx.x >> 5)
                          : blockIdx.x * (uint64_t)kSerialFoldThreads + threadIdx.x;
  if (u >= units) return;
  if (len == 0) {
    if (!WARP || lane == 0) out[u] = 0.0f;
    return;
  }
  const float* s = x + (u / per_row) * row_stride + (u % per_row) * len;
  const float acc = WARP ? warp_serial_fold(s, len, lane) : thread_serial_fold(s, len);
  if (!WARP || lane == 0) out[u] = canon(acc);
}

static void launch_serial_folds(const float* x, uint64_t units, uint64_t per_row, uint64_t row_stride, uint64_t len,
                                float* out, cudaStream_t stream) {
  if (units == 0) return;
  if (len >= kWarpFoldMin) {
    const uint64_t per_block = kSerialFoldThreads / 32;
    serial_folds_kernel<true><<<(unsigned)((units + per_block - 1) / per_block), kSerialFoldThreads, 0, stream>>>(
        x, units, per_row, row_stride, len, out);
  } else {
    serial_folds_kernel<false><<<(unsigned)((units + kSerialFoldThreads - 1) / kSerialFoldThreads),
                                 kSerialFoldThreads, 0, stream>>>(x, units, per_row, row_stride, len, out);
  }
}

// strict_sum (evaluate.rs:498-589): one fold per row, in order.
void launch_strict_sum(const float* x, uint64_t rows, uint64_t count, float* out, cudaStream_t stream) {
  launch_serial_folds(x, rows, 1, count, count, out, stream);
}

// strict_partial_sums (evaluate.rs:612-747) then the strict fold of each row's
// partials (strict_partitioned_sum, :749-832).
void launch_partitioned_sum(const float* x, uint64_t rows, uint64_t count, uint64_t P, uint64_t per,
                            float* partials, float* out, cudaStream_t stream) {
  launch_serial_folds(x, rows * P, P, count, per, partials, stream);
  launch_strict_sum(partials, rows, P, out, stream);
}

// cooperative_grouped_sum / fold_cooperative_sequence (evaluate.rs:936-1158):
// one CTA per row; each round the participants' strict partials are staged in
// shared memory and folded in ascending participant order by one thread.
__global__ void cooperative_sum_kernel(const float* __restrict__ x, uint64_t count, uint64_t participants,
                                       uint64_t per, uint64_t rounds, int participant_major,
                                       float* __restrict__ out) {
  extern __shared__ float staged[];
  const float* s = x + blockIdx.x * count;
  float total = 0.0f;
  for (uint64_t r = 0; r < rounds; ++r) {
    for (uint64_t p = threadIdx.x; p < participants; p += blockDim.x) {
      uint64_t cell = participant_major ? p * rounds + r : r * participants + p;
      const float* c = s + cell * per;
      float partial = c[0];
      for (uint64_t i = 1; i < per; ++i) partial = __fadd_rn(partial, c[i]);
      staged[p] = partial;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
      float st = staged[0];
      for (uint64_t p = 1; p < participants; ++p) st = __fadd_rn(st, staged[p]);
      total = r == 0 ? st : __fadd_rn(total, st);
    }
    __syncthreads();
  }
  if (threadIdx.x == 0) out[blockIdx.x] = canon(total);
}

void launch_cooperative_sum(const float* x, uint64_t rows, uint64_t count, uint64_t participants, uint64_t per,
                            uint64_t rounds, int participant_major, float* out, cudaStream_t stream) {
  unsigned threads = (unsigned)std::min<uint64_t>(participants, 1024);
  threads = std::max(32u, (threads + 31) / 32 * 32);
  size_t smem = participants * sizeof(float);
  cooperative_sum_kernel<<<(unsigned)rows, threads, smem, stream>>>(x, count, participants, per, rounds,
                                                                   participant_major, out);
}

}  // namespace tc
