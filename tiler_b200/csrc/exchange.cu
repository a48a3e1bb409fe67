// The multi-GPU sum's exchange step: every rank's partial sums go to every
// rank over NVLink (peer stores into each rank's exchange buffer), and each
// rank folds the W partials strictly in rank order -- the declared order of
// the multi-GPU grouping (partition r = rank r's shard; a
// strict_partitioned_sum over W partitions, evaluate.rs:749-832).  One kernel
// of one block per call replaces an NCCL all-gather plus a fold launch.
//
// Exchange buffer of each rank (caller-allocated, mapped into every rank):
//   flags  uint32 [2][kXchMaxRanks]   seq of the call that filled each slot
//   count  uint32 at byte 64           calls made on this rank (seq = 0 takes count + 1)
//   slots  float  [2][kXchMaxRanks][rows] from byte 128
// Calls alternate between the two halves by the parity of `seq` (the caller
// increments it by one per call, the same on every rank).  A rank reaches call
// n + 2 only after every rank has written call n + 1, which each did after
// reading call n, so a half is never rewritten while a peer still reads it.
// Every wait is bounded (about one second of %globaltimer); a wait that runs
// out records a timeout in the status word and leaves the result NaN.
#include "common.cuh"
#include "kernels.h"

namespace tc {

constexpr uint32_t kXchMaxRanks = 8;
constexpr uint64_t kXchWaitNs = 1000000000ull;

__host__ __device__ __forceinline__ uint64_t xch_slot_offset(uint32_t half, uint32_t q, uint64_t row, uint64_t rows) {
  return 128 + ((uint64_t)half * kXchMaxRanks + q) * rows * 4 + row * 4;
}

__device__ __forceinline__ void st_release_sys_u32(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys_u32(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// every rank's exchange buffer as mapped in this process, passed by value
struct XchBuffers {
  uint8_t* p[kXchMaxRanks];
};

__global__ void __launch_bounds__(256) sum_exchange_kernel(const float* __restrict__ partial, uint64_t rows,
                                                           uint32_t rank, uint32_t world, const XchBuffers bufs_in,
                                                           uint32_t seq, float* __restrict__ out,
                                                           tiler_cuda_status* st) {
  uint8_t* const* bufs = bufs_in.p;
  __shared__ int timed_out;
  __shared__ uint32_t call_seq;
  if (threadIdx.x == 0) {
    timed_out = 0;
    // seq 0: the call number kept in this rank's buffer, so that the same
    // launch (captured in a CUDA graph, say) serves every call
    uint32_t* count = reinterpret_cast<uint32_t*>(bufs[rank] + 64);
    call_seq = seq ? seq : *count + 1;
    *count = call_seq;
  }
  __syncthreads();
  seq = call_seq;
  const uint32_t half = seq & 1u;
  // 1. this rank's partials into slot `rank` of every rank's buffer
  for (uint64_t r = threadIdx.x; r < rows; r += blockDim.x) {
    const float v = partial[r];
    for (uint32_t q = 0; q < world; ++q)
      *reinterpret_cast<float*>(bufs[q] + xch_slot_offset(half, rank, r, rows)) = v;
  }
  __syncthreads();
  // 2. then the flag: the fence orders the block's slot stores before it
  if (threadIdx.x < world) {
    __threadfence_system();
    st_release_sys_u32(reinterpret_cast<uint32_t*>(bufs[threadIdx.x]) + half * kXchMaxRanks + rank, seq);
  }
  // 3. wait (bounded) for every rank's flag of this call in the local buffer
  if (threadIdx.x < world) {
    const uint32_t* flag = reinterpret_cast<const uint32_t*>(bufs[rank]) + half * kXchMaxRanks + threadIdx.x;
    if (ld_acquire_sys_u32(flag) != seq) {
      const uint64_t t0 = global_ns();
      for (uint32_t i = 1;; ++i) {
        if (ld_acquire_sys_u32(flag) == seq) break;
        if ((i & 63) == 0 && global_ns() - t0 > kXchWaitNs) {
          timed_out = 1;
          if (st) atomicAdd(&st->timeouts, 1u);
          break;
        }
      }
    }
  }
  __syncthreads();
  // 4. the strict fold of the W partials in rank order (seeded at rank 0's)
  const uint8_t* mine = bufs[rank];
  for (uint64_t r = threadIdx.x; r < rows; r += blockDim.x) {
    float acc = __ldcv(reinterpret_cast<const float*>(mine + xch_slot_offset(half, 0, r, rows)));
    for (uint32_t q = 1; q < world; ++q)
      acc = __fadd_rn(acc, __ldcv(reinterpret_cast<const float*>(mine + xch_slot_offset(half, q, r, rows))));
    out[r] = timed_out ? __uint_as_float(kCanonicalNan) : canon(acc);
  }
}

}  // namespace tc

extern "C" {

uint64_t tiler_cuda_sum_exchange_buffer_bytes(uint64_t rows) {
  return tc::xch_slot_offset(2, 0, 0, rows);
}

int32_t tiler_cuda_sum_f32_exchange(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* st,
                                    const float* partial, uint64_t rows, uint32_t rank, uint32_t world,
                                    void* const* buffers, uint32_t seq, float* out) {
  using namespace tc;
  CHECK_CTX(ctx);
  if (world == 0 || rank >= world || !buffers || !partial || !out) return TILER_CUDA_INVALID_APPLICATION;
  if (world > kXchMaxRanks) return TILER_CUDA_UNSUPPORTED;
  if (rows == 0) return TILER_CUDA_OK;
  if (rows > (1u << 20)) return TILER_CUDA_SHAPE_TOO_LARGE;
  XchBuffers ptrs{};
  for (uint32_t q = 0; q < world; ++q) {
    if (!buffers[q] || (uintptr_t)buffers[q] % 16) return TILER_CUDA_INVALID_APPLICATION;
    ptrs.p[q] = (uint8_t*)buffers[q];
  }
  sum_exchange_kernel<<<1, 256, 0, S(stream)>>>(partial, rows, rank, world, ptrs, seq, out, st);
  return last_error_status();
}

}  // extern "C"
