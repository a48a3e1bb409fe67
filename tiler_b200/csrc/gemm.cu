// Contraction family.
//
//  * contract_f32: the reference-exact `td,od->to` f32 contraction
//    (contraction.rs:558-630): every output is a strict fold over k in
//    ascending order, seeded at the first product, product and sum rounded
//    separately.  16x16 output tiles stage 32-wide k slabs of A and B in
//    shared memory; each thread still folds its own output in k order.
//
//  * gemm_bf16: the config's bf16 contraction on the 5th-generation tensor
//    cores.  A persistent kernel, one CTA per SM, 128x256 output tiles:
//      warp 0     TMA producer: 128x64 A and 256x64 B bf16 boxes, 128-byte
//                 swizzle, into a 4-stage shared-memory ring (no multicast);
//      warp 1     allocates 512 TMEM columns (two 128x256 f32 accumulators)
//                 and one lane issues tcgen05.mma (kind::f16, M=128, N=256,
//                 K=16) and tcgen05.commit back to the ring / accumulators;
//      warps 2-9  epilogue (two per TMEM lane quarter, half the columns each):
//                 tcgen05.ld 32 columns at a time, the SiLU of
//                 silu.rs:158-180 (hardware exp/divide with a certified
//                 fallback for the rare values near a bf16 rounding
//                 boundary, one warp-uniform branch), RNE to bf16, into a
//                 32x64 swizzled shared-memory box that one TMA store writes
//                 to C; accumulator b of tile i+1 fills while tile i drains.
//    Every mbarrier wait is bounded; a wait that gives up records a timeout
//    in the status word and the CTA stops, frees its TMEM and returns.
#include "common.cuh"
#include "tmap.cuh"
#include "kernels.h"

namespace tc {

// ---------------------------------------------------------------------------
// Strict f32 contraction
// ---------------------------------------------------------------------------
__global__ void contract_f32_kernel(const float* __restrict__ a, const float* __restrict__ b, uint64_t m,
                                    uint64_t n, uint64_t k, float* __restrict__ c) {
  __shared__ float As[16][33], Bs[16][33];
  const uint32_t tx = threadIdx.x, ty = threadIdx.y;
  const uint64_t row = blockIdx.y * 16ull + ty, col = blockIdx.x * 16ull + tx;
  const uint64_t arow = blockIdx.y * 16ull + ty, brow = blockIdx.x * 16ull + ty;
  float acc = 0.0f;
  for (uint64_t k0 = 0; k0 < k; k0 += 32) {
    for (uint32_t kk = tx; kk < 32; kk += 16) {
      As[ty][kk] = (arow < m && k0 + kk < k) ? a[arow * k + k0 + kk] : 0.0f;
      Bs[ty][kk] = (brow < n && k0 + kk < k) ? b[brow * k + k0 + kk] : 0.0f;
    }
    __syncthreads();
    const uint32_t lim = (uint32_t)umin64(32, k - k0);
    for (uint32_t kk = 0; kk < lim; ++kk) {
      const float p = canon(__fmul_rn(As[ty][kk], Bs[tx][kk]));
      acc = (k0 == 0 && kk == 0) ? p : canon(__fadd_rn(acc, p));
    }
    __syncthreads();
  }
  if (row < m && col < n) c[row * n + col] = canon(acc);
}

void launch_contract_f32(const float* a, const float* b, uint64_t m, uint64_t n, uint64_t k, float* c,
                         cudaStream_t stream) {
  dim3 block(16, 16), grid((unsigned)((n + 15) / 16), (unsigned)((m + 15) / 16));
  contract_f32_kernel<<<grid, block, 0, stream>>>(a, b, m, n, k, c);
}

// ---------------------------------------------------------------------------
// tcgen05 bf16 GEMM
// ---------------------------------------------------------------------------
constexpr int kBM = 128, kBN = 256, kBK = 64, kStages = 4;
constexpr int kTileABytes = kBM * kBK * 2;  // 16 KB
constexpr int kTileBBytes = kBN * kBK * 2;  // 32 KB
constexpr int kStageBytes = kTileABytes + kTileBBytes;
constexpr int kGemmEpiWarps = 8;  // two per TMEM lane quarter, each draining half the columns
constexpr int kGemmThreads = 32 * (2 + kGemmEpiWarps);
constexpr uint32_t kTmemCols = 512;

// All-gather fused into the epilogue: every output box of this rank is also
// written into the same place of each peer's block buffer [world, m, n]
// (rank-major blocks; block r holds rank r's columns), with plain 16-byte
// stores over NVLink from the staged box.  The local copy goes out by TMA.
constexpr int kGemmMaxPeers = 8;
struct GemmPeers {
  uint16_t* block[kGemmMaxPeers];  // this rank's block inside each rank's buffer (nullptr: skip)
  uint32_t count;
  // Or: this rank's block inside an NVLink multicast mapping of every rank's
  // buffer.  One multimem.st per 16 bytes then reaches every rank's copy
  // (this rank's included) through the switch, so each box crosses NVLink
  // once instead of once per peer, and the local TMA store is skipped.
  uint16_t* multicast;
};

// Epilogue staging: per epilogue warp one 32-row x 64-column bf16 box
// (4 KB, 128-byte swizzle) that a TMA store writes to C.
constexpr int kEpiBoxCols = 64;
constexpr int kEpiStageBytes = 32 * kEpiBoxCols * 2;

struct GemmBars {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint32_t tmem_base;
  int abort;
};
constexpr size_t kGemmSmem = 1024 /*alignment slack*/ + (size_t)kStages * kStageBytes +
                             (size_t)kGemmEpiWarps * kEpiStageBytes + sizeof(GemmBars) + 64;

// Shared-memory matrix descriptor (tcgen05 "matrix descriptor"): K-major,
// 128-byte swizzle, 8-row core groups 1024 bytes apart.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3fff);        // start address
  d |= (uint64_t)1 << 16;                         // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;               // stride byte offset
  d |= (uint64_t)1 << 46;                         // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;                         // SWIZZLE_128B
  return d;
}

// Instruction descriptor: kind::f16, A/B bf16, D f32, both K-major, M=128, N=256.
constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kBN >> 3) << 17) |
                            ((uint32_t)(kBM >> 4) << 24);

__device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void mma_bf16(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(kIdesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

#define TMEM_LD32(taddr, r)                                                                                         \
  asm volatile(                                                                                                     \
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19," \
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"                                                    \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),           \
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),     \
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),   \
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])    \
      : "r"(taddr))

// One epilogue warp's share of a finished accumulator: TMEM lanes of its
// quarter (32 rows, row_base in C), columns [col0, col0 + kBN/2) of the tile
// starting at TMEM column tmem_tile, in 32x64 boxes: tcgen05.ld, SiLU (or the
// plain bf16 rounding), swizzled staging, one TMA store per box, and the box
// to every peer block when the all-gather is fused.
__device__ __forceinline__ void gemm_epilogue_tile(uint32_t tmem_tile, uint32_t col0, uint32_t stage_u32, uint32_t lane,
                                                   uint64_t row_base, uint64_t col_base, int epilogue,
                                                   const CUtensorMap* tmap_c, const GemmPeers& peers, uint64_t ldp,
                                                   tiler_cuda_status* st) {
#pragma unroll 1
  for (uint32_t box = col0; box < col0 + (uint32_t)kBN / 2; box += kEpiBoxCols) {
    // the previous box's store has finished reading the staging buffer
    if (lane == 0) asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
    __syncwarp();
#pragma unroll 1
    for (uint32_t half = 0; half < 2; ++half) {
      uint32_t r[32];
      const uint32_t taddr = tmem_tile + box + half * 32;
      TMEM_LD32(taddr, r);
      asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
      if (epilogue == 1) {
        uint32_t uncertain = 0;
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          bool certain;
          const uint32_t bits = silu_bf16_fast(__uint_as_float(r[j]), &certain);
          uncertain |= (certain ? 0u : 1u) << j;
          r[j] = bits;
        }
        if (__any_sync(0xffffffffu, uncertain != 0)) {
          // rare: reload the accumulators and certify the flagged ones
          uint32_t x[32];
          TMEM_LD32(taddr, x);
          asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
          for (int j = 0; j < 32; ++j)
            if ((uncertain >> j) & 1u) r[j] = silu_bf16_certified(__uint_as_float(x[j]), g_exp2_hi, st);
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) r[j] = f32_to_bf16(canon(__uint_as_float(r[j])));
      }
      // row `lane` of the box: 16-byte chunk c (of 8) at c ^ (row & 7)
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const uint32_t chunk = half * 4 + q;
        const uint32_t off = lane * 128 + ((chunk ^ (lane & 7)) * 16);
        asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(stage_u32 + off),
                     "r"(r[8 * q] | (r[8 * q + 1] << 16)), "r"(r[8 * q + 2] | (r[8 * q + 3] << 16)),
                     "r"(r[8 * q + 4] | (r[8 * q + 5] << 16)), "r"(r[8 * q + 6] | (r[8 * q + 7] << 16))
                     : "memory");
      }
    }
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
    __syncwarp();
    if (lane == 0 && !peers.multicast) {
      const int32_t x = (int32_t)(col_base + box), y = (int32_t)row_base;
      asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];" ::"l"(tmap_c),
                   "r"(x), "r"(y), "r"(stage_u32)
                   : "memory");
      asm volatile("cp.async.bulk.commit_group;" ::: "memory");
    }
    if (peers.multicast) {
      // the box to every rank at once: 8 lanes per 128-byte row, 4 rows per step
      const uint32_t c = lane & 7, rr = lane >> 3;
      const uint64_t col = col_base + box + c * 8;
#pragma unroll
      for (uint32_t r0 = 0; r0 < 32; r0 += 4) {
        const uint32_t r = r0 + rr;
        const uint4 v = lds_u4(stage_u32 + r * 128 + ((c ^ (r & 7)) * 16));
        uint16_t* dst = peers.multicast + (row_base + r) * ldp + col;
        asm volatile("multimem.st.relaxed.sys.global.v4.f32 [%0], {%1, %2, %3, %4};" ::"l"(dst), "r"(v.x), "r"(v.y),
                     "r"(v.z), "r"(v.w)
                     : "memory");
      }
      __syncwarp();  // the staging buffer is rewritten by the next box
    } else if (peers.count) {
      // the box to each peer: 8 lanes per 128-byte row, 4 rows per step
      const uint32_t c = lane & 7, rr = lane >> 3;
      const uint64_t col = col_base + box + c * 8;
#pragma unroll
      for (uint32_t r0 = 0; r0 < 32; r0 += 4) {
        const uint32_t r = r0 + rr;
        const uint4 v = lds_u4(stage_u32 + r * 128 + ((c ^ (r & 7)) * 16));
        const uint64_t row = row_base + r;
        for (uint32_t q = 0; q < peers.count; ++q)
          if (peers.block[q]) *reinterpret_cast<uint4*>(peers.block[q] + row * ldp + col) = v;
      }
    }
  }
}

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_tcgen05_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                             const __grid_constant__ CUtensorMap tmap_c, uint32_t m_blocks, uint32_t n_blocks,
                             uint32_t k_blocks, int epilogue, tiler_cuda_status* st,
                             const __grid_constant__ GemmPeers peers, uint64_t ldp) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t pad = ((raw + 1023) & ~1023u) - raw;
  uint8_t* tiles = smem_raw + pad;
  uint8_t* epi_stage = tiles + (size_t)kStages * kStageBytes;  // 1024-byte aligned
  GemmBars& B = *reinterpret_cast<GemmBars*>(epi_stage + (size_t)kGemmEpiWarps * kEpiStageBytes);
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t num_tiles = m_blocks * n_blocks;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) { mbar_init(&B.full[s], 1); mbar_init(&B.empty[s], 1); }
    for (int s = 0; s < 2; ++s) { mbar_init(&B.tmem_full[s], 1); mbar_init(&B.tmem_empty[s], 32 * kGemmEpiWarps); }
    B.abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&B.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem_base = B.tmem_base;
  volatile int* abort_flag = &B.abort;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t keep = policy_evict_last();
      uint64_t it = 0;
      for (uint32_t tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x) {
        const uint32_t mb = tile % m_blocks, nb = tile / m_blocks;
        for (uint32_t kb = 0; kb < k_blocks; ++kb, ++it) {
          const uint32_t s = it % kStages;
          const uint64_t use = it / kStages;
          if (use > 0 && !mbar_wait(&B.empty[s], (uint32_t)((use - 1) & 1), st)) { *abort_flag = 1; break; }
          uint8_t* sa = tiles + (size_t)s * kStageBytes;
          mbar_arrive_expect_tx(&B.full[s], kStageBytes);
          tma_load_2d(sa, &tmap_a, (int)(kb * kBK), (int)(mb * kBM), &B.full[s], keep);
          tma_load_2d(sa + kTileABytes, &tmap_b, (int)(kb * kBK), (int)(nb * kBN), &B.full[s], keep);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0) {
      uint64_t it = 0;
      uint32_t local = 0;
      for (uint32_t tile = blockIdx.x; tile < num_tiles && !*abort_flag; tile += gridDim.x, ++local) {
        const uint32_t buf = local & 1;
        const uint32_t use = local >> 1;
        if (use > 0 && !mbar_wait(&B.tmem_empty[buf], (use - 1) & 1, st)) { *abort_flag = 1; break; }
        tmem_fence_after();
        const uint32_t d_tmem = tmem_base + buf * kBN;
        for (uint32_t kb = 0; kb < k_blocks; ++kb, ++it) {
          const uint32_t s = it % kStages;
          if (!mbar_wait(&B.full[s], (uint32_t)((it / kStages) & 1), st)) { *abort_flag = 1; break; }
          tmem_fence_after();
          const uint32_t sa = smem_u32(tiles + (size_t)s * kStageBytes);
          const uint32_t sb = sa + kTileABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_bf16(d_tmem, smem_desc_sw128(sa + kk * 32), smem_desc_sw128(sb + kk * 32), (kb | kk) != 0);
          mma_commit(&B.empty[s]);  // the stage is free once these MMAs have read it
        }
        if (*abort_flag) break;
        mma_commit(&B.tmem_full[buf]);  // the accumulator is complete
      }
    }
  } else {
    // epilogue warps 2..9: TMEM lane quarter (warp % 4), column half (warp - 2) / 4
    const uint32_t quarter = warp & 3;
    const uint32_t col0 = ((warp - 2) / 4) * (kBN / 2);
    uint8_t* stage = epi_stage + (size_t)(warp - 2) * kEpiStageBytes;
    const uint32_t stage_u32 = smem_u32(stage);
    uint32_t local = 0;
    for (uint32_t tile = blockIdx.x; tile < num_tiles; tile += gridDim.x, ++local) {
      const uint32_t mb = tile % m_blocks, nb = tile / m_blocks;
      const uint32_t buf = local & 1;
      if (!mbar_wait(&B.tmem_full[buf], (local >> 1) & 1, st)) { *abort_flag = 1; break; }
      if (*abort_flag) break;
      tmem_fence_after();
      gemm_epilogue_tile(tmem_base + ((quarter * 32) << 16) + buf * kBN, col0, stage_u32, lane,
                         (uint64_t)mb * kBM + quarter * 32, (uint64_t)nb * kBN, epilogue, &tmap_c, peers, ldp, st);
      tmem_fence_before();
      mbar_arrive(&B.tmem_empty[buf]);
    }
    // the stores have completed before the CTA (and its shared memory) goes away
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    if (peers.count || peers.multicast) __threadfence_system();  // the peer stores are visible before the kernel ends
  }
  tmem_fence_before();
  __syncthreads();
  if (warp == 1) {
    tmem_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                 : "memory");
  }
}

// ---- the CTA-pair form: cta_group::2, 256 x 256 tiles per cluster of two ----
//
// A cluster of two CTAs (on the two SMs of a TPC) computes one 256 x 256 tile:
// CTA r holds rows [128 r, 128 r + 128) of the A tile and rows [128 r,
// 128 r + 128) of the B tile (N-split) in its shared memory, and its TMEM
// holds its 128 rows x 256 columns of the accumulator.  CTA 0's MMA thread
// issues tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16), which reads
// both CTAs' operands; each SM therefore loads 32 KB per K-step of 64 for the
// same FLOPs that take 48 KB in the single-CTA form.  Both CTAs' TMA loads
// complete on CTA 0's full barrier (plain tiled loads with the cta_group::2
// barrier form, no multicast); CTA 0's commits arrive on both CTAs' empty and
// accumulator-full barriers; every epilogue warp of both CTAs arrives on CTA
// 0's accumulator-empty barrier.  All waits are bounded as in the single-CTA
// kernel.
constexpr int kPairStages = 6;
constexpr int kPairTileBBytes = (kBN / 2) * kBK * 2;  // this CTA's half of the 256 B rows: 16 KB
constexpr int kPairStageBytes = kTileABytes + kPairTileBBytes;
constexpr uint32_t kIdescPair = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(kBN >> 3) << 17) |
                                ((uint32_t)((2 * kBM) >> 4) << 24);

struct PairBars {
  uint64_t full[kPairStages];
  uint64_t empty[kPairStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint32_t tmem_base;
  int abort;
};
constexpr size_t kPairSmem = 1024 + (size_t)kPairStages * kPairStageBytes + (size_t)kGemmEpiWarps * kEpiStageBytes +
                             sizeof(PairBars) + 64;

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// the shared::cluster address of the same variable in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx_u32(uint32_t saddr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(saddr), "r"(bytes) : "memory");
}
// a tiled 2-D load into this CTA's shared memory whose bytes complete on the
// barrier at `bar_cluster` (CTA 0's), without multicast
__device__ __forceinline__ void tma_load_2d_pair(uint32_t smem_dst, const void* tmap, int32_t x, int32_t y,
                                                 uint32_t bar_cluster, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(smem_dst),
      "l"(tmap), "r"(x), "r"(y), "r"(bar_cluster), "l"(policy)
      : "memory");
}
__device__ __forceinline__ void mma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, {%5, %5, %5, %5, %5, %5, %5, %5}, p;\n}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(kIdescPair), "r"(accumulate), "r"(0u)
      : "memory");
}
// CTA 0's commit: the barrier at the same offset in both CTAs receives one arrival
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kGemmThreads, 1)
    gemm_bf16_pair_kernel(const __grid_constant__ CUtensorMap tmap_a, const __grid_constant__ CUtensorMap tmap_b,
                          const __grid_constant__ CUtensorMap tmap_c, uint32_t m_blocks, uint32_t n_blocks,
                          uint32_t k_blocks, int epilogue, tiler_cuda_status* st,
                          const __grid_constant__ GemmPeers peers, uint64_t ldp) {
  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw = smem_u32(smem_raw);
  const uint32_t pad = ((raw + 1023) & ~1023u) - raw;
  uint8_t* tiles = smem_raw + pad;
  uint8_t* epi_stage = tiles + (size_t)kPairStages * kPairStageBytes;  // 1024-byte aligned
  PairBars& B = *reinterpret_cast<PairBars*>(epi_stage + (size_t)kGemmEpiWarps * kEpiStageBytes);
  const uint32_t warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const uint32_t cluster = blockIdx.x >> 1, clusters = gridDim.x >> 1;
  const uint32_t num_tiles = m_blocks * n_blocks;  // 256 x 256 tiles

  if (threadIdx.x == 0) {
    for (int s = 0; s < kPairStages; ++s) { mbar_init(&B.full[s], 1); mbar_init(&B.empty[s], 1); }
    for (int s = 0; s < 2; ++s) { mbar_init(&B.tmem_full[s], 1); mbar_init(&B.tmem_empty[s], 2 * kGemmEpiWarps); }
    B.abort = 0;
    fence_barrier_init();
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&B.tmem_base)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tmem_fence_before();
  cluster_sync_all();  // both CTAs' barriers are initialised before either signals the other
  tmem_fence_after();
  const uint32_t tmem_base = B.tmem_base;
  volatile int* abort_flag = &B.abort;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t keep = policy_evict_last();
      uint64_t it = 0;
      for (uint32_t tile = cluster; tile < num_tiles && !*abort_flag; tile += clusters) {
        const uint32_t mb = tile % m_blocks, nb = tile / m_blocks;
        for (uint32_t kb = 0; kb < k_blocks; ++kb, ++it) {
          const uint32_t s = it % kPairStages;
          const uint64_t use = it / kPairStages;
          if (use > 0 && !mbar_wait(&B.empty[s], (uint32_t)((use - 1) & 1), st)) { *abort_flag = 1; break; }
          const uint32_t sa = smem_u32(tiles + (size_t)s * kPairStageBytes);
          const uint32_t full0 = mapa_shared(smem_u32(&B.full[s]), 0);
          if (rank == 0) mbar_arrive_expect_tx_u32(smem_u32(&B.full[s]), 2 * kPairStageBytes);
          tma_load_2d_pair(sa, &tmap_a, (int)(kb * kBK), (int)(mb * 2 * kBM + rank * kBM), full0, keep);
          tma_load_2d_pair(sa + kTileABytes, &tmap_b, (int)(kb * kBK), (int)(nb * kBN + rank * (kBN / 2)), full0,
                           keep);
        }
      }
    }
  } else if (warp == 1) {
    if (lane == 0 && rank == 0) {
      uint64_t it = 0;
      uint32_t local = 0;
      for (uint32_t tile = cluster; tile < num_tiles && !*abort_flag; tile += clusters, ++local) {
        const uint32_t buf = local & 1;
        const uint32_t use = local >> 1;
        if (use > 0 && !mbar_wait(&B.tmem_empty[buf], (use - 1) & 1, st)) { *abort_flag = 1; break; }
        tmem_fence_after();
        const uint32_t d_tmem = tmem_base + buf * kBN;
        for (uint32_t kb = 0; kb < k_blocks; ++kb, ++it) {
          const uint32_t s = it % kPairStages;
          if (!mbar_wait(&B.full[s], (uint32_t)((it / kPairStages) & 1), st)) { *abort_flag = 1; break; }
          tmem_fence_after();
          const uint32_t sa = smem_u32(tiles + (size_t)s * kPairStageBytes);
          const uint32_t sb = sa + kTileABytes;
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)
            mma_bf16_pair(d_tmem, smem_desc_sw128(sa + kk * 32), smem_desc_sw128(sb + kk * 32), (kb | kk) != 0);
          mma_commit_pair(&B.empty[s]);  // both CTAs' stage s is free once these MMAs have read it
        }
        if (*abort_flag) break;
        mma_commit_pair(&B.tmem_full[buf]);  // both halves of the accumulator are complete
      }
    }
  } else {
    const uint32_t quarter = warp & 3;
    const uint32_t col0 = ((warp - 2) / 4) * (kBN / 2);
    const uint32_t stage_u32 = smem_u32(epi_stage + (size_t)(warp - 2) * kEpiStageBytes);
    uint32_t local = 0;
    for (uint32_t tile = cluster; tile < num_tiles; tile += clusters, ++local) {
      const uint32_t mb = tile % m_blocks, nb = tile / m_blocks;
      const uint32_t buf = local & 1;
      if (!mbar_wait(&B.tmem_full[buf], (local >> 1) & 1, st)) { *abort_flag = 1; break; }
      if (*abort_flag) break;
      tmem_fence_after();
      gemm_epilogue_tile(tmem_base + ((quarter * 32) << 16) + buf * kBN, col0, stage_u32, lane,
                         (uint64_t)mb * 2 * kBM + rank * kBM + quarter * 32, (uint64_t)nb * kBN, epilogue, &tmap_c,
                         peers, ldp, st);
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_remote(mapa_shared(smem_u32(&B.tmem_empty[buf]), 0));
    }
    if (lane == 0) asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
    if (peers.count || peers.multicast) __threadfence_system();
  }
  tmem_fence_before();
  cluster_sync_all();  // no arrival or load of one CTA targets the other after this
  if (warp == 1) {
    tmem_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                 : "memory");
  }
}

// K-major bf16 matrix [rows, k] -> tensor map with a (64 x box_rows) box.
static bool make_tmap(CUtensorMap* map, const void* base, uint64_t rows, uint64_t k, uint32_t box_rows) {
  return make_tmap_2d(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, base, k, rows, k * 2, (uint32_t)kBK, box_rows,
                      CU_TENSOR_MAP_SWIZZLE_128B);
}

int launch_gemm_bf16(const uint16_t* a, const uint16_t* b, uint64_t m, uint64_t n, uint64_t k, int epilogue,
                     uint16_t* c, uint64_t ldc, tiler_cuda_status* st, int sm_count, cudaStream_t stream,
                     uint16_t* const* peer_blocks, uint32_t npeers, uint16_t* multicast) {
  if (npeers > (uint32_t)kGemmMaxPeers) return TILER_CUDA_UNSUPPORTED;
  GemmPeers peers{};
  peers.count = npeers;
  peers.multicast = multicast;
  if ((uintptr_t)multicast % 16) return TILER_CUDA_UNSUPPORTED;
  for (uint32_t q = 0; q < npeers; ++q) {
    peers.block[q] = peer_blocks[q];
    if (peer_blocks[q] && (uintptr_t)peer_blocks[q] % 16) return TILER_CUDA_UNSUPPORTED;
  }
  if (m % kBM || n % kBN || k % kBK || k == 0) return TILER_CUDA_UNSUPPORTED;
  if ((uintptr_t)a % 16 || (uintptr_t)b % 16 || (uintptr_t)c % 16 || ldc % 8 || ldc < n) return TILER_CUDA_UNSUPPORTED;
  CUtensorMap ta, tb, tcm;
  if (!make_tmap(&ta, a, m, k, kBM) || !make_tmap(&tb, b, n, k, kBN)) return TILER_CUDA_DEVICE_ERROR;
  // C [m, n] bf16 row-major with row pitch ldc: 64 x 32 boxes, 128-byte swizzle
  if (!make_tmap_2d(&tcm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, c, n, m, ldc * 2, (uint32_t)kEpiBoxCols, 32,
                    CU_TENSOR_MAP_SWIZZLE_128B))
    return TILER_CUDA_DEVICE_ERROR;
  const uint32_t kbk = (uint32_t)(k / kBK);
  static const int pair_env = [] {
    const char* e = getenv("TILER_GEMM_PAIR");
    return e ? atoi(e) : 1;
  }();
  if (pair_env && m % (2 * kBM) == 0 && sm_count >= 2) {
    // the CTA-pair form: B's tensor map boxes are half the N rows of a tile
    CUtensorMap tbp;
    if (!make_tmap(&tbp, b, n, k, kBN / 2)) return TILER_CUDA_DEVICE_ERROR;
    const uint32_t mb2 = (uint32_t)(m / (2 * kBM)), nbk2 = (uint32_t)(n / kBN);
    const uint32_t grid = 2 * std::min<uint32_t>(mb2 * nbk2, (uint32_t)sm_count / 2);
    cudaFuncSetAttribute(gemm_bf16_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kPairSmem);
    gemm_bf16_pair_kernel<<<grid, kGemmThreads, kPairSmem, stream>>>(ta, tbp, tcm, mb2, nbk2, kbk, epilogue, st,
                                                                     peers, ldc);
    return TILER_CUDA_OK;
  }
  const uint32_t mbk = (uint32_t)(m / kBM), nbk = (uint32_t)(n / kBN);
  const uint32_t tiles = mbk * nbk;
  const unsigned grid = std::min<uint32_t>(tiles, (uint32_t)sm_count);
  cudaFuncSetAttribute(gemm_bf16_tcgen05_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kGemmSmem);
  gemm_bf16_tcgen05_kernel<<<grid, kGemmThreads, kGemmSmem, stream>>>(ta, tb, tcm, mbk, nbk, kbk, epilogue, st, peers,
                                                                      ldc);
  return TILER_CUDA_OK;
}

}  // namespace tc
