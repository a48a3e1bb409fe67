// Internal launch interface between the C-ABI layer (abi.cu) and the family
// kernels.  Not part of the public ABI.
#pragma once
#include <cuda_runtime.h>
#include <stdint.h>

#include <algorithm>

#include "../../include/tiler_cuda.h"

namespace tc {

struct GroupedParams {
  uint64_t partitions;
  uint32_t threads, k, rounds;
  uint32_t combine_threads, combine_k, combine_rounds;
};

// reduce.cu
void launch_grouped_fold(int op, const float* x, uint64_t rows, uint64_t count, const GroupedParams& gp,
                         float* partials, unsigned int* tickets, float* out, cudaStream_t stream);
void launch_strict_sum(const float* x, uint64_t rows, uint64_t count, float* out, cudaStream_t stream);
void launch_partitioned_sum(const float* x, uint64_t rows, uint64_t count, uint64_t P, uint64_t per,
                            float* partials, float* out, cudaStream_t stream);
void launch_cooperative_sum(const float* x, uint64_t rows, uint64_t count, uint64_t participants, uint64_t per,
                            uint64_t rounds, int participant_major, float* out, cudaStream_t stream);

// rows.cu
int launch_rms_norm(int bf16, const void* x, const void* w, int64_t w_row_stride, uint64_t rows, uint64_t extent,
                    float eps, void* y, tiler_cuda_status* st, int sm_count, cudaStream_t stream);
// mask (nullable): the additive mask tensor [mask_rows, extent] added to row r
// as mask[(row_offset + r) mod mask_rows]; TILER_CUDA_UNSUPPORTED unless the
// staged kernel applies (extent % 4 == 0, extent <= 8192, 16-byte aligned)
// and causal_period == 0.
int launch_softmax(const float* x, uint64_t rows, uint64_t extent, uint64_t causal_period, uint64_t row_offset,
                   float* y, tiler_cuda_status* st, int sm_count, cudaStream_t stream, const float* mask = nullptr,
                   uint64_t mask_rows = 0);
// Fused RMS norm (f32) -> per-row int8 quantize of y; TILER_CUDA_UNSUPPORTED for
// unaligned operands or an extent that is not a multiple of 4.
int launch_rms_norm_quantize_i8(const float* x, const float* w, int64_t w_row_stride, uint64_t rows,
                                uint64_t extent, float eps, int8_t* codes, float* scales, tiler_cuda_status* st,
                                int sm_count, cudaStream_t stream);
// rms_scan.cu: the warp-per-row RMS kernel (and its fused int8 quantize form);
// false when the operands do not fit it (per-row weights, rows over 16 KB or
// not a multiple of 16 bytes, unaligned pointers): the caller takes another form.
bool rms_scan_launch(int bf16, int quant, const void* x, const void* w, int64_t w_row_stride, uint64_t rows,
                     uint64_t extent, float eps, void* y, int8_t* codes, float* scales, tiler_cuda_status* st,
                     int sm_count, cudaStream_t stream);
// The chunk-streamed RMS kernel (rms_stream.cu); false where it does not apply
// (a weight row per row, rows not a multiple of 16 bytes or longer than its
// chunk rings hold).
bool rms_stream_launch(int bf16, const void* x, const void* w, int64_t w_row_stride, uint64_t rows, uint64_t extent,
                       float eps, void* y, tiler_cuda_status* st, int sm_count, cudaStream_t stream);
bool rms_stream_quant_launch(const float* x, const float* w, int64_t w_row_stride, uint64_t rows, uint64_t extent,
                             float eps, int8_t* codes, float* scales, tiler_cuda_status* st, int sm_count,
                             cudaStream_t stream);
void launch_bounded_wait_selftest(tiler_cuda_status* st, uint64_t limit_ns, cudaStream_t stream);
void launch_quantize_i8_rows(const float* x, uint64_t rows, uint64_t extent, int8_t* codes, float* scales,
                             tiler_cuda_status* st, int sm_count, cudaStream_t stream);
void launch_dequantize_i8_rows(const int8_t* codes, const float* scales, uint64_t rows, uint64_t extent, float* y,
                               int sm_count, cudaStream_t stream, tiler_cuda_status* st);

// maps.cu
void launch_silu(const float* x, uint64_t n, float* y, tiler_cuda_status* st, int sm_count, cudaStream_t stream);
void launch_scale_bias(const float* x, uint64_t n, const float* a, int a_scalar, const float* b, int b_scalar,
                       float* y, int sm_count, cudaStream_t stream);
void launch_gather_rows(const void* table, uint64_t table_rows, uint64_t row_bytes, const void* ids,
                        int ids_unsigned, uint64_t n_ids, void* out, tiler_cuda_status* st, int sm_count,
                        cudaStream_t stream);
void launch_quantize_affine_u8(const float* x, uint64_t n, float scale, uint32_t zp, uint32_t maximum,
                               uint8_t* codes, tiler_cuda_status* st, int sm_count, cudaStream_t stream);
void launch_dequantize_affine_u8(const uint8_t* codes, uint64_t n, float scale, uint32_t zp, uint32_t maximum,
                                 float* y, tiler_cuda_status* st, int sm_count, cudaStream_t stream);
void launch_status_reset(tiler_cuda_status* st, cudaStream_t stream);

// gemm.cu
void launch_contract_f32(const float* a, const float* b, uint64_t m, uint64_t n, uint64_t k, float* c,
                         cudaStream_t stream);
// peer_blocks (nullable entries): where this rank's C also goes, one pointer per
// rank (row pitch ldc); the all-gather fused into the epilogue.
int launch_gemm_bf16(const uint16_t* a, const uint16_t* b, uint64_t m, uint64_t n, uint64_t k, int epilogue,
                     uint16_t* c, uint64_t ldc, tiler_cuda_status* st, int sm_count, cudaStream_t stream,
                     uint16_t* const* peer_blocks = nullptr, uint32_t npeers = 0, uint16_t* multicast = nullptr);

// Kernel registry (entry symbols for payload validation / entry queries).
struct EntryInfo {
  const char* symbol;
  const void* func;
  int threads;
  size_t dynamic_smem;
};
int entry_count();
const EntryInfo* entry_at(int i);

}  // namespace tc
