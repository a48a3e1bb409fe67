/*
 * CPU parity oracle for the tiler-cuda hot path — TEST INFRASTRUCTURE ONLY.
 *
 * A C++ restatement of moderately-ai/tiler's `tiler-reference` crate for the
 * operation families the CUDA backend realizes.  It is the checker the parity
 * tests, `__graft_entry__.smoke()` and `bench.py`'s CPU-baseline leg call; the
 * product library (`tiler_b200/libtiler_cuda.so`) never links or calls it.
 *
 * Pinning: the reference is Rust (nightly) and cannot be built in this image,
 * so this restatement is pinned against the golden bit patterns the
 * reference's own tests assert (tests/golden/reference_vectors.json, each
 * vector citing its reference test file:line) and the six SHA-256 digests of
 * crates/tiler-reference/tests/contraction_profile_cells.rs:175-222.
 * Groupings with no reference evaluator (the ADR-0096/0100 subgroup
 * composition) and the config extensions (signed per-row int8, bf16 RMS,
 * i32 ids, bf16 contraction + SiLU) are "parity unpinned" beyond the
 * identities the reference states for them.
 *
 * Arithmetic: compiled with -ffp-contract=off and without fast-math, so
 * every `a + b` / `a * b` / `a / b` below is one IEEE binary32 operation
 * rounded to nearest-even with subnormals preserved, as the reference's host
 * arithmetic is.  Transcendentals are certified through __float128.
 */
#ifndef TILER_ORACLE_H
#define TILER_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes shared with the product ABI (include/tiler_cuda.h). */
enum {
  ORACLE_OK = 0,
  ORACLE_INVALID_APPLICATION = 1,
  ORACLE_GATHER_INDEX_OUT_OF_BOUNDS = 3,
  ORACLE_NAN_INPUT = 4,
  ORACLE_UNDECIDED = 5,
  ORACLE_SCALE_DOMAIN = 9,
};

typedef struct oracle_error {
  int32_t code;
  uint64_t position;
  int64_t value;
  uint64_t extent;
} oracle_error;

/* ---- scalar primitives ------------------------------------------------- */
float oracle_canonicalize(float v);
float oracle_maximum(float a, float b);
float oracle_exp(float x, int32_t* undecided);
float oracle_rsqrt(float t, int32_t* undecided);
float oracle_silu(float x, int32_t* undecided);
uint16_t oracle_f32_to_bf16(float v);
float oracle_bf16_to_f32(uint16_t b);

/* ---- reductions (rows x count, contiguous rows) ------------------------ */
int32_t oracle_strict_sum(const float* x, uint64_t rows, uint64_t count, float* out);
int32_t oracle_partitioned_sum(const float* x, uint64_t rows, uint64_t count,
                               uint64_t partitions, uint64_t per_partition,
                               float* out);
int32_t oracle_cooperative_sum(const float* x, uint64_t rows, uint64_t count,
                               uint64_t participants, uint64_t per_partition,
                               uint64_t rounds, int32_t participant_major,
                               float* out);
/* ADR-0100 composition (op 0 = sum, 1 = maximum) over one sequence. */
int32_t oracle_compose_fold(const float* seq, uint64_t n, uint32_t threads,
                            uint32_t k, uint32_t rounds, int32_t op, float* out);
/* The backend's declared grid grouping: exact partitions, each folded by the
 * composition (threads,k,rounds); partials combined by a strict fold
 * (combine_threads == 0) or by a second composition. */
int32_t oracle_grid_fold(const float* x, uint64_t rows, uint64_t count,
                         uint64_t partitions, uint32_t threads, uint32_t k,
                         uint32_t rounds, uint32_t combine_threads,
                         uint32_t combine_k, uint32_t combine_rounds,
                         int32_t op, int32_t nthreads, float* out);
int32_t oracle_strict_max(const float* x, uint64_t rows, uint64_t count, float* out);

/* ---- row families ------------------------------------------------------ */
int32_t oracle_rms_norm_f32(const float* x, const float* w, int64_t w_row_stride,
                            uint64_t rows, uint64_t extent, uint32_t eps_bits,
                            float* y, int32_t nthreads);
int32_t oracle_rms_norm_bf16(const uint16_t* x, const uint16_t* w, int64_t w_row_stride,
                             uint64_t rows, uint64_t extent, uint32_t eps_bits,
                             uint16_t* y, int32_t nthreads);
int32_t oracle_softmax_f32(const float* x, uint64_t rows, uint64_t extent,
                           uint64_t causal_period, uint64_t row_offset,
                           float* y, int32_t nthreads);
int32_t oracle_silu_f32(const float* x, uint64_t n, float* y);
int32_t oracle_scale_bias_f32(const float* x, uint64_t n, const float* a, int32_t a_scalar,
                              const float* b, int32_t b_scalar, float* y);
int32_t oracle_gather_rows(const void* table, uint64_t table_rows, uint64_t row_bytes,
                           const void* ids, int32_t ids_unsigned, uint64_t n_ids,
                           void* out, oracle_error* err);
int32_t oracle_quantize_i8_rows(const float* x, uint64_t rows, uint64_t extent,
                                int8_t* codes, float* scales, oracle_error* err,
                                int32_t nthreads);
int32_t oracle_dequantize_i8_rows(const int8_t* codes, const float* scales,
                                  uint64_t rows, uint64_t extent, float* y,
                                  int32_t nthreads);
int32_t oracle_quantize_affine_u8(const float* x, uint64_t n, float scale,
                                  uint32_t zero_point, uint32_t maximum,
                                  uint8_t* codes, oracle_error* err);
int32_t oracle_dequantize_affine_u8(const uint8_t* codes, uint64_t n, float scale,
                                    uint32_t zero_point, float* y);

/* ---- contraction ------------------------------------------------------- */
/* td,od->to strict f32 contraction: A[M,K], B[N,K] -> C[M,N]; seed = first
 * product, product and sum rounded separately. */
int32_t oracle_contract_f32(const float* a, const float* b, uint64_t m, uint64_t n,
                            uint64_t k, float* c, int32_t nthreads);
/* Config extension: bf16 A[M,K], B[N,K], f32 strict fold, SiLU epilogue,
 * bf16 RNE output.  Rows [row_begin,row_end) only (sampled oracle). */
int32_t oracle_gemm_bf16_silu(const uint16_t* a, const uint16_t* b, uint64_t m,
                              uint64_t n, uint64_t k, uint64_t row_begin,
                              uint64_t row_end, int32_t apply_silu, uint16_t* c,
                              int32_t nthreads);

#ifdef __cplusplus
}
#endif
#endif
