/*
 * libtiler_cuda — the C-ABI boundary of the B200-native (sm_100a) execution
 * backend for moderately-ai/tiler.
 *
 * The reference exposes its device seam as Rust traits, not a C ABI:
 *   - RuntimeAdapter (crates/tiler-runtime/src/adapter.rs:260-511) driven by
 *     route_with_adapter (adapter.rs:545-678): bind_execution_context,
 *     observe_live_device, validate_payload, prepare_entries,
 *     observe_prepared_entry, plan_dispatch, allocate_dispatch, dispatch;
 *   - PhysicalImplementationProvider::propose (crates/tiler-compiler/src/
 *     frontier.rs:1507-1527), which states a realization's reduction grouping;
 *   - the registered operation families evaluated by tiler-reference
 *     (crates/tiler-reference/src/lib.rs:86-110).
 * Each export below names the reference interface it stands in for.  A Rust
 * `tiler-cuda` crate binds these with `extern "C"` declarations.
 *
 * Conventions (mirroring RoutedBinding, crates/tiler-runtime/src/load/
 * route.rs:145-191):
 *   - every buffer is a caller-owned DEVICE pointer; shapes are plain
 *     integers; the library allocates no device memory on any launch path;
 *   - every call returns an int32_t status; argument refusals are returned
 *     synchronously before anything is enqueued (the reference's typed
 *     refusals before the routing commit, adapter.rs:693-800);
 *   - data-dependent refusals (an out-of-range gather index, a NaN quantize
 *     input, an undecided transcendental, a bounded wait that gave up) are
 *     written by the kernels into a caller-owned device status word
 *     (tiler_cuda_status) and decoded on the host after synchronizing;
 *   - launches are asynchronous on the caller's cudaStream_t (passed as
 *     void*); no exception or abort crosses the ABI;
 *   - a context is externally synchronized (one host thread at a time).
 */
#ifndef TILER_CUDA_H
#define TILER_CUDA_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TILER_CUDA_ABI_VERSION 1u

/* Status codes.  The data-dependent ones mirror ReferenceOperationError
 * variants of crates/tiler-reference/src/error.rs. */
enum {
  TILER_CUDA_OK = 0,
  TILER_CUDA_INVALID_APPLICATION = 1,        /* ReferenceOperationError::InvalidApplication */
  TILER_CUDA_SHAPE_TOO_LARGE = 2,            /* ReferenceOperationError::ShapeTooLarge */
  TILER_CUDA_GATHER_INDEX_OUT_OF_BOUNDS = 3, /* GatherIndexOutOfBounds{position,value,extent} */
  TILER_CUDA_NAN_INPUT = 4,                  /* quantize_one's NaN refusal (quantization.rs:411-413) */
  TILER_CUDA_UNDECIDED = 5,                  /* UndecidedTranscendentalReference */
  TILER_CUDA_DEVICE_ERROR = 6,               /* a CUDA runtime error */
  TILER_CUDA_TIMEOUT = 7,                    /* a bounded wait gave up */
  TILER_CUDA_UNSUPPORTED = 8,                /* a shape/layout this backend does not realize */
  TILER_CUDA_SCALE_DOMAIN = 9,               /* scale not positive-normal (quantization.rs:377-379) */
  TILER_CUDA_PAYLOAD_REFUSED = 10,           /* validate_payload refusal */
  TILER_CUDA_WORKSPACE_TOO_SMALL = 11
};

/* Device-resident status word written by the kernels (32 bytes, 8-aligned).
 * Reset it with tiler_cuda_status_reset before a launch that reports. */
typedef struct tiler_cuda_status {
  uint64_t error_key;  /* UINT64_MAX: none; else (position << 8) | code, smallest position wins */
  uint64_t value_key;  /* gather: (position << 32) | (uint32_t)offending index value */
  uint32_t undecided;  /* transcendental results the certification could not decide */
  uint32_t timeouts;   /* bounded device waits that gave up */
  uint64_t reserved;
} tiler_cuda_status;

/* Host-side decoded error (GatherIndexOutOfBounds carries all three fields). */
typedef struct tiler_cuda_error {
  int32_t code;
  uint32_t undecided;
  uint32_t timeouts;
  uint32_t pad;
  uint64_t position;
  int64_t value;
} tiler_cuda_error;

typedef struct tiler_cuda_context tiler_cuda_context;

/* observe_live_device (adapter.rs:648-651): the facts a route compares. */
typedef struct tiler_cuda_device_facts {
  int32_t device;
  int32_t cc_major;
  int32_t cc_minor;
  int32_t sm_count;
  int32_t warp_size; /* the subgroup width, checked as an equality (docs/artifact-abi.md:427-429) */
  int32_t max_threads_per_block;
  int64_t smem_per_block_optin;
  int64_t l2_bytes;
  int64_t global_mem_bytes;
  char name[96];
} tiler_cuda_device_facts;

/* observe_prepared_entry (adapter.rs:657-658). */
typedef struct tiler_cuda_entry_props {
  int32_t num_regs;
  int32_t max_threads_per_block;
  int64_t static_smem_bytes;
  int64_t dynamic_smem_bytes; /* what the planned launch requests */
  int32_t threads_per_block;  /* the planned launch geometry (RoutedLaunch, route.rs:69-97) */
  int32_t pad;
} tiler_cuda_entry_props;

/* A declared reduction grouping (the realization a provider proposes; the
 * oracle evaluates exactly this order):
 *   level 1: `partitions` exact contiguous partitions of count/partitions
 *            contributors (strict_partial_sums, evaluate.rs:612-832);
 *   level 2: each partition folded by the ADR-0100 composition (docs/decisions/
 *            0100-admit-the-multi-round-two-level-reduction-composition.md):
 *            `threads` = G*32 participants, `k` contiguous contributors per
 *            lane, `rounds` rounds, ascending XOR butterfly, tail padding
 *            with the two-sided identity;
 *   level 3: the partials folded strictly (combine_threads == 0, the second
 *            pass of strict_partitioned_sum) or by a second composition. */
typedef struct tiler_cuda_grouping {
  uint64_t partitions;
  uint32_t threads;
  uint32_t k;
  uint32_t rounds;
  uint32_t combine_threads;
  uint32_t combine_k;
  uint32_t combine_rounds;
} tiler_cuda_grouping;

/* ---- execution context (bind_execution_context, adapter.rs:552) ---------- */
uint32_t tiler_cuda_abi_version(void);
int32_t tiler_cuda_context_create(int32_t device, tiler_cuda_context** out);
int32_t tiler_cuda_context_destroy(tiler_cuda_context* ctx);
int32_t tiler_cuda_device_facts_query(const tiler_cuda_context* ctx, tiler_cuda_device_facts* out);
const char* tiler_cuda_status_string(int32_t code);

/* ---- payload (validate_payload / prepare_entries, adapter.rs:639-655) ----
 * The compiled payload is this library's sm_100a code.  Validation checks the
 * declared target ("sm_100a"), the subgroup width equality (32) and that each
 * entry symbol is one this library realizes; *refused_index names the first
 * refused symbol. */
int32_t tiler_cuda_payload_validate(const tiler_cuda_context* ctx, const char* target,
                                    uint32_t subgroup_width, const char* const* symbols,
                                    uint32_t n_symbols, uint32_t* refused_index);
uint32_t tiler_cuda_entry_count(void);
const char* tiler_cuda_entry_symbol(uint32_t index);
int32_t tiler_cuda_entry_query(const tiler_cuda_context* ctx, const char* symbol,
                               tiler_cuda_entry_props* out);

/* ---- payload code (PayloadContent.code, crates/tiler-artifact/src/program/
 * codec/payload.rs:228-424; validate_payload / prepare_entries /
 * observe_prepared_entry, crates/tiler-runtime/src/adapter.rs:639-657) ----
 * `code` is the artifact's code bytes: an sm_100a cubin built from this
 * library's kernel sources (tiler_b200/tiler_kernels.cubin).  Loading checks
 * that it is an image the device accepts and that it carries this C-ABI's
 * version; anything else is TILER_CUDA_PAYLOAD_REFUSED.  A module bound to a
 * context runs, for every launch on that context, the kernels it carries
 * (RMS norm f32 / bf16 / fused quantize, grouped sum and maximum) in place of
 * the library's built-in copies; unbind with NULL.  Unload only after unbinding
 * it from every context and after its launches have finished. */
typedef struct tiler_cuda_module tiler_cuda_module;
int32_t tiler_cuda_module_load(tiler_cuda_context* ctx, const void* code, uint64_t code_bytes,
                               tiler_cuda_module** out);
/* observe_prepared_entry for a module: TILER_CUDA_PAYLOAD_REFUSED when the
 * module does not carry the entry's kernel. */
int32_t tiler_cuda_module_entry(const tiler_cuda_module* module, const char* symbol,
                                tiler_cuda_entry_props* out);
int32_t tiler_cuda_context_bind_module(tiler_cuda_context* ctx, tiler_cuda_module* module);
/* Launches made from the module so far (evidence that its code is what ran). */
int32_t tiler_cuda_module_launch_count(const tiler_cuda_module* module, uint64_t* out);
int32_t tiler_cuda_module_unload(tiler_cuda_module* module);

/* ---- status word and completion (dispatch completion, adapter.rs:675-677) */
int32_t tiler_cuda_status_reset(void* stream, tiler_cuda_status* status_dev);
int32_t tiler_cuda_status_fetch(void* stream, const tiler_cuda_status* status_dev,
                                tiler_cuda_error* out); /* synchronizes `stream` */
int32_t tiler_cuda_status_decode(const tiler_cuda_status* status_host, tiler_cuda_error* out);
int32_t tiler_cuda_sync(void* stream, uint64_t timeout_ns);

/* ---- reductions ----------------------------------------------------------
 * x is [rows, count] row-major; out is [rows].  Sum: empty domain -> +0.0.
 * Maximum: identity-less, empty domain refused.  Results NaN-canonicalized. */

/* PhysicalImplementationProvider::propose for a reduction (frontier.rs:
 * 3828-4040): the grouping this backend declares for [rows, count]. */
int32_t tiler_cuda_plan_grouping(const tiler_cuda_context* ctx, uint64_t rows, uint64_t count,
                                 tiler_cuda_grouping* out);
/* The same proposal for a stated SM count, without a device (planning runs
 * on a build host in the reference: session::compile, session.rs:2587). */
int32_t tiler_cuda_plan_grouping_for(int32_t sm_count, uint64_t rows, uint64_t count, tiler_cuda_grouping* out);
/* allocate_dispatch (adapter.rs:672-674): workspace bytes the grouped fold
 * needs (partials + per-row completion tickets). */
uint64_t tiler_cuda_grouped_workspace_bytes(uint64_t rows, const tiler_cuda_grouping* g);
/* Grouped sum (tiler::strict-serial-sum-f32 realized under a declared
 * grouping; conformance against partitioned/cooperative references,
 * crates/tiler-conformance/src/serial_sum.rs:768-872). */
int32_t tiler_cuda_sum_f32(tiler_cuda_context* ctx, void* stream, const float* x, uint64_t rows,
                           uint64_t count, const tiler_cuda_grouping* g, void* workspace,
                           uint64_t workspace_bytes, float* out);
/* Governed maximum (maximum_f32 fold, softmax.rs:168-186; any grouping is
 * bit-exact). */
int32_t tiler_cuda_max_f32(tiler_cuda_context* ctx, void* stream, const float* x, uint64_t rows,
                           uint64_t count, const tiler_cuda_grouping* g, void* workspace,
                           uint64_t workspace_bytes, float* out);
/* No counterpart in the reference.  The grouped sum above for callers that
 * cannot allocate device memory (a host framework that plans every buffer
 * itself, a loop that must not call cudaMalloc): the partials and tickets
 * live in a fixed array inside the library (about 260 KB on every GPU that
 * loads it, kept until the process exits) instead of a caller workspace.
 * Limits: rows <= 1024 and rows * partitions <= 65536, else
 * TILER_CUDA_SHAPE_TOO_LARGE.  The first call on a device looks up the
 * array's device address (make it before any stream capture); calls that
 * overlap on the GPU share the array and race.  Allocates nothing. */
int32_t tiler_cuda_sum_f32_no_alloc(tiler_cuda_context* ctx, void* stream, const float* x, uint64_t rows,
                                    uint64_t count, const tiler_cuda_grouping* g, float* out);
/* The multi-GPU sum's exchange (the declared order: partition r = rank r's
 * shard, folded strictly in rank order as strict_partitioned_sum does,
 * evaluate.rs:749-832): `partial` [rows] is this rank's shard sum (e.g. from
 * tiler_cuda_sum_f32); it is stored over NVLink into slot `rank` of every
 * rank's exchange buffer (`buffers[q]`: rank q's buffer mapped in this
 * process, tiler_cuda_sum_exchange_buffer_bytes(rows) bytes, zeroed once);
 * each rank waits (bounded, ~1 s; a timeout is counted in `status` and the
 * result is NaN) for all W slots of this call and writes the fold to `out`.
 * `seq` starts at 1 and grows by one per call, the same on every rank; or
 * pass 0 on every call to use the call count kept in the buffer (the same
 * arguments then serve every call, e.g. from a captured CUDA graph).
 * world <= 8. */
uint64_t tiler_cuda_sum_exchange_buffer_bytes(uint64_t rows);
int32_t tiler_cuda_sum_f32_exchange(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* status,
                                    const float* partial, uint64_t rows, uint32_t rank, uint32_t world,
                                    void* const* buffers, uint32_t seq, float* out);
/* strict_sum, evaluate.rs:498-589 (one serial fold per row). */
int32_t tiler_cuda_strict_sum_f32(tiler_cuda_context* ctx, void* stream, const float* x,
                                  uint64_t rows, uint64_t count, float* out);
/* strict_partitioned_sum, evaluate.rs:749-832. */
int32_t tiler_cuda_partitioned_sum_f32(tiler_cuda_context* ctx, void* stream, const float* x,
                                       uint64_t rows, uint64_t count, uint64_t partitions,
                                       uint64_t per_partition, void* workspace,
                                       uint64_t workspace_bytes, float* out);
uint64_t tiler_cuda_partitioned_workspace_bytes(uint64_t rows, uint64_t partitions);
/* cooperative_grouped_sum, evaluate.rs:936-1158. */
int32_t tiler_cuda_cooperative_sum_f32(tiler_cuda_context* ctx, void* stream, const float* x,
                                       uint64_t rows, uint64_t count, uint64_t participants,
                                       uint64_t per_partition, uint64_t rounds,
                                       int32_t participant_major, float* out);

/* ---- row families -------------------------------------------------------- */
/* RmsNormF32Reference (rms_norm.rs:91-132, :453-489).  w is [extent] when
 * w_row_stride == 0 (the program's explicit broadcast) or [rows, extent]. */
int32_t tiler_cuda_rms_norm_f32(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* status,
                                const float* x,
                                const float* w, int64_t w_row_stride, uint64_t rows,
                                uint64_t extent, uint32_t eps_bits, float* y);
/* Config extension: bf16 x, w, y with the binary32 path in between. */
int32_t tiler_cuda_rms_norm_bf16(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* status,
                                 const uint16_t* x,
                                 const uint16_t* w, int64_t w_row_stride, uint64_t rows,
                                 uint64_t extent, uint32_t eps_bits, uint16_t* y);
/* RMS normalization of HOST rows: the dispatch path that uploads the
 * caller's input, launches and reads the output back
 * (prototypes/candle-metal-adapter/src/adapter.rs:1311-1384, allocate_dispatch
 * + dispatch), chunked so the upload of chunk i+1, the kernel on chunk i and
 * the download of chunk i-1 overlap (the copy engines are full duplex).
 * dtype 0 = f32, 1 = bf16.  x_host / y_host should be pinned (page-locked)
 * for the copies to run asynchronously; x_dev / y_dev are device buffers of
 * rows*extent elements owned by the caller (the library allocates nothing);
 * w is on the device ([extent], or [rows, extent] with w_row_stride =
 * extent).  chunk_rows 0 lets the library choose; at most 32 chunks.  The
 * whole operation is ordered after the work already on `stream`, and work
 * enqueued on `stream` afterwards sees y_host complete. */
int32_t tiler_cuda_rms_norm_host(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* status, int32_t dtype,
                                 const void* x_host, void* x_dev, const void* w, int64_t w_row_stride,
                                 uint64_t rows, uint64_t extent, uint32_t eps_bits, void* y_dev, void* y_host,
                                 uint64_t chunk_rows);
/* SoftmaxF32Reference (softmax.rs:99-137, :260-315) over the last axis.
 * causal_period > 0 adds -inf where col > (row_offset + row) % causal_period
 * (the program's upstream add-f32 of a broadcast mask, standard.rs:211-221). */
int32_t tiler_cuda_softmax_f32(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* status,
                               const float* x, uint64_t rows, uint64_t extent,
                               uint64_t causal_period, uint64_t row_offset, float* y);
/* Softmax of x + mask: the program's upstream add-f32 of a broadcast mask
 * tensor (standard.rs:211-221) followed by SoftmaxF32Reference, fused: row r
 * adds mask[(row_offset + r) mod mask_rows] (one rounding, NaN
 * canonicalized) and takes the softmax of the sum.  mask is f32
 * [mask_rows, extent] on the device.  With the block-causal 0 / -inf mask it
 * equals tiler_cuda_softmax_f32 with causal_period = mask_rows bit for bit.
 * Requires extent % 4 == 0, extent <= 8192, 16-byte aligned x, y, mask (else
 * UNSUPPORTED). */
int32_t tiler_cuda_softmax_masked_f32(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* status,
                                      const float* x, uint64_t rows, uint64_t extent, const float* mask,
                                      uint64_t mask_rows, uint64_t row_offset, float* y);
/* Strict-affine quantize, signed per-row extension of quantize
 * (quantization.rs:188-247, :404-430): scales[r] = max|x_r| / 127. */
int32_t tiler_cuda_quantize_i8_rows(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* status,
                                    const float* x, uint64_t rows, uint64_t extent, int8_t* codes,
                                    float* scales);
/* Fused RMS norm -> per-row int8 quantize (the "RMS norm -> quantize, one HBM
 * read" fusion): codes/scales equal tiler_cuda_quantize_i8_rows applied to
 * the y of tiler_cuda_rms_norm_f32 (rms_norm.rs:453-489, then
 * quantization.rs:188-247, :404-430), bit for bit, with the same refusals
 * (NaN y -> NAN_INPUT at its first column, scale not positive-normal ->
 * SCALE_DOMAIN); y itself is never written.  x, w 16-byte aligned, extent a
 * multiple of 4 (else UNSUPPORTED). */
int32_t tiler_cuda_rms_norm_quantize_i8(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* status,
                                        const float* x, const float* w, int64_t w_row_stride, uint64_t rows,
                                        uint64_t extent, uint32_t eps_bits, int8_t* codes, float* scales);
/* dequantize_one (quantization.rs:440-451) with zero point 0, per-row scale.
 * Decoding cannot fail on any input; `status` (nullable) only counts bounded
 * waits of the staged kernel that ran out (TILER_CUDA_TIMEOUT). */
int32_t tiler_cuda_dequantize_i8_rows(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* status,
                                      const int8_t* codes, const float* scales, uint64_t rows,
                                      uint64_t extent, float* y);
/* The reference's own per-tensor unsigned family (U4: maximum 15, U8: 255). */
int32_t tiler_cuda_quantize_affine_u8(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* status,
                                      const float* x, uint64_t n, uint32_t scale_bits,
                                      uint32_t zero_point, uint32_t maximum, uint8_t* codes);
int32_t tiler_cuda_dequantize_affine_u8(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* status,
                                        const uint8_t* codes, uint64_t n, uint32_t scale_bits,
                                        uint32_t zero_point, uint32_t maximum, float* y);

/* ---- elementwise maps -------------------------------------------------------- */
/* SiluF32Reference (silu.rs:78-180). */
int32_t tiler_cuda_silu_f32(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* status,
                            const float* x, uint64_t n, float* y);
/* multiply-f32 then add-f32 (standard.rs:105-120, evaluate.rs:448-485):
 * y = (x*a) + b, two roundings; a / b are device scalars when *_scalar != 0. */
int32_t tiler_cuda_scale_bias_f32(tiler_cuda_context* ctx, void* stream, const float* x, uint64_t n,
                                  const float* a, int32_t a_scalar, const float* b, int32_t b_scalar,
                                  float* y);

/* ---- gather (GatherF32Reference, structural.rs:513-606) -------------------
 * Copies row_bytes-sized rows table[ids[i]] -> out[i] bit-exactly.  ids are
 * int32 (ids_unsigned == 0; negative is out of range) or uint32. */
int32_t tiler_cuda_gather_rows(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* status,
                               const void* table, uint64_t table_rows, uint64_t row_bytes,
                               const void* ids, int32_t ids_unsigned, uint64_t n_ids, void* out);

/* ---- contraction --------------------------------------------------------------- */
/* TensorContractionF32Reference for `td,od->to` (contraction.rs:255-630):
 * strict fold, first-product seed, separate roundings.  A[m,k], B[n,k]. */
int32_t tiler_cuda_contract_f32(tiler_cuda_context* ctx, void* stream, const float* a, const float* b,
                                uint64_t m, uint64_t n, uint64_t k, float* c);
/* Config extension: bf16 A[m,k] x B[n,k] (both K-major) with binary32
 * accumulation on the tcgen05 tensor cores (TMEM accumulators, TMA operand
 * staging), epilogue 0 = none, 1 = SiLU (silu.rs:158-180), bf16 RNE output
 * C[m,n] with row stride ldc (elements).  m % 128 == 0, n % 256 == 0,
 * k % 64 == 0. */
int32_t tiler_cuda_gemm_bf16(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* status,
                             const uint16_t* a, const uint16_t* b, uint64_t m, uint64_t n, uint64_t k,
                             int32_t epilogue, uint16_t* c, uint64_t ldc);

/* Failure detection without a GPU fault: runs the bounded device wait every
 * kernel uses on an mbarrier phase that nothing completes, with a limit of
 * limit_ns (<= 2 s).  The wait gives up, counts a timeout in `status`
 * (tiler_cuda_status_decode then reports TILER_CUDA_TIMEOUT) and the kernel
 * returns with nothing in flight, so the context stays usable. */
int32_t tiler_cuda_bounded_wait_selftest(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* status,
                                         uint64_t limit_ns);

/* ---- multi-GPU: device buffers shared between the processes of one node ---- */
/* cudaIpc handle (64 bytes) of the allocation holding `ptr`, and ptr's offset
 * inside it. */
int32_t tiler_cuda_ipc_export(tiler_cuda_context* ctx, const void* ptr, uint8_t* handle, uint64_t* offset);
/* Maps a peer's exported buffer into this process: *out = base + offset. */
int32_t tiler_cuda_ipc_open(tiler_cuda_context* ctx, const uint8_t* handle, uint64_t offset, void** out);
int32_t tiler_cuda_ipc_close(tiler_cuda_context* ctx, void* ptr, uint64_t offset);
/* The N-sharded contraction with its all-gather fused into the epilogue
 * (the exchange step of the multi-GPU contraction; ncclAllGather is the
 * unfused form): rank `rank` computes C_rank = A x B_shard^T ([m, n_shard],
 * optional SiLU, bf16) and writes it into block `rank` of EVERY rank's block
 * buffer [world, m, n_shard]: its own through TMA stores, the peers' with
 * 16-byte stores over NVLink from the same staged boxes.  blocks[q] is rank
 * q's buffer as mapped in this process (tiler_cuda_ipc_open for q != rank).
 * The peers' blocks are complete once every rank's launch has completed:
 * follow it with a collective on the same stream (e.g. a one-element
 * all-reduce) before reading them.  world <= 8. */
int32_t tiler_cuda_gemm_bf16_allgather(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* status,
                                       const uint16_t* a, const uint16_t* b_shard, uint64_t m, uint64_t n_shard,
                                       uint64_t k, int32_t epilogue, uint32_t rank, uint32_t world,
                                       void* const* blocks);
/* The same exchange through an NVLink multicast mapping of every rank's
 * [world, m, n_shard] buffer (NVSwitch replicates each store to every bound
 * GPU): `local_buffer` is this rank's buffer, `multicast_buffer` the multicast
 * address of the same buffer (e.g. torch symmetric memory's multicast_ptr).
 * Each output box crosses NVLink once instead of once per peer.  The same two
 * ordering collectives as above apply. */
int32_t tiler_cuda_gemm_bf16_allgather_multicast(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* status,
                                                 const uint16_t* a, const uint16_t* b_shard, uint64_t m,
                                                 uint64_t n_shard, uint64_t k, int32_t epilogue, uint32_t rank,
                                                 uint32_t world, void* local_buffer, void* multicast_buffer);

#ifdef __cplusplus
}
#endif
#endif /* TILER_CUDA_H */
