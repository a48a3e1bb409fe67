// The C-ABI (include/tiler_cuda.h): execution context, device facts, payload
// validation and entry queries, the status word, the grouping provider and
// one validated launch wrapper per family.  Argument refusals return before
// anything is enqueued; nothing here allocates device memory.
#include <quadmath.h>
#include <string.h>
#include <time.h>

#include <mutex>
#include <vector>

#include "common.cuh"
#include "kernels.h"
#include "launch.cuh"

struct tiler_cuda_context {
  int device;
  tiler_cuda_device_facts facts;
  // copy streams and events of the host-buffer entry points (made on first use)
  cudaStream_t copy_in = nullptr, copy_out = nullptr;
  cudaEvent_t ev[2 * 32 + 2] = {};
  tiler_cuda_module* module = nullptr;  // bound payload module (launches run its kernels)
};

namespace {

using namespace tc;

std::mutex g_init_mutex;
std::vector<bool> g_table_ready;

// 2^(j/256) as a double-double (hi + lo, |error| < 2^-106), computed in
// binary128 and written once per device into g_exp2_table.
struct Exp2Table {
  double pairs[256][2];
  double hi[256];
};

const Exp2Table& exp2_table_host() {
  static const Exp2Table t = [] {
    Exp2Table e;
    for (int j = 0; j < 256; ++j) {
      __float128 v = exp2q((__float128)j / 256);
      double hi = (double)v;
      e.pairs[j][0] = hi;
      e.pairs[j][1] = (double)(v - (__float128)hi);
      e.hi[j] = hi;
    }
    return e;
  }();
  return t;
}

int init_exp_table(int device) {
  std::lock_guard<std::mutex> lock(g_init_mutex);
  if ((int)g_table_ready.size() <= device) g_table_ready.resize(device + 1, false);
  if (g_table_ready[device]) return TILER_CUDA_OK;
  const Exp2Table& t = exp2_table_host();
  if (cudaMemcpyToSymbol(g_exp2_table, t.pairs, sizeof(t.pairs)) != cudaSuccess) return TILER_CUDA_DEVICE_ERROR;
  if (cudaMemcpyToSymbol(g_exp2_hi, t.hi, sizeof(t.hi)) != cudaSuccess) return TILER_CUDA_DEVICE_ERROR;
  g_table_ready[device] = true;
  return TILER_CUDA_OK;
}

int32_t last_error_status() {
  cudaError_t e = cudaGetLastError();
  const bool module_failed = tl_module_launch_failed;
  tl_module_launch_failed = false;
  return e == cudaSuccess && !module_failed ? TILER_CUDA_OK : TILER_CUDA_DEVICE_ERROR;
}

bool bind(const tiler_cuda_context* ctx) {
  tl_module = ctx->module;
  int cur = -1;
  cudaGetDevice(&cur);
  if (cur != ctx->device) return cudaSetDevice(ctx->device) == cudaSuccess;
  return true;
}

#define CHECK_CTX(ctx)                                              \
  do {                                                              \
    if (!(ctx)) return TILER_CUDA_INVALID_APPLICATION;              \
    if (!bind(ctx)) return TILER_CUDA_DEVICE_ERROR;                 \
  } while (0)

cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }

bool canonical_composition(uint64_t n, uint32_t T, uint32_t k, uint32_t R) {
  if (T == 0 || T % 32 || T > 1024 || k == 0 || R == 0 || n == 0) return false;
  const uint64_t per_round = (uint64_t)T * k;
  return per_round * (R - 1) < n && n <= per_round * R;
}

constexpr uint64_t kMaxSlotFloats = 12 * 1024;  // 48 KB of staged warp slots

int32_t validate_grouping(uint64_t rows, uint64_t count, const tiler_cuda_grouping* g, uint64_t workspace_bytes,
                          const void* workspace) {
  if (!g || g->partitions == 0 || count % g->partitions) return TILER_CUDA_INVALID_APPLICATION;
  const uint64_t per = count / g->partitions;
  if (!canonical_composition(per, g->threads, g->k, g->rounds)) return TILER_CUDA_INVALID_APPLICATION;
  if (g->k != 1 && g->k != 2 && g->k != 4) return TILER_CUDA_UNSUPPORTED;
  if ((uint64_t)g->rounds * (g->threads / 32 + 1) > kMaxSlotFloats) return TILER_CUDA_UNSUPPORTED;
  if (g->combine_threads) {
    if (g->combine_threads > g->threads ||
        !canonical_composition(g->partitions, g->combine_threads, g->combine_k, g->combine_rounds))
      return TILER_CUDA_INVALID_APPLICATION;
    if ((uint64_t)g->combine_rounds * (g->combine_threads / 32 + 1) > kMaxSlotFloats) return TILER_CUDA_UNSUPPORTED;
  }
  if (rows && g->partitions > 0x7fffffffull / rows) return TILER_CUDA_SHAPE_TOO_LARGE;
  if (g->partitions > 1) {
    if (!workspace) return TILER_CUDA_INVALID_APPLICATION;
    if (workspace_bytes < tiler_cuda_grouped_workspace_bytes(rows, g)) return TILER_CUDA_WORKSPACE_TOO_SMALL;
    if ((uintptr_t)workspace % 16) return TILER_CUDA_INVALID_APPLICATION;
  }
  return TILER_CUDA_OK;
}

// Family registry: the entry symbols a payload may name.
struct Entry {
  const char* symbol;
  const void* func;
  int threads;
  size_t smem;
  const char* kernel = nullptr;  // C name of the kernel a payload module carries for it (or none)
};

const Entry kEntries[] = {
    {"tiler_cuda.sum_f32.grouped", (const void*)tiler_grouped_sum_k4, 512, 0, "tiler_grouped_sum_k4"},
    {"tiler_cuda.max_f32.grouped", (const void*)tiler_grouped_max_k4, 512, 0, "tiler_grouped_max_k4"},
    {"tiler_cuda.sum_f32.strict", (const void*)serial_folds_kernel<true>, kSerialFoldThreads, 0},
    {"tiler_cuda.sum_f32.partitioned", (const void*)serial_folds_kernel<false>, kSerialFoldThreads, 0},
    {"tiler_cuda.sum_f32.cooperative", (const void*)cooperative_sum_kernel, 1024, 0},
    {"tiler_cuda.rms_norm_f32", (const void*)tiler_rms_norm_stream_f32, RmsStreamF32::kThreads,
     rms_stream_smem_bytes<RmsStreamF32>(), "tiler_rms_norm_stream_f32"},
    {"tiler_cuda.rms_norm_bf16", (const void*)tiler_rms_norm_stream_bf16, RmsStreamBF16::kThreads,
     rms_stream_smem_bytes<RmsStreamBF16>(), "tiler_rms_norm_stream_bf16"},
    {"tiler_cuda.softmax_f32", (const void*)softmax_group_kernel, 32 * 7, 2048 + 256 + 6 * 8192},
    {"tiler_cuda.quantize_i8_rows", (const void*)quantize_i8_rows_kernel, kQThreads, 0},
    {"tiler_cuda.rms_norm_quantize_i8", (const void*)tiler_rms_norm_wave_quantize_i8, kRmsThreads, kRmsSmemBytes,
     "tiler_rms_norm_wave_quantize_i8"},
    {"tiler_cuda.softmax_masked_f32", (const void*)softmax_group_kernel, 32 * 7, 2048 + 256 + 6 * 8192},
    {"tiler_cuda.dequantize_i8_rows", (const void*)dequantize_i8_rows_kernel, 256, 0},
    {"tiler_cuda.quantize_affine_u8", (const void*)quantize_affine_u8_kernel, 256, 0},
    {"tiler_cuda.dequantize_affine_u8", (const void*)dequantize_affine_u8_kernel, 256, 0},
    {"tiler_cuda.silu_f32", (const void*)silu_kernel, 256, 0},
    {"tiler_cuda.scale_bias_f32", (const void*)scale_bias_kernel, 256, 0},
    {"tiler_cuda.gather_rows", (const void*)gather_rows_kernel, 256, 0},
    {"tiler_cuda.contract_f32", (const void*)contract_f32_kernel, 256, 0},
    {"tiler_cuda.gemm_bf16", (const void*)gemm_bf16_tcgen05_kernel, kGemmThreads, kGemmSmem},
};
constexpr uint32_t kEntryCount = sizeof(kEntries) / sizeof(kEntries[0]);

const Entry* find_entry(const char* symbol) {
  if (!symbol) return nullptr;
  for (uint32_t i = 0; i < kEntryCount; ++i)
    if (strcmp(kEntries[i].symbol, symbol) == 0) return &kEntries[i];
  return nullptr;
}

}  // namespace

extern "C" {

uint32_t tiler_cuda_abi_version(void) { return TILER_CUDA_ABI_VERSION; }

const char* tiler_cuda_status_string(int32_t code) {
  switch (code) {
    case TILER_CUDA_OK: return "ok";
    case TILER_CUDA_INVALID_APPLICATION: return "invalid application";
    case TILER_CUDA_SHAPE_TOO_LARGE: return "shape too large";
    case TILER_CUDA_GATHER_INDEX_OUT_OF_BOUNDS: return "gather index out of bounds";
    case TILER_CUDA_NAN_INPUT: return "NaN input refused";
    case TILER_CUDA_UNDECIDED: return "undecided transcendental reference";
    case TILER_CUDA_DEVICE_ERROR: return "device error";
    case TILER_CUDA_TIMEOUT: return "timeout";
    case TILER_CUDA_UNSUPPORTED: return "unsupported";
    case TILER_CUDA_SCALE_DOMAIN: return "scale outside positive-normal";
    case TILER_CUDA_PAYLOAD_REFUSED: return "payload refused";
    case TILER_CUDA_WORKSPACE_TOO_SMALL: return "workspace too small";
    default: return "unknown status";
  }
}

int32_t tiler_cuda_context_create(int32_t device, tiler_cuda_context** out) {
  if (!out) return TILER_CUDA_INVALID_APPLICATION;
  *out = nullptr;
  int n = 0;
  if (cudaGetDeviceCount(&n) != cudaSuccess || device < 0 || device >= n) return TILER_CUDA_DEVICE_ERROR;
  if (cudaSetDevice(device) != cudaSuccess) return TILER_CUDA_DEVICE_ERROR;
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, device) != cudaSuccess) return TILER_CUDA_DEVICE_ERROR;
  auto* ctx = new tiler_cuda_context();
  ctx->device = device;
  tiler_cuda_device_facts& f = ctx->facts;
  f.device = device;
  f.cc_major = p.major;
  f.cc_minor = p.minor;
  f.sm_count = p.multiProcessorCount;
  f.warp_size = p.warpSize;
  f.max_threads_per_block = p.maxThreadsPerBlock;
  f.smem_per_block_optin = (int64_t)p.sharedMemPerBlockOptin;
  f.l2_bytes = p.l2CacheSize;
  f.global_mem_bytes = (int64_t)p.totalGlobalMem;
  strncpy(f.name, p.name, sizeof(f.name) - 1);
  int32_t st = init_exp_table(device);
  if (st != TILER_CUDA_OK) {
    delete ctx;
    return st;
  }
  *out = ctx;
  return TILER_CUDA_OK;
}

int32_t tiler_cuda_context_destroy(tiler_cuda_context* ctx) {
  if (ctx && ctx->copy_in) {
    int cur = -1;
    cudaGetDevice(&cur);
    cudaSetDevice(ctx->device);
    cudaStreamSynchronize(ctx->copy_in);
    cudaStreamSynchronize(ctx->copy_out);
    for (cudaEvent_t e : ctx->ev)
      if (e) cudaEventDestroy(e);
    cudaStreamDestroy(ctx->copy_in);
    cudaStreamDestroy(ctx->copy_out);
    if (cur >= 0) cudaSetDevice(cur);
  }
  delete ctx;
  return TILER_CUDA_OK;
}

int32_t tiler_cuda_device_facts_query(const tiler_cuda_context* ctx, tiler_cuda_device_facts* out) {
  if (!ctx || !out) return TILER_CUDA_INVALID_APPLICATION;
  *out = ctx->facts;
  return TILER_CUDA_OK;
}

uint32_t tiler_cuda_entry_count(void) { return kEntryCount; }

const char* tiler_cuda_entry_symbol(uint32_t index) { return index < kEntryCount ? kEntries[index].symbol : nullptr; }

int32_t tiler_cuda_payload_validate(const tiler_cuda_context* ctx, const char* target, uint32_t subgroup_width,
                                    const char* const* symbols, uint32_t n_symbols, uint32_t* refused_index) {
  if (refused_index) *refused_index = UINT32_MAX;
  if (!ctx || !target) return TILER_CUDA_INVALID_APPLICATION;
  // The compiled code is sm_100a: it runs on compute capability 10.0 only.
  if (strcmp(target, "sm_100a") != 0 || ctx->facts.cc_major != 10 || ctx->facts.cc_minor != 0)
    return TILER_CUDA_PAYLOAD_REFUSED;
  // The subgroup width is an equality, never a floor (ADR 0094 decision 7).
  if (subgroup_width != 32 || ctx->facts.warp_size != 32) return TILER_CUDA_PAYLOAD_REFUSED;
  for (uint32_t i = 0; i < n_symbols; ++i) {
    if (!find_entry(symbols ? symbols[i] : nullptr)) {
      if (refused_index) *refused_index = i;
      return TILER_CUDA_PAYLOAD_REFUSED;
    }
  }
  return TILER_CUDA_OK;
}

int32_t tiler_cuda_entry_query(const tiler_cuda_context* ctx, const char* symbol, tiler_cuda_entry_props* out) {
  CHECK_CTX(ctx);
  const Entry* e = find_entry(symbol);
  if (!e || !out) return TILER_CUDA_INVALID_APPLICATION;
  cudaFuncAttributes a;
  if (cudaFuncGetAttributes(&a, e->func) != cudaSuccess) return TILER_CUDA_DEVICE_ERROR;
  out->num_regs = a.numRegs;
  out->max_threads_per_block = a.maxThreadsPerBlock;
  out->static_smem_bytes = (int64_t)a.sharedSizeBytes;
  out->dynamic_smem_bytes = (int64_t)e->smem;
  out->threads_per_block = e->threads;
  out->pad = 0;
  return TILER_CUDA_OK;
}

// ---- payload code: load, prepare, bind ----------------------------------------

int32_t tiler_cuda_module_load(tiler_cuda_context* ctx, const void* code, uint64_t code_bytes,
                               tiler_cuda_module** out) {
  if (out) *out = nullptr;
  CHECK_CTX(ctx);
  if (!out || !code) return TILER_CUDA_INVALID_APPLICATION;
  // an ELF image (a cubin); anything else is refused before the driver sees it
  if (code_bytes < 64 || memcmp(code, "\x7f" "ELF", 4) != 0) return TILER_CUDA_PAYLOAD_REFUSED;
  const ModuleDriver& d = module_driver();
  if (!d.ok) return TILER_CUDA_DEVICE_ERROR;
  if (cudaFree(nullptr) != cudaSuccess) return TILER_CUDA_DEVICE_ERROR;  // the device's context is current
  CUcontext cur = nullptr;
  if (d.ctx_current(&cur) != CUDA_SUCCESS || !cur) return TILER_CUDA_DEVICE_ERROR;
  CUmodule mod = nullptr;
  // code for another architecture, or not a loadable image: refused
  if (d.load(&mod, code) != CUDA_SUCCESS) return TILER_CUDA_PAYLOAD_REFUSED;
  auto refuse = [&](int32_t st) {
    d.unload(mod);
    return st;
  };
  // provenance: the module was built from this library's sources, for this C-ABI
  CUdeviceptr abi_ptr = 0;
  size_t abi_size = 0;
  uint32_t abi = 0;
  if (d.get_global(&abi_ptr, &abi_size, mod, "tiler_cuda_payload_abi") != CUDA_SUCCESS || abi_size != 4 ||
      d.memcpy_dtoh(&abi, abi_ptr, 4) != CUDA_SUCCESS || abi != TILER_CUDA_ABI_VERSION)
    return refuse(TILER_CUDA_PAYLOAD_REFUSED);
  // the module's own copy of the certified-exp table
  const Exp2Table& t = exp2_table_host();
  CUdeviceptr tp = 0, hp = 0;
  size_t tsz = 0, hsz = 0;
  if (d.get_global(&tp, &tsz, mod, "g_exp2_table") == CUDA_SUCCESS && tsz == sizeof(t.pairs) &&
      d.memcpy_htod(tp, t.pairs, sizeof(t.pairs)) != CUDA_SUCCESS)
    return refuse(TILER_CUDA_DEVICE_ERROR);
  if (d.get_global(&hp, &hsz, mod, "g_exp2_hi") == CUDA_SUCCESS && hsz == sizeof(t.hi) &&
      d.memcpy_htod(hp, t.hi, sizeof(t.hi)) != CUDA_SUCCESS)
    return refuse(TILER_CUDA_DEVICE_ERROR);
  auto* m = new tiler_cuda_module();
  m->device = ctx->device;
  m->cu_ctx = cur;
  m->mod = mod;
  for (int i = 0; i < kModuleKernelCount; ++i) {
    CUfunction f = nullptr;
    m->fn[i] = d.get_function(&f, mod, kModuleKernels[i]) == CUDA_SUCCESS ? f : nullptr;
    m->smem_allowed[i] = 48 * 1024;
  }
  *out = m;
  return TILER_CUDA_OK;
}

int32_t tiler_cuda_module_entry(const tiler_cuda_module* m, const char* symbol, tiler_cuda_entry_props* out) {
  if (!m || !out) return TILER_CUDA_INVALID_APPLICATION;
  const Entry* e = find_entry(symbol);
  if (!e) return TILER_CUDA_INVALID_APPLICATION;
  const int i = e->kernel ? module_kernel_index(e->kernel) : -1;
  if (i < 0 || !m->fn[i]) return TILER_CUDA_PAYLOAD_REFUSED;  // the module does not carry this entry
  const ModuleDriver& d = module_driver();
  int regs = 0, maxt = 0, ssmem = 0;
  if (d.func_get_attribute(&regs, CU_FUNC_ATTRIBUTE_NUM_REGS, m->fn[i]) != CUDA_SUCCESS ||
      d.func_get_attribute(&maxt, CU_FUNC_ATTRIBUTE_MAX_THREADS_PER_BLOCK, m->fn[i]) != CUDA_SUCCESS ||
      d.func_get_attribute(&ssmem, CU_FUNC_ATTRIBUTE_SHARED_SIZE_BYTES, m->fn[i]) != CUDA_SUCCESS)
    return TILER_CUDA_DEVICE_ERROR;
  out->num_regs = regs;
  out->max_threads_per_block = maxt;
  out->static_smem_bytes = ssmem;
  out->dynamic_smem_bytes = (int64_t)e->smem;
  out->threads_per_block = e->threads;
  out->pad = 0;
  return TILER_CUDA_OK;
}

int32_t tiler_cuda_context_bind_module(tiler_cuda_context* ctx, tiler_cuda_module* m) {
  if (!ctx) return TILER_CUDA_INVALID_APPLICATION;
  if (m && m->device != ctx->device) return TILER_CUDA_INVALID_APPLICATION;
  ctx->module = m;
  if (!m) tl_module = nullptr;
  return TILER_CUDA_OK;
}

int32_t tiler_cuda_module_launch_count(const tiler_cuda_module* m, uint64_t* out) {
  if (!m || !out) return TILER_CUDA_INVALID_APPLICATION;
  *out = m->launches.load();
  return TILER_CUDA_OK;
}

int32_t tiler_cuda_module_unload(tiler_cuda_module* m) {
  if (!m) return TILER_CUDA_OK;
  if (tl_module == m) tl_module = nullptr;
  const ModuleDriver& d = module_driver();
  const CUresult r = d.unload(m->mod);
  delete m;
  return r == CUDA_SUCCESS ? TILER_CUDA_OK : TILER_CUDA_DEVICE_ERROR;
}

int32_t tiler_cuda_status_reset(void* stream, tiler_cuda_status* status_dev) {
  if (!status_dev) return TILER_CUDA_INVALID_APPLICATION;
  launch_status_reset(status_dev, S(stream));
  return last_error_status();
}

int32_t tiler_cuda_status_decode(const tiler_cuda_status* s, tiler_cuda_error* out) {
  if (!s || !out) return TILER_CUDA_INVALID_APPLICATION;
  memset(out, 0, sizeof(*out));
  out->undecided = s->undecided;
  out->timeouts = s->timeouts;
  if (s->error_key != UINT64_MAX) {
    out->code = (int32_t)(s->error_key & 0xff);
    out->position = s->error_key >> 8;
    if (out->code == TILER_CUDA_GATHER_INDEX_OUT_OF_BOUNDS && s->value_key != UINT64_MAX)
      out->value = (int64_t)(int32_t)(uint32_t)(s->value_key & 0xffffffffu);
  } else if (s->timeouts) {
    out->code = TILER_CUDA_TIMEOUT;
  } else if (s->undecided) {
    out->code = TILER_CUDA_UNDECIDED;
  }
  return out->code;
}

int32_t tiler_cuda_status_fetch(void* stream, const tiler_cuda_status* status_dev, tiler_cuda_error* out) {
  if (!status_dev || !out) return TILER_CUDA_INVALID_APPLICATION;
  tiler_cuda_status host;
  if (cudaMemcpyAsync(&host, status_dev, sizeof(host), cudaMemcpyDeviceToHost, S(stream)) != cudaSuccess)
    return TILER_CUDA_DEVICE_ERROR;
  if (cudaStreamSynchronize(S(stream)) != cudaSuccess) return TILER_CUDA_DEVICE_ERROR;
  return tiler_cuda_status_decode(&host, out);
}

int32_t tiler_cuda_sync(void* stream, uint64_t timeout_ns) {
  timespec t0;
  clock_gettime(CLOCK_MONOTONIC, &t0);
  for (;;) {
    cudaError_t e = cudaStreamQuery(S(stream));
    if (e == cudaSuccess) return TILER_CUDA_OK;
    if (e != cudaErrorNotReady) return TILER_CUDA_DEVICE_ERROR;
    timespec t1;
    clock_gettime(CLOCK_MONOTONIC, &t1);
    uint64_t el = (uint64_t)(t1.tv_sec - t0.tv_sec) * 1000000000ull + (uint64_t)(t1.tv_nsec - t0.tv_nsec);
    if (timeout_ns && el > timeout_ns) return TILER_CUDA_TIMEOUT;
    timespec nap = {0, 20000};
    nanosleep(&nap, nullptr);
  }
}

// ---- reductions --------------------------------------------------------------

int32_t tiler_cuda_plan_grouping_for(int32_t sm_count, uint64_t rows, uint64_t count, tiler_cuda_grouping* out) {
  if (sm_count <= 0 || !out || count == 0) return TILER_CUDA_INVALID_APPLICATION;
  const uint32_t T = 512, k = 4;
  const uint64_t per_round = (uint64_t)T * k;
  // Partitions: an exact divisor of count, aiming at 32 rounds per partition
  // and at least two CTAs per SM across all rows (2^24 contributors: 256
  // partitions measured 18.4 us against 19.4 us for 512 and 22.5 us for 1024).
  const uint64_t target_per = per_round * 32;
  uint64_t want = std::max<uint64_t>(1, count / target_per);
  const uint64_t min_ctas = 2ull * (uint64_t)sm_count;
  if (rows * want < min_ctas) want = std::max<uint64_t>(want, std::min<uint64_t>(count / per_round, (min_ctas + rows - 1) / rows));
  uint64_t best = 1;
  for (uint64_t d = std::max<uint64_t>(want, 1); d >= 1; --d)
    if (count % d == 0) { best = d; break; }
  const uint64_t per = count / best;
  const uint64_t R = (per + per_round - 1) / per_round;
  if (R * (T / 32 + 1) > kMaxSlotFloats) return TILER_CUDA_UNSUPPORTED;
  out->partitions = best;
  out->threads = T;
  out->k = k;
  out->rounds = (uint32_t)R;
  if (best >= 64) {
    const uint32_t k2 = best >= 1024 ? 4 : 2;
    uint64_t t2 = ((best + k2 - 1) / k2 + 31) / 32 * 32;
    t2 = std::min<uint64_t>(t2, T);
    out->combine_threads = (uint32_t)t2;
    out->combine_k = k2;
    out->combine_rounds = (uint32_t)((best + t2 * k2 - 1) / (t2 * k2));
  } else {
    out->combine_threads = out->combine_k = out->combine_rounds = 0;
  }
  return TILER_CUDA_OK;
}

int32_t tiler_cuda_plan_grouping(const tiler_cuda_context* ctx, uint64_t rows, uint64_t count,
                                 tiler_cuda_grouping* out) {
  if (!ctx) return TILER_CUDA_INVALID_APPLICATION;
  return tiler_cuda_plan_grouping_for(ctx->facts.sm_count, rows, count, out);
}

uint64_t tiler_cuda_grouped_workspace_bytes(uint64_t rows, const tiler_cuda_grouping* g) {
  if (!g || g->partitions <= 1) return 0;
  const uint64_t partial_bytes = (rows * g->partitions * 4 + 255) / 256 * 256;
  return partial_bytes + rows * 4;
}

static int32_t grouped(int op, tiler_cuda_context* ctx, void* stream, const float* x, uint64_t rows, uint64_t count,
                       const tiler_cuda_grouping* g, void* ws, uint64_t ws_bytes, float* out) {
  CHECK_CTX(ctx);
  if (!x || !out) return TILER_CUDA_INVALID_APPLICATION;
  if (rows == 0) return TILER_CUDA_OK;
  if (count == 0) {
    if (op == 1) return TILER_CUDA_INVALID_APPLICATION;  // the maximum has no identity
    launch_strict_sum(x, rows, 0, out, S(stream));
    return last_error_status();
  }
  int32_t v = validate_grouping(rows, count, g, ws_bytes, ws);
  if (v != TILER_CUDA_OK) return v;
  GroupedParams gp{g->partitions, g->threads, g->k, g->rounds, g->combine_threads, g->combine_k, g->combine_rounds};
  float* partials = (float*)ws;
  unsigned int* tickets =
      ws ? (unsigned int*)((uint8_t*)ws + (rows * g->partitions * 4 + 255) / 256 * 256) : nullptr;
  launch_grouped_fold(op, x, rows, count, gp, partials, tickets, out, S(stream));
  return last_error_status();
}

int32_t tiler_cuda_sum_f32(tiler_cuda_context* ctx, void* stream, const float* x, uint64_t rows, uint64_t count,
                           const tiler_cuda_grouping* g, void* ws, uint64_t ws_bytes, float* out) {
  return grouped(0, ctx, stream, x, rows, count, g, ws, ws_bytes, out);
}

int32_t tiler_cuda_max_f32(tiler_cuda_context* ctx, void* stream, const float* x, uint64_t rows, uint64_t count,
                           const tiler_cuda_grouping* g, void* ws, uint64_t ws_bytes, float* out) {
  return grouped(1, ctx, stream, x, rows, count, g, ws, ws_bytes, out);
}

int32_t tiler_cuda_strict_sum_f32(tiler_cuda_context* ctx, void* stream, const float* x, uint64_t rows,
                                  uint64_t count, float* out) {
  CHECK_CTX(ctx);
  if ((!x && rows * count) || (!out && rows)) return TILER_CUDA_INVALID_APPLICATION;
  if (rows == 0) return TILER_CUDA_OK;
  launch_strict_sum(x, rows, count, out, S(stream));
  return last_error_status();
}

uint64_t tiler_cuda_partitioned_workspace_bytes(uint64_t rows, uint64_t partitions) {
  return rows * partitions * 4;
}

int32_t tiler_cuda_partitioned_sum_f32(tiler_cuda_context* ctx, void* stream, const float* x, uint64_t rows,
                                       uint64_t count, uint64_t partitions, uint64_t per, void* ws,
                                       uint64_t ws_bytes, float* out) {
  CHECK_CTX(ctx);
  if (partitions == 0 || partitions * per != count) return TILER_CUDA_INVALID_APPLICATION;
  if (rows == 0) return TILER_CUDA_OK;
  if (!x || !out || !ws) return TILER_CUDA_INVALID_APPLICATION;
  if (ws_bytes < tiler_cuda_partitioned_workspace_bytes(rows, partitions)) return TILER_CUDA_WORKSPACE_TOO_SMALL;
  launch_partitioned_sum(x, rows, count, partitions, per, (float*)ws, out, S(stream));
  return last_error_status();
}

int32_t tiler_cuda_cooperative_sum_f32(tiler_cuda_context* ctx, void* stream, const float* x, uint64_t rows,
                                       uint64_t count, uint64_t participants, uint64_t per, uint64_t rounds,
                                       int32_t participant_major, float* out) {
  CHECK_CTX(ctx);
  if (participants == 0 || per == 0 || rounds == 0 || participants * per * rounds != count)
    return TILER_CUDA_INVALID_APPLICATION;
  if (participants > 12288) return TILER_CUDA_UNSUPPORTED;
  if (rows == 0) return TILER_CUDA_OK;
  if (!x || !out) return TILER_CUDA_INVALID_APPLICATION;
  launch_cooperative_sum(x, rows, count, participants, per, rounds, participant_major, out, S(stream));
  return last_error_status();
}

// ---- row families --------------------------------------------------------------

static bool eps_admitted(uint32_t bits) {
  float e;
  memcpy(&e, &bits, 4);
  return e > 0.0f && e <= 3.40282347e38f;  // positive, finite (rms_norm.rs:465-467)
}

static int32_t rms(int bf16, tiler_cuda_context* ctx, void* stream, tiler_cuda_status* st, const void* x,
                   const void* w, int64_t w_row_stride, uint64_t rows, uint64_t extent, uint32_t eps_bits, void* y) {
  CHECK_CTX(ctx);
  if (!eps_admitted(eps_bits) || w_row_stride < 0) return TILER_CUDA_INVALID_APPLICATION;
  if (extent > (1ull << 24)) return TILER_CUDA_SHAPE_TOO_LARGE;
  if (rows == 0 || extent == 0) return TILER_CUDA_OK;
  if (!x || !w || !y) return TILER_CUDA_INVALID_APPLICATION;
  if (w_row_stride != 0 && (uint64_t)w_row_stride != extent) return TILER_CUDA_UNSUPPORTED;
  float eps;
  memcpy(&eps, &eps_bits, 4);
  launch_rms_norm(bf16, x, w, w_row_stride, rows, extent, eps, y, st, ctx->facts.sm_count, S(stream));
  return last_error_status();
}

int32_t tiler_cuda_rms_norm_f32(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* st, const float* x,
                                const float* w, int64_t w_row_stride, uint64_t rows, uint64_t extent,
                                uint32_t eps_bits, float* y) {
  return rms(0, ctx, stream, st, x, w, w_row_stride, rows, extent, eps_bits, y);
}

static int32_t ensure_copy_streams(tiler_cuda_context* ctx) {
  if (ctx->copy_in) return TILER_CUDA_OK;
  if (cudaStreamCreateWithFlags(&ctx->copy_in, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&ctx->copy_out, cudaStreamNonBlocking) != cudaSuccess)
    return TILER_CUDA_DEVICE_ERROR;
  for (cudaEvent_t& e : ctx->ev)
    if (cudaEventCreateWithFlags(&e, cudaEventDisableTiming) != cudaSuccess) return TILER_CUDA_DEVICE_ERROR;
  return TILER_CUDA_OK;
}

int32_t tiler_cuda_rms_norm_host(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* st, int32_t dtype,
                                 const void* x_host, void* x_dev, const void* w, int64_t w_row_stride,
                                 uint64_t rows, uint64_t extent, uint32_t eps_bits, void* y_dev, void* y_host,
                                 uint64_t chunk_rows) {
  CHECK_CTX(ctx);
  if (dtype != 0 && dtype != 1) return TILER_CUDA_UNSUPPORTED;
  if (!eps_admitted(eps_bits) || w_row_stride < 0) return TILER_CUDA_INVALID_APPLICATION;
  if (extent > (1ull << 24)) return TILER_CUDA_SHAPE_TOO_LARGE;
  if (rows == 0 || extent == 0) return TILER_CUDA_OK;
  if (!x_host || !x_dev || !w || !y_dev || !y_host) return TILER_CUDA_INVALID_APPLICATION;
  if (w_row_stride != 0 && (uint64_t)w_row_stride != extent) return TILER_CUDA_UNSUPPORTED;
  int32_t r = ensure_copy_streams(ctx);
  if (r != TILER_CUDA_OK) return r;
  constexpr uint64_t kMaxChunks = 32;
  if (chunk_rows == 0) chunk_rows = std::max<uint64_t>(1, (rows + 7) / 8);
  chunk_rows = std::max(chunk_rows, (rows + kMaxChunks - 1) / kMaxChunks);
  const uint64_t esize = dtype ? 2 : 4, row_bytes = extent * esize;
  float eps;
  memcpy(&eps, &eps_bits, 4);
  cudaStream_t s = S(stream);
  cudaEvent_t* ev = ctx->ev;
  // everything below runs after the work already on `stream`
  if (cudaEventRecord(ev[0], s) != cudaSuccess || cudaStreamWaitEvent(ctx->copy_in, ev[0], 0) != cudaSuccess)
    return TILER_CUDA_DEVICE_ERROR;
  uint32_t k = 0;
  for (uint64_t r0 = 0; r0 < rows; r0 += chunk_rows, ++k) {
    const uint64_t n = std::min(chunk_rows, rows - r0);
    const uint64_t off = r0 * row_bytes, bytes = n * row_bytes;
    cudaEvent_t in_done = ev[2 + 2 * k], out_ready = ev[3 + 2 * k];
    if (cudaMemcpyAsync((uint8_t*)x_dev + off, (const uint8_t*)x_host + off, bytes, cudaMemcpyHostToDevice,
                        ctx->copy_in) != cudaSuccess ||
        cudaEventRecord(in_done, ctx->copy_in) != cudaSuccess || cudaStreamWaitEvent(s, in_done, 0) != cudaSuccess)
      return TILER_CUDA_DEVICE_ERROR;
    const uint8_t* wc = (const uint8_t*)w + (w_row_stride ? off : 0);
    launch_rms_norm(dtype, (const uint8_t*)x_dev + off, wc, w_row_stride, n, extent, eps, (uint8_t*)y_dev + off, st,
                    ctx->facts.sm_count, s);
    if (cudaEventRecord(out_ready, s) != cudaSuccess || cudaStreamWaitEvent(ctx->copy_out, out_ready, 0) != cudaSuccess ||
        cudaMemcpyAsync((uint8_t*)y_host + off, (const uint8_t*)y_dev + off, bytes, cudaMemcpyDeviceToHost,
                        ctx->copy_out) != cudaSuccess)
      return TILER_CUDA_DEVICE_ERROR;
  }
  // work enqueued on `stream` afterwards sees every chunk downloaded
  if (cudaEventRecord(ev[1], ctx->copy_out) != cudaSuccess || cudaStreamWaitEvent(s, ev[1], 0) != cudaSuccess)
    return TILER_CUDA_DEVICE_ERROR;
  return last_error_status();
}

int32_t tiler_cuda_rms_norm_bf16(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* st, const uint16_t* x,
                                 const uint16_t* w, int64_t w_row_stride, uint64_t rows, uint64_t extent,
                                 uint32_t eps_bits, uint16_t* y) {
  return rms(1, ctx, stream, st, x, w, w_row_stride, rows, extent, eps_bits, y);
}

int32_t tiler_cuda_softmax_f32(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* st, const float* x,
                               uint64_t rows, uint64_t extent, uint64_t causal_period, uint64_t row_offset,
                               float* y) {
  CHECK_CTX(ctx);
  if (rows == 0 || extent == 0) return TILER_CUDA_OK;
  if (!x || !y) return TILER_CUDA_INVALID_APPLICATION;
  launch_softmax(x, rows, extent, causal_period, row_offset, y, st, ctx->facts.sm_count, S(stream));
  return last_error_status();
}

int32_t tiler_cuda_bounded_wait_selftest(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* st,
                                         uint64_t limit_ns) {
  CHECK_CTX(ctx);
  if (!st || limit_ns == 0 || limit_ns > kWaitLimitNs) return TILER_CUDA_INVALID_APPLICATION;
  launch_bounded_wait_selftest(st, limit_ns, S(stream));
  return last_error_status();
}

int32_t tiler_cuda_softmax_masked_f32(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* st, const float* x,
                                      uint64_t rows, uint64_t extent, const float* mask, uint64_t mask_rows,
                                      uint64_t row_offset, float* y) {
  CHECK_CTX(ctx);
  if (rows == 0 || extent == 0) return TILER_CUDA_OK;
  if (!x || !y || !mask || mask_rows == 0) return TILER_CUDA_INVALID_APPLICATION;
  const int r = launch_softmax(x, rows, extent, 0, row_offset, y, st, ctx->facts.sm_count, S(stream), mask, mask_rows);
  if (r != 0) return r;
  return last_error_status();
}

int32_t tiler_cuda_quantize_i8_rows(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* st, const float* x,
                                    uint64_t rows, uint64_t extent, int8_t* codes, float* scales) {
  CHECK_CTX(ctx);
  if (extent == 0) return TILER_CUDA_INVALID_APPLICATION;
  if (rows == 0) return TILER_CUDA_OK;
  if (!x || !codes || !scales || rows > 0x7fffffffull) return TILER_CUDA_INVALID_APPLICATION;
  launch_quantize_i8_rows(x, rows, extent, codes, scales, st, ctx->facts.sm_count, S(stream));
  return last_error_status();
}

int32_t tiler_cuda_rms_norm_quantize_i8(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* st, const float* x,
                                        const float* w, int64_t w_row_stride, uint64_t rows, uint64_t extent,
                                        uint32_t eps_bits, int8_t* codes, float* scales) {
  CHECK_CTX(ctx);
  if (!eps_admitted(eps_bits) || w_row_stride < 0) return TILER_CUDA_INVALID_APPLICATION;
  if (extent > (1ull << 24)) return TILER_CUDA_SHAPE_TOO_LARGE;
  if (extent == 0) return TILER_CUDA_INVALID_APPLICATION;  // quantize has no empty row
  if (rows == 0) return TILER_CUDA_OK;
  if (!x || !w || !codes || !scales || rows > 0x7fffffffull) return TILER_CUDA_INVALID_APPLICATION;
  if (w_row_stride != 0 && (uint64_t)w_row_stride != extent) return TILER_CUDA_UNSUPPORTED;
  float eps;
  memcpy(&eps, &eps_bits, 4);
  const int r = launch_rms_norm_quantize_i8(x, w, w_row_stride, rows, extent, eps, codes, scales, st,
                                            ctx->facts.sm_count, S(stream));
  if (r != 0) return r;
  return last_error_status();
}

int32_t tiler_cuda_dequantize_i8_rows(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* status,
                                      const int8_t* codes, const float* scales, uint64_t rows,
                                      uint64_t extent, float* y) {
  CHECK_CTX(ctx);
  if (rows == 0 || extent == 0) return TILER_CUDA_OK;
  if (!codes || !scales || !y || rows > 0x7fffffffull) return TILER_CUDA_INVALID_APPLICATION;
  launch_dequantize_i8_rows(codes, scales, rows, extent, y, ctx->facts.sm_count, S(stream), status);
  return last_error_status();
}

static bool scale_admitted(uint32_t bits, float* out) {
  float s;
  memcpy(&s, &bits, 4);
  *out = s;
  return s >= 1.17549435e-38f && s <= 3.40282347e38f;  // positive normal (quantization.rs:377-379)
}

int32_t tiler_cuda_quantize_affine_u8(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* st, const float* x,
                                      uint64_t n, uint32_t scale_bits, uint32_t zp, uint32_t maximum,
                                      uint8_t* codes) {
  CHECK_CTX(ctx);
  float scale;
  if (!scale_admitted(scale_bits, &scale) || (maximum != 15 && maximum != 255) || zp > maximum)
    return TILER_CUDA_INVALID_APPLICATION;
  if (n == 0) return TILER_CUDA_OK;
  if (!x || !codes) return TILER_CUDA_INVALID_APPLICATION;
  launch_quantize_affine_u8(x, n, scale, zp, maximum, codes, st, ctx->facts.sm_count, S(stream));
  return last_error_status();
}

int32_t tiler_cuda_dequantize_affine_u8(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* st,
                                        const uint8_t* codes, uint64_t n, uint32_t scale_bits, uint32_t zp,
                                        uint32_t maximum, float* y) {
  CHECK_CTX(ctx);
  float scale;
  if (!scale_admitted(scale_bits, &scale) || (maximum != 15 && maximum != 255) || zp > maximum)
    return TILER_CUDA_INVALID_APPLICATION;
  if (n == 0) return TILER_CUDA_OK;
  if (!codes || !y) return TILER_CUDA_INVALID_APPLICATION;
  launch_dequantize_affine_u8(codes, n, scale, zp, maximum, y, st, ctx->facts.sm_count, S(stream));
  return last_error_status();
}

// ---- maps ------------------------------------------------------------------------

int32_t tiler_cuda_silu_f32(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* st, const float* x,
                            uint64_t n, float* y) {
  CHECK_CTX(ctx);
  if (n == 0) return TILER_CUDA_OK;
  if (!x || !y) return TILER_CUDA_INVALID_APPLICATION;
  launch_silu(x, n, y, st, ctx->facts.sm_count, S(stream));
  return last_error_status();
}

int32_t tiler_cuda_scale_bias_f32(tiler_cuda_context* ctx, void* stream, const float* x, uint64_t n, const float* a,
                                  int32_t a_scalar, const float* b, int32_t b_scalar, float* y) {
  CHECK_CTX(ctx);
  if (n == 0) return TILER_CUDA_OK;
  if (!x || !a || !b || !y) return TILER_CUDA_INVALID_APPLICATION;
  launch_scale_bias(x, n, a, a_scalar, b, b_scalar, y, ctx->facts.sm_count, S(stream));
  return last_error_status();
}

int32_t tiler_cuda_gather_rows(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* st, const void* table,
                               uint64_t table_rows, uint64_t row_bytes, const void* ids, int32_t ids_unsigned,
                               uint64_t n_ids, void* out) {
  CHECK_CTX(ctx);
  if (n_ids == 0 || row_bytes == 0) return TILER_CUDA_OK;
  if (!ids || !out || (!table && table_rows)) return TILER_CUDA_INVALID_APPLICATION;
  if (n_ids > 0xffffffffull) return TILER_CUDA_SHAPE_TOO_LARGE;
  launch_gather_rows(table, table_rows, row_bytes, ids, ids_unsigned, n_ids, out, st, ctx->facts.sm_count,
                     S(stream));
  return last_error_status();
}

// ---- contraction ---------------------------------------------------------------

int32_t tiler_cuda_contract_f32(tiler_cuda_context* ctx, void* stream, const float* a, const float* b, uint64_t m,
                                uint64_t n, uint64_t k, float* c) {
  CHECK_CTX(ctx);
  if (k == 0) return TILER_CUDA_INVALID_APPLICATION;  // a first-product seed needs a product
  if (m == 0 || n == 0) return TILER_CUDA_OK;
  if (!a || !b || !c || m > 65535ull * 16 || n > 0x7fffffffull) return TILER_CUDA_INVALID_APPLICATION;
  launch_contract_f32(a, b, m, n, k, c, S(stream));
  return last_error_status();
}

int32_t tiler_cuda_gemm_bf16(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* st, const uint16_t* a,
                             const uint16_t* b, uint64_t m, uint64_t n, uint64_t k, int32_t epilogue, uint16_t* c,
                             uint64_t ldc) {
  CHECK_CTX(ctx);
  if (epilogue != 0 && epilogue != 1) return TILER_CUDA_INVALID_APPLICATION;
  if (k == 0) return TILER_CUDA_INVALID_APPLICATION;
  if (m == 0 || n == 0) return TILER_CUDA_OK;
  if (!a || !b || !c) return TILER_CUDA_INVALID_APPLICATION;
  if (m / 128 * (n / 256) > 0xffffffffull || k > (1ull << 31)) return TILER_CUDA_SHAPE_TOO_LARGE;
  int32_t r = launch_gemm_bf16(a, b, m, n, k, epilogue, c, ldc, st, ctx->facts.sm_count, S(stream));
  if (r != TILER_CUDA_OK) return r;
  return last_error_status();
}

// ---- device buffers shared between the processes of a node -------------------

typedef CUresult (*AddressRangeFn)(CUdeviceptr*, size_t*, CUdeviceptr);

int32_t tiler_cuda_ipc_export(tiler_cuda_context* ctx, const void* ptr, uint8_t* handle, uint64_t* offset) {
  CHECK_CTX(ctx);
  if (!ptr || !handle || !offset) return TILER_CUDA_INVALID_APPLICATION;
  static AddressRangeFn range = nullptr;
  if (!range) {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return TILER_CUDA_DEVICE_ERROR;
    range = (AddressRangeFn)p;
  }
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range(&base, &size, (CUdeviceptr)(uintptr_t)ptr) != CUDA_SUCCESS) return TILER_CUDA_INVALID_APPLICATION;
  cudaIpcMemHandle_t h;
  if (cudaIpcGetMemHandle(&h, (void*)(uintptr_t)base) != cudaSuccess) return TILER_CUDA_DEVICE_ERROR;
  memcpy(handle, &h, sizeof(h));
  *offset = (uint64_t)((uintptr_t)ptr - (uintptr_t)base);
  return TILER_CUDA_OK;
}

int32_t tiler_cuda_ipc_open(tiler_cuda_context* ctx, const uint8_t* handle, uint64_t offset, void** out) {
  CHECK_CTX(ctx);
  if (!handle || !out) return TILER_CUDA_INVALID_APPLICATION;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) return TILER_CUDA_DEVICE_ERROR;
  *out = (uint8_t*)base + offset;
  return TILER_CUDA_OK;
}

int32_t tiler_cuda_ipc_close(tiler_cuda_context* ctx, void* ptr, uint64_t offset) {
  CHECK_CTX(ctx);
  if (!ptr) return TILER_CUDA_INVALID_APPLICATION;
  return cudaIpcCloseMemHandle((uint8_t*)ptr - offset) == cudaSuccess ? TILER_CUDA_OK : TILER_CUDA_DEVICE_ERROR;
}

int32_t tiler_cuda_gemm_bf16_allgather(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* st,
                                       const uint16_t* a, const uint16_t* b_shard, uint64_t m, uint64_t n_shard,
                                       uint64_t k, int32_t epilogue, uint32_t rank, uint32_t world,
                                       void* const* blocks) {
  CHECK_CTX(ctx);
  if (epilogue != 0 && epilogue != 1) return TILER_CUDA_INVALID_APPLICATION;
  if (k == 0 || world == 0 || rank >= world || !blocks) return TILER_CUDA_INVALID_APPLICATION;
  if (world > 8) return TILER_CUDA_UNSUPPORTED;
  if (m == 0 || n_shard == 0) return TILER_CUDA_OK;
  if (!a || !b_shard) return TILER_CUDA_INVALID_APPLICATION;
  for (uint32_t q = 0; q < world; ++q)
    if (!blocks[q]) return TILER_CUDA_INVALID_APPLICATION;
  if (m / 128 * (n_shard / 256) > 0xffffffffull || k > (1ull << 31)) return TILER_CUDA_SHAPE_TOO_LARGE;
  // block r of every buffer holds rank r's [m, n_shard] columns
  const uint64_t block_elems = m * n_shard;
  uint16_t* local = (uint16_t*)blocks[rank] + (uint64_t)rank * block_elems;
  uint16_t* peer[8] = {};
  uint32_t np = 0;
  for (uint32_t q = 0; q < world; ++q)
    if (q != rank) peer[np++] = (uint16_t*)blocks[q] + (uint64_t)rank * block_elems;
  int32_t r = launch_gemm_bf16(a, b_shard, m, n_shard, k, epilogue, local, n_shard, st, ctx->facts.sm_count,
                               S(stream), peer, np);
  if (r != TILER_CUDA_OK) return r;
  return last_error_status();
}

int32_t tiler_cuda_gemm_bf16_allgather_multicast(tiler_cuda_context* ctx, void* stream, tiler_cuda_status* st,
                                                 const uint16_t* a, const uint16_t* b_shard, uint64_t m,
                                                 uint64_t n_shard, uint64_t k, int32_t epilogue, uint32_t rank,
                                                 uint32_t world, void* local_buffer, void* multicast_buffer) {
  CHECK_CTX(ctx);
  if (epilogue != 0 && epilogue != 1) return TILER_CUDA_INVALID_APPLICATION;
  if (k == 0 || world == 0 || rank >= world || !local_buffer || !multicast_buffer)
    return TILER_CUDA_INVALID_APPLICATION;
  if (m == 0 || n_shard == 0) return TILER_CUDA_OK;
  if (!a || !b_shard) return TILER_CUDA_INVALID_APPLICATION;
  if (m / 128 * (n_shard / 256) > 0xffffffffull || k > (1ull << 31)) return TILER_CUDA_SHAPE_TOO_LARGE;
  const uint64_t block_elems = m * n_shard;
  uint16_t* local = (uint16_t*)local_buffer + (uint64_t)rank * block_elems;
  uint16_t* mc = (uint16_t*)multicast_buffer + (uint64_t)rank * block_elems;
  int32_t r = launch_gemm_bf16(a, b_shard, m, n_shard, k, epilogue, local, n_shard, st, ctx->facts.sm_count,
                               S(stream), nullptr, 0, mc);
  if (r != TILER_CUDA_OK) return r;
  return last_error_status();
}

}  // extern "C"
