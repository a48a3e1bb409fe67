// Allocation-free variant of the grouped sum (tiler_cuda_sum_f32_no_alloc).
//
// Some callers cannot allocate device memory at the point where they need a
// reduction: code running under an allocator that is frozen or owned by
// someone else (a host framework that pre-plans every buffer, a real-time
// loop that must not call cudaMalloc, a plugin handed only its inputs and
// outputs).  tiler_cuda_sum_f32 needs a caller-provided workspace for its
// per-partition partials and per-row completion tickets; this entry point
// keeps that workspace in a fixed array compiled into the library instead.
//
// The array lives in every GPU that loads the library, for as long as the
// process runs (kNoAllocScratchBytes, about 260 KB).  Its name is only a
// host-side stand-in: the device address comes from cudaGetSymbolAddress,
// taken once per device (with that device current) the first time the entry
// point runs there.  Make that first call before capturing a stream.
// All calls share the array; calls that overlap on the GPU race with each
// other.  The tickets are cleared on every call; the partials are always
// written before they are read.
#include "common.cuh"
#include "drv.cuh"
#include "kernels.h"

namespace tc {

constexpr uint64_t kNoAllocMaxPartials = 65536;  // rows * partitions
constexpr uint64_t kNoAllocMaxRows = 1024;
constexpr size_t kNoAllocScratchBytes = kNoAllocMaxPartials * 4 + kNoAllocMaxRows * 4;

static __device__ __align__(256) uint8_t g_no_alloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_no_alloc_mutex;
struct NoAllocSlot {
  CUcontext owner = nullptr;  // the context the address was taken in
  void* ptr = nullptr;
};
NoAllocSlot g_no_alloc_slot[64];

// Device address of g_no_alloc_scratch on the current device.  It is taken
// once per device and taken again if the device's context was replaced (after
// cudaDeviceReset the module, and with it the array, is loaded anew).
int32_t no_alloc_scratch(void** out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return TILER_CUDA_DEVICE_ERROR;
  typedef CUresult (*CtxGetCurrentFn)(CUcontext*);
  static CtxGetCurrentFn ctx_current = driver_fn<CtxGetCurrentFn>("cuCtxGetCurrent");
  if (!ctx_current) return TILER_CUDA_DEVICE_ERROR;
  CUcontext cur = nullptr;
  if (ctx_current(&cur) != CUDA_SUCCESS) return TILER_CUDA_DEVICE_ERROR;
  std::lock_guard<std::mutex> lock(g_no_alloc_mutex);
  NoAllocSlot& slot = g_no_alloc_slot[dev];
  if (!slot.ptr || slot.owner != cur) {
    void* p = nullptr;
    if (cudaGetSymbolAddress(&p, g_no_alloc_scratch) != cudaSuccess || !p) return TILER_CUDA_DEVICE_ERROR;
    if (ctx_current(&cur) != CUDA_SUCCESS) return TILER_CUDA_DEVICE_ERROR;  // the runtime may have made it
    slot.ptr = p;
    slot.owner = cur;
  }
  *out = slot.ptr;
  return TILER_CUDA_OK;
}
}  // namespace

}  // namespace tc

extern "C" int32_t tiler_cuda_sum_f32_no_alloc(tiler_cuda_context* ctx, void* stream, const float* x, uint64_t rows,
                                               uint64_t count, const tiler_cuda_grouping* g, float* out) {
  using namespace tc;
  if (!ctx || !g) return TILER_CUDA_INVALID_APPLICATION;
  if (rows > kNoAllocMaxRows || (rows && g->partitions > kNoAllocMaxPartials / rows)) return TILER_CUDA_SHAPE_TOO_LARGE;
  if (rows == 0 || count == 0 || g->partitions <= 1)
    return tiler_cuda_sum_f32(ctx, stream, x, rows, count, g, nullptr, 0, out);
  if (!x || !out) return TILER_CUDA_INVALID_APPLICATION;
  if (!bind(ctx)) return TILER_CUDA_DEVICE_ERROR;
  void* scratch = nullptr;
  int32_t r = no_alloc_scratch(&scratch);
  if (r != TILER_CUDA_OK) return r;
  // every refusal happens before the shared array is touched
  r = validate_grouping(rows, count, g, kNoAllocScratchBytes, scratch);
  if (r != TILER_CUDA_OK) return r;
  const uint64_t partial_bytes = (rows * g->partitions * 4 + 255) / 256 * 256;
  // The tickets must start at zero; a memset allocates nothing.
  if (cudaMemsetAsync((uint8_t*)scratch + partial_bytes, 0, rows * 4, S(stream)) != cudaSuccess)
    return TILER_CUDA_DEVICE_ERROR;
  return tiler_cuda_sum_f32(ctx, stream, x, rows, count, g, scratch, kNoAllocScratchBytes, out);
}
