// Kernel launches that can run from a loaded payload module.
//
// A Tiler plan artifact carries its backend code as bytes (PayloadContent.code,
// crates/tiler-artifact/src/program/codec/payload.rs:228-424); the runtime
// validates and prepares it before any dispatch (validate_payload /
// prepare_entries, crates/tiler-runtime/src/adapter.rs:639-655).  Here that
// code is an sm_100a cubin built from this library's own kernel sources
// (tiler_kernels.cubin).  Once tiler_cuda_module_load has loaded it and
// tiler_cuda_context_bind_module has bound it to a context, every family
// launch on that context whose kernel the module carries launches the
// module's function (cuLaunchKernel) instead of the library's built-in copy.
//
// The module-launchable kernels have C names (extern "C" __global__), so the
// same name finds them in the library and in the cubin.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#include <atomic>
#include <mutex>

#include "drv.cuh"

// Kernels a payload module may carry, by C name.
constexpr int kModuleKernelCount = 15;
inline const char* const kModuleKernels[kModuleKernelCount] = {
    "tiler_rms_norm_wave_f32", "tiler_rms_norm_wave_bf16", "tiler_rms_norm_wave_quantize_i8",
    "tiler_rms_norm_stream_f32", "tiler_rms_norm_stream_bf16", "tiler_rms_norm_stream_quantize_i8",
    "tiler_rms_norm_f32",   "tiler_rms_norm_bf16",  "tiler_rms_norm_quantize_i8",
    "tiler_grouped_sum_k1", "tiler_grouped_sum_k2", "tiler_grouped_sum_k4",
    "tiler_grouped_max_k1", "tiler_grouped_max_k2", "tiler_grouped_max_k4",
};

struct tiler_cuda_module {
  int device;
  CUcontext cu_ctx;  // the context the module was loaded into
  CUmodule mod;
  CUfunction fn[kModuleKernelCount];        // null where the module lacks the kernel
  size_t smem_allowed[kModuleKernelCount];  // dynamic shared memory opted in so far
  std::mutex mutex;
  std::atomic<uint64_t> launches{0};
};

namespace tc {

struct ModuleDriver {
  CUresult (*load)(CUmodule*, const void*) = nullptr;
  CUresult (*unload)(CUmodule) = nullptr;
  CUresult (*get_function)(CUfunction*, CUmodule, const char*) = nullptr;
  CUresult (*get_global)(CUdeviceptr*, size_t*, CUmodule, const char*) = nullptr;
  CUresult (*func_get_attribute)(int*, CUfunction_attribute, CUfunction) = nullptr;
  CUresult (*func_set_attribute)(CUfunction, CUfunction_attribute, int) = nullptr;
  CUresult (*launch)(CUfunction, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, unsigned, CUstream,
                     void**, void**) = nullptr;
  CUresult (*memcpy_htod)(CUdeviceptr, const void*, size_t) = nullptr;
  CUresult (*memcpy_dtoh)(void*, CUdeviceptr, size_t) = nullptr;
  CUresult (*ctx_current)(CUcontext*) = nullptr;
  bool ok = false;
};

inline const ModuleDriver& module_driver() {
  static ModuleDriver d = [] {
    ModuleDriver m;
    m.load = driver_fn<decltype(m.load)>("cuModuleLoadData");
    m.unload = driver_fn<decltype(m.unload)>("cuModuleUnload");
    m.get_function = driver_fn<decltype(m.get_function)>("cuModuleGetFunction");
    m.get_global = driver_fn<decltype(m.get_global)>("cuModuleGetGlobal");
    m.func_get_attribute = driver_fn<decltype(m.func_get_attribute)>("cuFuncGetAttribute");
    m.func_set_attribute = driver_fn<decltype(m.func_set_attribute)>("cuFuncSetAttribute");
    m.launch = driver_fn<decltype(m.launch)>("cuLaunchKernel");
    m.memcpy_htod = driver_fn<decltype(m.memcpy_htod)>("cuMemcpyHtoD");
    m.memcpy_dtoh = driver_fn<decltype(m.memcpy_dtoh)>("cuMemcpyDtoH");
    m.ctx_current = driver_fn<decltype(m.ctx_current)>("cuCtxGetCurrent");
    m.ok = m.load && m.unload && m.get_function && m.get_global && m.func_get_attribute && m.func_set_attribute &&
           m.launch && m.memcpy_htod && m.memcpy_dtoh && m.ctx_current;
    return m;
  }();
  return d;
}

// The module bound to the context of the calling thread's current C-ABI call
// (set by every entry point that binds a context), or null.
inline thread_local tiler_cuda_module* tl_module = nullptr;

// A module launch that failed (reported by the C-ABI call, as a failed
// runtime launch is through cudaGetLastError).
inline thread_local bool tl_module_launch_failed = false;

inline int module_kernel_index(const char* name) {
  for (int i = 0; i < kModuleKernelCount; ++i)
    if (strcmp(kModuleKernels[i], name) == 0) return i;
  return -1;
}

// Launches kernel `name` (the library's function `fn`) with `args`, whose
// types must be exactly the kernel's parameter types: from the bound
// module when it carries the kernel, else the library's own copy.
template <class... A>
inline cudaError_t launch_kernel(const void* fn, const char* name, dim3 grid, dim3 block, size_t smem,
                                 cudaStream_t stream, A... args) {
  void* params[] = {(void*)&args...};
  if (tiler_cuda_module* m = tl_module) {
    const int i = module_kernel_index(name);
    if (i >= 0 && m->fn[i]) {
      const ModuleDriver& d = module_driver();
      if (smem > m->smem_allowed[i]) {
        std::lock_guard<std::mutex> lock(m->mutex);
        if (d.func_set_attribute(m->fn[i], CU_FUNC_ATTRIBUTE_MAX_DYNAMIC_SHARED_SIZE_BYTES, (int)smem) !=
            CUDA_SUCCESS) {
          tl_module_launch_failed = true;
          return cudaErrorInvalidValue;
        }
        m->smem_allowed[i] = smem;
      }
      if (d.launch(m->fn[i], grid.x, grid.y, grid.z, block.x, block.y, block.z, (unsigned)smem, (CUstream)stream,
                   params, nullptr) != CUDA_SUCCESS) {
        tl_module_launch_failed = true;
        return cudaErrorLaunchFailure;
      }
      m->launches.fetch_add(1, std::memory_order_relaxed);
      return cudaSuccess;
    }
  }
  // programmatic dependent launch: the kernel may begin while the previous
  // kernel on the stream drains (every kernel launched here waits for it in
  // grid_dependency_wait before touching global memory); TILER_PDL=0 in the
  // environment (read once per process) launches plainly
  static const bool pdl = [] {
    const char* v = getenv("TILER_PDL");
    return !(v && strcmp(v, "0") == 0);
  }();
  if (!pdl) return cudaLaunchKernel(fn, grid, block, params, smem, stream);
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, fn, params);
}

}  // namespace tc
