// Driver-API entry points reached through cudaGetDriverEntryPoint, so the
// library does not link libcuda directly.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

namespace tc {

// The driver function `name`, or nullptr when the driver does not export it.
template <class Fn>
inline Fn driver_fn(const char* name) {
  void* p = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint(name, &p, cudaEnableDefault, &q) != cudaSuccess || q != cudaDriverEntryPointSuccess)
    return nullptr;
  return reinterpret_cast<Fn>(p);
}

}  // namespace tc
