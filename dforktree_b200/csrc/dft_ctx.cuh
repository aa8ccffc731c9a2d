// The driver context current on this thread, through the runtime's driver
// entry point (no -lcuda at link time).  Per-device state that the library
// keeps across calls (a device symbol's address, a side stream and its
// events) belongs to one context; comparing the context recorded with that
// state against this one tells whether a device reset has invalidated it.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>

namespace dft {

typedef CUresult (*CtxGetCurrentFn)(CUcontext*);

inline CtxGetCurrentFn ctx_get_current_fn() {
  static CtxGetCurrentFn fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      return reinterpret_cast<CtxGetCurrentFn>(p);
    return static_cast<CtxGetCurrentFn>(nullptr);
  }();
  return fn;
}

// Current device and its runtime context (made current on this thread first);
// false when either is unavailable.
inline bool current_device_context(int* dev, CUcontext* ctx) {
  *dev = -1;
  *ctx = nullptr;
  if (cudaGetDevice(dev) != cudaSuccess || *dev < 0) return false;
  if (cudaSetDevice(*dev) != cudaSuccess) return false;
  CtxGetCurrentFn get = ctx_get_current_fn();
  return get && get(ctx) == CUDA_SUCCESS && *ctx;
}

}  // namespace dft
