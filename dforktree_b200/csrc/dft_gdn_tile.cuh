// Helpers shared by the tensor-core GDN verifiers (dft_gdn_tc.cu for trees of
// up to 32 nodes, dft_gdn_tc64.cu for 33-64 nodes): tf32 rounding, raw
// element loads, loads issued a unit ahead, the kernel argument block and the
// host-side tensor-map encoder / SM count.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <mutex>

#include "dforktree_b200.h"

namespace dft {
namespace gtile {

__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}

// raw element bits (fp32, or bf16 / f16 in the low half) and their value
__device__ __forceinline__ uint32_t ld_bits(const void* p, int dtype, int64_t i) {
  if (dtype == DFT_F32) return __ldg(reinterpret_cast<const uint32_t*>(p) + i);
  return (uint32_t)__ldg(reinterpret_cast<const unsigned short*>(p) + i);
}
__device__ __forceinline__ float bits_f32(uint32_t v, int dtype) {
  if (dtype == DFT_F32) return __uint_as_float(v);
  if (dtype == DFT_BF16) return __uint_as_float(v << 16);
  return __half2float(__ushort_as_half((unsigned short)v));
}

// global loads the compiler keeps where they are written (prefetch one unit ahead)
__device__ __forceinline__ uint4 ldg_keep_v4(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t ldg_keep_u32(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
}
__device__ __forceinline__ unsigned short ldg_keep_u16(const void* p) {
  unsigned short r;
  asm volatile("ld.global.nc.u16 %0, [%1];" : "=h"(r) : "l"(p));
  return r;
}
__device__ __forceinline__ uint32_t ld_s32(const unsigned char* p) { return *reinterpret_cast<const uint32_t*>(p); }
__device__ __forceinline__ void st_s32(unsigned char* p, uint32_t v) { *reinterpret_cast<uint32_t*>(p) = v; }

// the verifiers' kernel argument block (by value, __grid_constant__)
struct TcArgs {
  dft_gdn_args g;
  dft_gdn_conv_args cv;
};

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda at link time)
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

inline int sm_count() {
  static int n = 0;
  if (!n) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    if (n <= 0) n = 148;
  }
  return n;
}

inline bool al16(const void* p) { return ((uintptr_t)p & 15) == 0; }

}  // namespace gtile
}  // namespace dft
