// Shared device helpers for the dforktree_b200 kernels (sm_100a).
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "../../include/dforktree_b200.h"

#define DFT_CUDA_CHECK(expr)                                   \
  do {                                                         \
    cudaError_t _e = (expr);                                   \
    if (_e != cudaSuccess) return DFT_ERR_CUDA;                \
  } while (0)

#define DFT_LAUNCH_CHECK() DFT_CUDA_CHECK(cudaGetLastError())

namespace dft {

constexpr unsigned long long kEmptyKey = 0xFFFFFFFFFFFFFFFFull;
constexpr int kMaxNodes = 64;

// ---------------------------------------------------------------- dtypes --
__device__ __forceinline__ float to_f32(float x) { return x; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 x) { return __bfloat162float(x); }
__device__ __forceinline__ float to_f32(__half x) { return __half2float(x); }

template <typename T> __device__ __forceinline__ T from_f32(float x);
template <> __device__ __forceinline__ float from_f32<float>(float x) { return x; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float x) { return __float2bfloat16_rn(x); }
template <> __device__ __forceinline__ __half from_f32<__half>(float x) { return __float2half_rn(x); }

__device__ __forceinline__ float load_any(const void* p, int dtype, int64_t i) {
  switch (dtype) {
    case DFT_BF16: return __bfloat162float(reinterpret_cast<const __nv_bfloat16*>(p)[i]);
    case DFT_F16: return __half2float(reinterpret_cast<const __half*>(p)[i]);
    default: return reinterpret_cast<const float*>(p)[i];
  }
}
__device__ __forceinline__ void store_any(void* p, int dtype, int64_t i, float v) {
  switch (dtype) {
    case DFT_BF16: reinterpret_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v); break;
    case DFT_F16: reinterpret_cast<__half*>(p)[i] = __float2half_rn(v); break;
    default: reinterpret_cast<float*>(p)[i] = v;
  }
}

inline bool valid_dtype(int d) { return d == DFT_F32 || d == DFT_BF16 || d == DFT_F16; }

// Score + build scratch layout (drafter lp / ids / rest rows, then the dense
// PMI tensor T of the closure's order), shared by dft_score_build's caller workspace and
// dft_score_build_static's fixed array, so both use the same offsets.
struct BuildScratch {
  int64_t lp, ids, rest, T, total;
};

inline int64_t up256(int64_t x) { return (x + 255) & ~(int64_t)255; }

// n-gram order of the PMI closure (0 selects the Builder's order 3) and the
// floats of T per (request, step): M^order.
inline int pmi_order_of(const dft_build_params* p) { return p->pmi_order == 0 ? 3 : p->pmi_order; }
inline int64_t pmi_step_floats(const dft_build_params* p) {
  int64_t n = 1;
  for (int k = 0; k < pmi_order_of(p); ++k) n *= p->M;
  return n;
}

inline BuildScratch build_scratch_layout(const dft_build_params* p) {
  BuildScratch w;
  const int64_t rows = (int64_t)p->B * p->S;
  int64_t o = 0;
  w.lp = o; o = up256(o + rows * p->M * 4);
  w.ids = o; o = up256(o + rows * p->M * 4);
  w.rest = o; o = up256(o + rows * 4);
  w.T = o; o = up256(o + (p->use_ngram ? (int64_t)p->B * (p->S - 1) * pmi_step_floats(p) * 4 : 0));
  w.total = o;
  return w;
}

// ---------------------------------------------------------------- SiLU --
// silu(x) = x / (1 + e^-x) with e^-x = 2^(-x log2 e) from the hardware
// base-2 exponential and 1 / d from the hardware reciprocal (both the
// documented .approx PTX forms).  The standalone tree conv and the conv fused
// into the tensor-core verifier share this exact sequence (the packed form
// below rounds each lane identically), so both give bit-identical y.
constexpr float kNegLog2e = -1.4426950408889634f;
__device__ __forceinline__ float ex2_approx(float x) {
  float r;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float rcp_approx(float x) {
  float r;
  asm("rcp.approx.ftz.f32 %0, %1;" : "=f"(r) : "f"(x));
  return r;
}
__device__ __forceinline__ float silu_hw(float x) {
  const float e = ex2_approx(__fmul_rn(x, kNegLog2e));
  return __fmul_rn(x, rcp_approx(__fadd_rn(1.f, e)));
}

// ------------------------------------------ packed fp32 pairs (sm_100a) --
// add / mul .rn.f32x2 round each lane exactly like the scalar .rn forms.
typedef unsigned long long f32x2;
__device__ __forceinline__ f32x2 pk2(float lo, float hi) {
  f32x2 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void upk2(f32x2 v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ f32x2 add2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f32x2 sub2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ f32x2 fma2(f32x2 a, f32x2 b, f32x2 c) {
  f32x2 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ f32x2 mul2(f32x2 a, f32x2 b) {
  f32x2 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
// two bf16 (low half = first element) <-> fp32 pair
__device__ __forceinline__ f32x2 bf16x2_to_f32x2(uint32_t v) {
  return pk2(__uint_as_float(v << 16), __uint_as_float(v & 0xFFFF0000u));
}
__device__ __forceinline__ uint32_t f32x2_to_bf16x2(f32x2 v) {
  float lo, hi;
  upk2(v, lo, hi);
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ f32x2 silu_hw2(f32x2 x) {
  const f32x2 t = mul2(x, pk2(kNegLog2e, kNegLog2e));
  float t0, t1;
  upk2(t, t0, t1);
  const f32x2 d = add2(pk2(1.f, 1.f), pk2(ex2_approx(t0), ex2_approx(t1)));
  float d0, d1;
  upk2(d, d0, d1);
  return mul2(x, pk2(rcp_approx(d0), rcp_approx(d1)));
}

// bytes at p (16-byte aligned, a multiple of 16) into L2; nothing waits for it
__device__ __forceinline__ void prefetch_l2(const void* p, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(p), "r"(bytes) : "memory");
}

// ------------------------------------------- programmatic dependent launch --
// pdl_wait: the preceding kernel in the stream has completed and its writes
// are visible (returns at once for a kernel launched without the programmatic
// attribute).  The score / PMI kernels trigger nothing early: an explicit
// launch_dependents at their start made score + build slower (0.503 against
// 0.449 ms at batch 64); without it the next launch still overlaps the
// previous grid's drain (0.448 against 0.451 ms).
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// launch k<<<grid, block, smem, st>>>(args...) with programmatic stream
// serialisation: its CTAs may be scheduled as the previous kernel drains, so
// every read of that kernel's outputs must come after pdl_wait()
template <typename... KArgs, typename... Args>
inline int launch_pdl(void (*k)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, k, static_cast<KArgs>(args)...) == cudaSuccess ? DFT_OK : DFT_ERR_CUDA;
}

// ------------------------------------------------------------ status word --
__device__ __forceinline__ void raise_status(int32_t* st, int bits) {
  if (st) atomicOr(st, bits);
}

// ------------------------------------------------------------------ hash --
// 64-bit finaliser (xor-shift-multiply), well mixed in the low bits.
__host__ __device__ __forceinline__ unsigned long long mix64(unsigned long long x) {
  x ^= x >> 33;
  x *= 0xff51afd7ed558ccdull;
  x ^= x >> 33;
  x *= 0xc4ceb9fe1a85ec53ull;
  x ^= x >> 33;
  return x;
}

// One 16-byte hash slot: 64-bit key + two 32-bit payload words.
struct __align__(16) Slot {
  unsigned long long key;
  float f0;      // pair: bigram count   | triple: c3     | quad: c4
  uint32_t u1;   // pair: n3c (as float) | triple: rank3  | quad: unused
};

__device__ __forceinline__ uint4 ldg_slot(const Slot* s) {
  return __ldg(reinterpret_cast<const uint4*>(s));
}
__device__ __forceinline__ unsigned long long slot_key(uint4 v) {
  return (static_cast<unsigned long long>(v.y) << 32) | v.x;
}
// What a probe that misses returns: the empty key (so `slot_key(s) == q` is
// an exact hit test, also for key 0) with zero counts and rank.
__device__ __forceinline__ uint4 miss_slot() { return make_uint4(0xFFFFFFFFu, 0xFFFFFFFFu, 0u, 0u); }

// Device view of the n-gram tables (POD, passed by value).  Each slot array
// has a fingerprint array beside it, one byte per slot: 0 for an empty slot,
// else fp_of(mix64(key)) (never 0).  The fingerprints are small enough to stay
// in L2 (1/16 of the slots' bytes), so a probe that misses -- the common case
// for drafted candidates -- resolves there without reading the slot in HBM.
struct TableView {
  int64_t V;
  const Slot* pair; unsigned long long pair_mask;
  const Slot* trip; unsigned long long trip_mask;
  const Slot* quad; unsigned long long quad_mask;
  const uint8_t* pair_fp;
  const uint8_t* trip_fp;
  const uint8_t* quad_fp;
  const float* prev;
  const float* pn;
  const float* n4c;
  int has_pair, has_trip, has_quad, has_ctx;
  float beta2, beta3, beta4, clip;
};

// Fingerprint of a key from the high bits of its hash (the bucket index uses
// the low bits): 1..255, 0 marks an empty slot.
__host__ __device__ __forceinline__ uint32_t fp_of(unsigned long long h) { return 1u + (uint32_t)(h >> 56) % 255u; }

__device__ __forceinline__ uint64_t l2_evict_last_policy() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
// the aligned 8 fingerprints around a slot (kept in L2: evict-last)
__device__ __forceinline__ uint2 ld_fp8(const uint8_t* p, uint64_t pol) {
  uint2 r;
  asm volatile("ld.global.nc.L2::cache_hint.v2.u32 {%0, %1}, [%2], %3;" : "=r"(r.x), "=r"(r.y) : "l"(p), "l"(pol));
  return r;
}
__device__ __forceinline__ uint32_t fp_byte(uint2 w, int k) { return ((k < 4 ? w.x : w.y) >> (8 * (k & 3))) & 0xFFu; }

// Probe with fingerprints from bucket `idx` on (fingerprint f of key q):
// fingerprint bytes decide emptiness and candidates; only a candidate's slot
// is read.  Returns the matching slot or miss_slot().  Inlined: as a call
// (it is the rare continuation past a bucket group) it made the PMI kernels
// keep their eight in-flight probes in callee-saved registers (order 3: 72
// registers and three CTAs per SM; inlined 62 and four): 119 -> ~85 us.
__device__ __forceinline__ uint4 probe_fp_from(const Slot* tab, const uint8_t* fp, unsigned long long mask,
                                            unsigned long long uq, uint32_t f, unsigned long long idx,
                                            int32_t* status) {
  const uint64_t pol = l2_evict_last_policy();
  for (unsigned long long n = 0; n <= mask;) {
    const uint2 w = ld_fp8(fp + (idx & ~7ull), pol);
    for (int k = (int)(idx & 7); k < 8 && n <= mask; ++k, ++n) {
      const uint32_t b = fp_byte(w, k);
      const unsigned long long at = (idx & ~7ull) + k;
      if (b == 0) return miss_slot();
      if (b == f) {
        const uint4 s = __ldg(reinterpret_cast<const uint4*>(tab + at));
        if (((static_cast<unsigned long long>(s.y) << 32) | s.x) == uq) return s;
      }
    }
    idx = ((idx & ~7ull) + 8) & mask;
  }
  raise_status(status, DFT_DEV_PROBE_LIMIT);
  return miss_slot();
}

// Probe an open-addressed table; returns the matching slot (key == q) or
// miss_slot() on a miss.  Negative keys never match (table keys are >= 0).
// With fingerprints (fp != nullptr) the slots are read only on a fingerprint match.
__device__ __forceinline__ uint4 probe_fp(const Slot* tab, const uint8_t* fp, unsigned long long mask, long long q,
                                          int32_t* status) {
  if (q < 0 || tab == nullptr) return miss_slot();
  const unsigned long long uq = static_cast<unsigned long long>(q), h = mix64(uq);
  return probe_fp_from(tab, fp, mask, uq, fp_of(h), h & mask, status);
}

__device__ __forceinline__ uint4 probe(const Slot* tab, unsigned long long mask, long long q,
                                       int32_t* status) {
  const uint4 z = miss_slot();
  if (q < 0 || tab == nullptr) return z;
  unsigned long long uq = static_cast<unsigned long long>(q);
  unsigned long long h = mix64(uq) & mask;
  for (unsigned long long n = 0; n <= mask; ++n) {
    uint4 s = ldg_slot(tab + h);
    unsigned long long k = slot_key(s);
    if (k == uq) return s;
    if (k == kEmptyKey) return z;
    h = (h + 1) & mask;
  }
  raise_status(status, DFT_DEV_PROBE_LIMIT);
  return z;
}

// Continue probing after a first slot `s0` was loaded from bucket mix64(q)&mask.
__device__ __forceinline__ uint4 probe_from(const Slot* tab, unsigned long long mask, long long q, uint4 s0,
                                            int32_t* status) {
  const uint4 z = miss_slot();
  if (q < 0 || tab == nullptr) return z;
  unsigned long long uq = static_cast<unsigned long long>(q);
  unsigned long long k = slot_key(s0);
  if (k == uq) return s0;
  if (k == kEmptyKey) return z;
  unsigned long long h = (mix64(uq) + 1) & mask;
  for (unsigned long long n = 1; n <= mask; ++n) {
    uint4 s = ldg_slot(tab + h);
    k = slot_key(s);
    if (k == uq) return s;
    if (k == kEmptyKey) return z;
    h = (h + 1) & mask;
  }
  raise_status(status, DFT_DEV_PROBE_LIMIT);
  return z;
}

__device__ __forceinline__ uint4 first_slot(const Slot* tab, unsigned long long mask, long long q) {
  if (q < 0 || tab == nullptr) return make_uint4(0xFFFFFFFFu, 0xFFFFFFFFu, 0, 0);
  return ldg_slot(tab + (mix64(static_cast<unsigned long long>(q)) & mask));
}

// torch-style wrap of a negative index into pn[] (ngram_gpu.py:42,70 index
// pn[c] with torch semantics); ids outside [-V, V) flag DFT_DEV_BAD_TOKEN.
__device__ __forceinline__ float pn_at(const TableView& t, long long c, int32_t* status) {
  if (c < 0) c += t.V;
  if (c < 0 || c >= t.V) {
    raise_status(status, DFT_DEV_BAD_TOKEN);
    return 1.0f;
  }
  return __ldg(t.pn + c);
}

// p2(b, c) = (n_bc + beta2 * pn[c]) / (prev[b] + beta2)   (ngram_gpu.py:39-42)
// The multiply and the adds are separate float32 roundings, as in torch.
__device__ __forceinline__ float p2_from(float n_bc, float prev_b, float pn_c, float beta2) {
  return __fdiv_rn(__fadd_rn(n_bc, __fmul_rn(beta2, pn_c)), __fadd_rn(prev_b, beta2));
}
// p3 = (n_abc + beta3 * p2) / (n_ab + beta3)               (ngram_gpu.py:44-51)
__device__ __forceinline__ float p3_from(float n_abc, float n_ab, float p2, float beta3) {
  return __fdiv_rn(__fadd_rn(n_abc, __fmul_rn(beta3, p2)), __fadd_rn(n_ab, beta3));
}
// p4 = (c4 + beta4 * p3) / (n4 + beta4)                    (ngram_gpu.py:53-61)
__device__ __forceinline__ float p4_from(float c4, float n4, float p3, float beta4) {
  return __fdiv_rn(__fadd_rn(c4, __fmul_rn(beta4, p3)), __fadd_rn(n4, beta4));
}
// pmi = clamp(log p - log pn[c], -clip, clip)               (ngram_gpu.py:70)
__device__ __forceinline__ float pmi_from(float p, float log_pn, float clip) {
  float v = __fsub_rn(logf(p), log_pn);
  return fminf(fmaxf(v, -clip), clip);
}

// ------------------------------------------------------------ warp utils --
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}
__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

}  // namespace dft
