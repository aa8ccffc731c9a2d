// Drafter-logit scoring (fc1_builder.py:27-28):
//   lp, ids = topk(log_softmax(logits), M);  rest = log(clamp(1 - sum exp(lp), 1e-6, 1))
// One CTA of 256 threads streams one [V] row once from HBM (128-bit loads, 8
// in flight per thread; measured against 512 threads x 4, 512 x 8, 128 x 8
// and others: 312 against 360 us for 1,536 full-vocabulary rows), keeping per
// lane an online (max, sum-exp) pair and per warp a top-16 list distributed
// over lanes 0..15.  A lane offers a value to the
// warp list only when it beats the list's current 16th entry, so after the
// first few hundred elements almost every element costs one compare.  The
// (max, sum-exp) pair is rescaled once per 32-element sweep (its maximum),
// and the sweep's exponent arguments (x - m) log2 e are formed in packed
// fp32 pairs (add / mul .f32x2) and summed in pairs: 0.521 -> 0.492 ms for
// score + build at batch 64 (one vote per sweep instead of one per float4
// for the top-16 offers measured 0.533, not kept).
// Order: values descending, equal values by ascending vocabulary index.
#include "dft_common.cuh"

#include <cfloat>

using namespace dft;

namespace {

constexpr int kThreads = 256;
constexpr int kWarps = kThreads / 32;
constexpr int kTopM = 16;

struct TopList {
  float v;   // lanes 0..15: sorted descending
  int i;
  float thr;  // value of entry 15 (warp-uniform)
  int thr_i;
};

__device__ __forceinline__ bool before(float va, int ia, float vb, int ib) {
  return va > vb || (va == vb && ia < ib);
}

// Insert (val, idx) into the warp's list; warp-uniform call.
__device__ __forceinline__ void list_insert(TopList& L, float val, int idx, int lane) {
  if (!before(val, idx, L.thr, L.thr_i)) return;
  bool ahead = lane < kTopM && before(L.v, L.i, val, idx);
  int pos = __popc(__ballot_sync(0xffffffffu, ahead));
  float up_v = __shfl_up_sync(0xffffffffu, L.v, 1);
  int up_i = __shfl_up_sync(0xffffffffu, L.i, 1);
  if (lane < kTopM) {
    if (lane > pos) {
      L.v = up_v;
      L.i = up_i;
    } else if (lane == pos) {
      L.v = val;
      L.i = idx;
    }
  }
  L.thr = __shfl_sync(0xffffffffu, L.v, kTopM - 1);
  L.thr_i = __shfl_sync(0xffffffffu, L.i, kTopM - 1);
}

// Offer the 4 values of every lane whose `cand` flag is set.
__device__ __forceinline__ void offer4(TopList& L, bool cand, float4 x, int base, int lane) {
  unsigned m = __ballot_sync(0xffffffffu, cand);
  while (m) {
    int src = __ffs(m) - 1;
    m &= m - 1;
    float a = __shfl_sync(0xffffffffu, x.x, src);
    float b = __shfl_sync(0xffffffffu, x.y, src);
    float c = __shfl_sync(0xffffffffu, x.z, src);
    float d = __shfl_sync(0xffffffffu, x.w, src);
    int bi = __shfl_sync(0xffffffffu, base, src);
    list_insert(L, a, bi, lane);
    list_insert(L, b, bi + 1, lane);
    list_insert(L, c, bi + 2, lane);
    list_insert(L, d, bi + 3, lane);
  }
}

__device__ __forceinline__ void online_add(float& m, float& s, float x) {
  if (x > m) {
    s = s * __expf(m - x) + 1.f;
    m = x;
  } else if (m != -INFINITY) {
    s += __expf(x - m);
  }
}

__device__ __forceinline__ void online_add4(float& m, float& s, float4 x) {
  float mx = fmaxf(fmaxf(x.x, x.y), fmaxf(x.z, x.w));
  if (mx > m) {
    s *= __expf(m - mx);  // m = -inf initially: exp(-inf) = 0
    m = mx;
  }
  if (m != -INFINITY) s += __expf(x.x - m) + __expf(x.y - m) + __expf(x.z - m) + __expf(x.w - m);
}

template <typename T>
__device__ __forceinline__ float4 load4(const T* p, int64_t i);  // elements i..i+3
template <>
__device__ __forceinline__ float4 load4<float>(const float* p, int64_t i) {
  return __ldcs(reinterpret_cast<const float4*>(p + i));
}
template <>
__device__ __forceinline__ float4 load4<__nv_bfloat16>(const __nv_bfloat16* p, int64_t i) {
  uint2 u = __ldcs(reinterpret_cast<const uint2*>(p + i));
  float4 r;
  r.x = __uint_as_float(u.x << 16);
  r.y = __uint_as_float(u.x & 0xffff0000u);
  r.z = __uint_as_float(u.y << 16);
  r.w = __uint_as_float(u.y & 0xffff0000u);
  return r;
}
template <>
__device__ __forceinline__ float4 load4<__half>(const __half* p, int64_t i) {
  uint2 u = __ldcs(reinterpret_cast<const uint2*>(p + i));
  __half2 a = *reinterpret_cast<__half2*>(&u.x), b = *reinterpret_cast<__half2*>(&u.y);
  float2 fa = __half22float2(a), fb = __half22float2(b);
  return make_float4(fa.x, fa.y, fb.x, fb.y);
}

template <typename T>
__global__ void __launch_bounds__(kThreads) score_kernel(const T* __restrict__ logits, int64_t ld_b, int64_t ld_s,
                                                         int S, int V, float* __restrict__ lp,
                                                         int32_t* __restrict__ ids, float* __restrict__ rest) {
  const int row = blockIdx.x;  // b * S + s
  const int b = row / S, s = row % S;
  const T* x = logits + (int64_t)b * ld_b + (int64_t)s * ld_s;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;

  TopList L;
  L.v = -INFINITY;
  L.i = INT_MAX;
  L.thr = -INFINITY;
  L.thr_i = INT_MAX;
  float m = -INFINITY, sum = 0.f;
  // Block-wide pruning bound: each warp list holds 16 values >= its 16th, so no
  // value below the largest warp 16th can reach the row's top 16.  Warps publish
  // their 16th after every sweep and offer only values >= the largest published
  // one (thresholds only rise, so any stale read is still a valid bound).
  __shared__ float s_thr[kWarps];
  if (lane == 0) s_thr[warp] = -INFINITY;
  __syncthreads();
  float bound = -INFINITY;

  // scalar head up to 16-byte alignment, vector body, scalar tail
  int head = (int)((((uintptr_t)x + 15) & ~(uintptr_t)15) - (uintptr_t)x) / (int)sizeof(T);
  if (head > V) head = V;
  const int nvec = (V - head) / 4;
  const int body_end = head + nvec * 4;
  // vector body: every loop bound is block-uniform (warp-synchronous inserts)
  const int stride = kThreads * 4;  // elements per block-wide vector sweep
  int64_t base = head;
  bool first = true;
  for (; base + 8 * stride <= body_end; base += 8 * stride) {
    const int64_t e = base + (int64_t)tid * 4;
    float4 vs[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) vs[r] = load4<T>(x, e + r * stride);
    // one rescale per sweep (the sweep's maximum), then the 32 exponentials
    // in packed pairs: exp(x - m) = 2^((x - m) log2 e)
    float mx4[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) mx4[r] = fmaxf(fmaxf(vs[r].x, vs[r].y), fmaxf(vs[r].z, vs[r].w));
    {
      const float M = fmaxf(fmaxf(fmaxf(mx4[0], mx4[1]), fmaxf(mx4[2], mx4[3])),
                            fmaxf(fmaxf(mx4[4], mx4[5]), fmaxf(mx4[6], mx4[7])));
      if (M > m) {
        sum *= __expf(m - M);   // m = -inf initially: exp(-inf) = 0
        m = M;
      }
      if (m != -INFINITY) {
        const f32x2 nm = pk2(-m, -m), l2e = pk2(-kNegLog2e, -kNegLog2e);
        f32x2 acc = 0ull;
#pragma unroll
        for (int r = 0; r < 8; ++r) {
          const f32x2 d01 = mul2(add2(pk2(vs[r].x, vs[r].y), nm), l2e);
          const f32x2 d23 = mul2(add2(pk2(vs[r].z, vs[r].w), nm), l2e);
          float a0, a1, a2, a3;
          upk2(d01, a0, a1);
          upk2(d23, a2, a3);
          acc = add2(acc, pk2(ex2_approx(a0), ex2_approx(a1)));
          acc = add2(acc, pk2(ex2_approx(a2), ex2_approx(a3)));
        }
        float lo, hi;
        upk2(acc, lo, hi);
        sum += lo + hi;
      }
    }
    if (first) {
      // Seed the pruning bound from the first sweep: if at least 16 lanes hold a
      // value >= v, the row's 16th largest is >= v, so smaller values can never
      // enter the top 16.  v = the largest lane maximum with that property.
      first = false;
      float lm = -INFINITY;
#pragma unroll
      for (int r = 0; r < 8; ++r) lm = fmaxf(lm, fmaxf(fmaxf(vs[r].x, vs[r].y), fmaxf(vs[r].z, vs[r].w)));
      int ge = 0;
#pragma unroll
      for (int j = 0; j < 32; ++j) ge += __shfl_sync(0xffffffffu, lm, j) >= lm;
      float seed = ge >= kTopM ? lm : -INFINITY;
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) seed = fmaxf(seed, __shfl_xor_sync(0xffffffffu, seed, o));
      bound = fmaxf(bound, seed);
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) offer4(L, mx4[r] >= L.thr && mx4[r] >= bound, vs[r], (int)(e + r * stride), lane);
    if (lane == 0) reinterpret_cast<volatile float*>(s_thr)[warp] = L.thr;
    float t = reinterpret_cast<volatile float*>(s_thr)[lane & (kWarps - 1)];
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) t = fmaxf(t, __shfl_xor_sync(0xffffffffu, t, o));
    bound = fmaxf(bound, t);
  }
  for (; base < body_end; base += stride) {
    const int64_t e = base + (int64_t)tid * 4;
    const bool in = e < body_end;  // body length is a multiple of 4
    float4 v = in ? load4<T>(x, e) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
    if (in) online_add4(m, sum, v);
    float mx = fmaxf(fmaxf(v.x, v.y), fmaxf(v.z, v.w));
    offer4(L, in && mx >= L.thr, v, (int)e, lane);
  }
  // scalar head and tail (fewer than 8 + 4 elements per row), warp 0
  {
    const int ntail = V - body_end;
    const bool in = warp == 0 && lane < head + ntail;
    const int idx = lane < head ? lane : body_end + (lane - head);
    const float v = in ? to_f32(x[idx]) : -INFINITY;
    if (in) online_add(m, sum, v);
    unsigned msk = __ballot_sync(0xffffffffu, in && v >= L.thr);
    while (msk) {
      int src = __ffs(msk) - 1;
      msk &= msk - 1;
      list_insert(L, __shfl_sync(0xffffffffu, v, src), __shfl_sync(0xffffffffu, idx, src), lane);
    }
  }

  // ---- block reduction of (max, sum) and of the 16 warp lists
  __shared__ float s_m[kWarps], s_s[kWarps];
  __shared__ float s_v[kWarps * kTopM];
  __shared__ int s_i[kWarps * kTopM];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float om = __shfl_xor_sync(0xffffffffu, m, o);
    float os = __shfl_xor_sync(0xffffffffu, sum, o);
    float nm = fmaxf(m, om);
    sum = (nm == -INFINITY) ? 0.f : sum * __expf(m - nm) + os * __expf(om - nm);
    m = nm;
  }
  if (lane == 0) {
    s_m[warp] = m;
    s_s[warp] = sum;
  }
  if (lane < kTopM) {
    s_v[warp * kTopM + lane] = L.v;
    s_i[warp * kTopM + lane] = L.i;
  }
  __syncthreads();
  if (warp != 0) return;
  m = lane < kWarps ? s_m[lane] : -INFINITY;
  sum = lane < kWarps ? s_s[lane] : 0.f;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    float om = __shfl_xor_sync(0xffffffffu, m, o);
    float os = __shfl_xor_sync(0xffffffffu, sum, o);
    float nm = fmaxf(m, om);
    sum = (nm == -INFINITY) ? 0.f : sum * __expf(m - nm) + os * __expf(om - nm);
    m = nm;
  }
  // merge: warp 0 keeps its list and offers the other warps' entries
  for (int c = kTopM; c < kWarps * kTopM; c += 32) {
    const int j = c + lane;
    const bool in = j < kWarps * kTopM;
    float v = in ? s_v[j] : -INFINITY;
    int i = in ? s_i[j] : INT_MAX;
    unsigned msk = __ballot_sync(0xffffffffu, before(v, i, L.thr, L.thr_i));
    while (msk) {
      int src = __ffs(msk) - 1;
      msk &= msk - 1;
      list_insert(L, __shfl_sync(0xffffffffu, v, src), __shfl_sync(0xffffffffu, i, src), lane);
    }
  }
  // log_softmax = (x - max) - log(sum exp(x - max)); rest from the 16 lp's
  const float lse = logf(sum);
  float lpv = lane < kTopM ? __fsub_rn(__fsub_rn(L.v, m), lse) : 0.f;
  float ex = lane < kTopM ? expf(lpv) : 0.f;
  float tot = warp_sum(ex);
  if (lane < kTopM) {
    lp[(int64_t)row * kTopM + lane] = lpv;
    ids[(int64_t)row * kTopM + lane] = L.i;
  }
  if (lane == 0) rest[row] = logf(fminf(fmaxf(__fsub_rn(1.f, tot), 1e-6f), 1.0f));
}

}  // namespace

int dft_score_launch(const dft_build_params* p, const void* logits, int32_t dtype, int64_t ld_b, int64_t ld_s,
                     float* lp, int32_t* ids, float* rest, cudaStream_t st) {
  dim3 grid((unsigned)(p->B * p->S));
  switch (dtype) {
    case DFT_F32:
      score_kernel<float><<<grid, kThreads, 0, st>>>((const float*)logits, ld_b, ld_s, p->S, p->V, lp, ids, rest);
      break;
    case DFT_BF16:
      score_kernel<__nv_bfloat16><<<grid, kThreads, 0, st>>>((const __nv_bfloat16*)logits, ld_b, ld_s, p->S, p->V,
                                                            lp, ids, rest);
      break;
    case DFT_F16:
      score_kernel<__half><<<grid, kThreads, 0, st>>>((const __half*)logits, ld_b, ld_s, p->S, p->V, lp, ids, rest);
      break;
    default:
      return DFT_ERR_INVALID;
  }
  DFT_LAUNCH_CHECK();
  return DFT_OK;
}

extern "C" int dft_score(const dft_build_params* p, const void* logits, int32_t logits_dtype, int64_t ld_b,
                         int64_t ld_s, float* lp, int32_t* ids, float* rest, void* stream) {
  if (!p || !logits || !lp || !ids || !rest) return DFT_ERR_INVALID;
  if (p->M != kTopM) return DFT_ERR_UNSUPPORTED;
  if (p->B <= 0 || p->S <= 0 || p->V < kTopM || (int64_t)p->B * p->S > (1ll << 31) - 1) return DFT_ERR_INVALID;
  return dft_score_launch(p, logits, logits_dtype, ld_b, ld_s, lp, ids, rest, reinterpret_cast<cudaStream_t>(stream));
}
