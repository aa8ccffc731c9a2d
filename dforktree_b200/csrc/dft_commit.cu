// Closed-form commit of the accepted path's recurrent state (fc1_fused.py:27-49).
// Reference: fc1_fused.snapshots (fc1_fused.py:27-49): for each layer, head
// and end node u,
//   S_u = e^{G_u} S0 + sum_{t in path, t anc-or-self of u} e^{G_u - G_t} k_t vn_t^T
// written to the intermediate state buffer (in place into the pool when the
// caller asks).  One CTA per (end, layer, request, v-head) streams the
// 64 KiB fp32 state tile once in and once out with 128-bit accesses (all
// sixteen loads of a thread in flight before the FMAs); the <= 64 path rows
// of k and e^{G_u-G_t} vn sit in shared memory.  fp32 FMA on CUDA cores: at
// L = 24 the tile needs ~6 FLOP/B, below the CUDA-core ridge on B200.
#include "dft_common.cuh"

using namespace dft;

namespace {

constexpr int kD = 128;
constexpr int kThreads = 256;
constexpr int kMaxPath = 64;

// ahead: the block `ahead` launches later (about two waves) has its path rows
// of k and vn prefetched into L2 by this block's warp 0, so that its own
// dependent row loads (after the path set-up) hit L2 instead of DRAM.
// ahead == 0x7fffffff marks rows that are not 16-byte aligned: no prefetch,
// scalar row loads.
__global__ void __launch_bounds__(kThreads, 2) gdn_commit_kernel(dft_commit_args a, int32_t* st, int ahead) {
  extern __shared__ __align__(16) float s_path[];  // [cap][kD] k*w, then [cap][kD] vn
  __shared__ int s_ids[kMaxPath];
  __shared__ float s_w[kMaxPath];
  __shared__ int s_n;

  // blockIdx.x = ((e * L + l) * B + b) * Hv + h
  int bid = blockIdx.x;
  const int h = bid % a.Hv;
  bid /= a.Hv;
  const int b = bid % a.B;
  bid /= a.B;
  const int l = bid % a.L;
  const int e = bid / a.L;
  const int tid = threadIdx.x;
  const int64_t u = a.ends[(int64_t)b * a.E + e];
  if (u < 0) return;  // fc1_fused.py:49 store masked by u >= 0
  if (u >= a.N) {
    if (tid == 0) raise_status(st, DFT_DEV_BAD_INDEX);
    return;
  }
  const int R = a.Hv / a.Hk;
  const int khead = a.aux_k_per_v ? h : h / R;
  const float* G = a.aux_g + (int64_t)l * a.ag_sl + (int64_t)b * a.ag_sb + (int64_t)h * a.ag_sh;
  const float gu = G[u];
  const int64_t slot = a.slots_in ? a.slots_in[b] : b;
  const int64_t dst = a.slots_out ? a.slots_out[b] : b;
  const float* S0 = a.state_in + (int64_t)l * a.si_sl + slot * a.si_ss + (int64_t)h * a.si_sh;
  float* So = a.state_out + (int64_t)l * a.so_sl + dst * a.so_ss + u * a.so_su + (int64_t)h * a.so_sh;
  const int k4 = (tid & 31) * 4;
  const int v0 = (tid >> 5) * 16;  // rows v0 .. v0 + 15 (the warp's 16 rows, 128 floats each)
  const bool vec = a.si_sk == 1 && a.so_sk == 1 && (a.si_sv % 4 == 0) && (a.so_sv % 4 == 0) &&
                   ((uintptr_t)S0 % 16 == 0) && ((uintptr_t)So % 16 == 0);
  // the state tile does not depend on the path: its loads go out first and
  // overlap the path set-up below
  float4 acc[16];
  if (vec) {
#pragma unroll
    for (int r = 0; r < 16; ++r) acc[r] = __ldcs(reinterpret_cast<const float4*>(S0 + (int64_t)(v0 + r) * a.si_sv + k4));
  } else {
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      const float* p = S0 + (int64_t)(v0 + r) * a.si_sv + (int64_t)k4 * a.si_sk;
      acc[r] = make_float4(p[0], p[a.si_sk], p[2 * a.si_sk], p[3 * a.si_sk]);
    }
  }
  if (tid < 32) {
    // path nodes that are ancestors-or-self of u, in path order (fc1_fused.py:30-35).
    // The ancestor row of u, the gate row (two entries per lane, N <= 64) and the
    // path entries (t and t + 32, P <= 64) are loaded at once; a path node's
    // ancestor flag and gate come from the lane holding them (no dependent
    // global loads); a ballot compacts the kept nodes in order.
    const float* anc_u = a.anc + ((int64_t)b * a.N + u) * a.N;
    const float an0 = tid < a.N ? anc_u[tid] : 0.f, an1 = tid + 32 < a.N ? anc_u[tid + 32] : 0.f;
    // the later block's request and path entries (its rows are prefetched below)
    const int64_t fblk = (int64_t)blockIdx.x + ahead;
    const bool fut = fblk < (int64_t)gridDim.x;
    int64_t fid[2] = {-1, -1};
    const float* fk = nullptr;
    const float* fv = nullptr;
    if (fut) {
      int f = (int)fblk;
      const int fh = f % a.Hv;
      f /= a.Hv;
      const int fb = f % a.B;
      f /= a.B;
      const int fl = f % a.L;
      fk = a.aux_k + (int64_t)fl * a.ak_sl + (int64_t)fb * a.ak_sb + (int64_t)(a.aux_k_per_v ? fh : fh / R) * a.ak_sh;
      fv = a.aux_vn + (int64_t)fl * a.av_sl + (int64_t)fb * a.av_sb + (int64_t)fh * a.av_sh;
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        const int t = 32 * j + tid;
        fid[j] = t < a.P ? a.path[(int64_t)fb * a.P + t] : -1;
      }
    }
    const float g0 = tid < a.N ? G[tid] : 0.f, g1 = tid + 32 < a.N ? G[tid + 32] : 0.f;
    int64_t pid[2];
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int t = 32 * j + tid;
      pid[j] = t < a.P ? a.path[(int64_t)b * a.P + t] : -1;
      if (pid[j] >= a.N) {
        raise_status(st, DFT_DEV_BAD_INDEX);
        pid[j] = -1;
      }
    }
    const int cap_n = a.P < a.N ? a.P : a.N;
    int base = 0;
#pragma unroll
    for (int j = 0; j < 2; ++j) {
      const int64_t id = pid[j];
      const int src = (int)(id & 31);
      const float alo = __shfl_sync(0xffffffffu, an0, src), ahi = __shfl_sync(0xffffffffu, an1, src);
      const float glo = __shfl_sync(0xffffffffu, g0, src), ghi = __shfl_sync(0xffffffffu, g1, src);
      const bool keep = id >= 0 && (id >= 32 ? ahi : alo) > 0.f;
      const uint32_t m = __ballot_sync(0xffffffffu, keep);
      const int pos = base + __popc(m & ((1u << tid) - 1u));
      if (keep && pos < cap_n) {
        s_ids[pos] = (int)id;
        s_w[pos] = expf(gu - (id >= 32 ? ghi : glo));
      }
      base += __popc(m);
    }
    if (tid == 0) s_n = base < cap_n ? base : cap_n;
    if (fut) {
#pragma unroll
      for (int j = 0; j < 2; ++j) {
        if (fid[j] >= 0 && fid[j] < a.N) {
          prefetch_l2(fk + fid[j] * a.ak_sn, kD * sizeof(float));
          prefetch_l2(fv + fid[j] * a.av_sn, kD * sizeof(float));
        }
      }
    }
  }
  __syncthreads();
  const int np = s_n;
  const int cap = a.P < a.N ? a.P : a.N;
  float (*skk)[kD] = reinterpret_cast<float (*)[kD]>(s_path);
  float (*svv)[kD] = reinterpret_cast<float (*)[kD]>(s_path + (size_t)cap * kD);
  const float* Kb = a.aux_k + (int64_t)l * a.ak_sl + (int64_t)b * a.ak_sb + (int64_t)khead * a.ak_sh;
  const float* Vb = a.aux_vn + (int64_t)l * a.av_sl + (int64_t)b * a.av_sb + (int64_t)h * a.av_sh;
  if (ahead != 0x7fffffff) {
    // 16-byte aligned rows (the launch checked them): one float4 of k and of vn per step
    for (int i = tid; i < np * (kD / 4); i += kThreads) {
      const int t = i >> 5, d4 = (i & 31) * 4;
      const int id = s_ids[t];
      const float w = s_w[t];
      float4 kq = *reinterpret_cast<const float4*>(Kb + (int64_t)id * a.ak_sn + d4);
      kq.x *= w;  // (k * w) (fc1_fused.py:39)
      kq.y *= w;
      kq.z *= w;
      kq.w *= w;
      *reinterpret_cast<float4*>(&skk[t][d4]) = kq;
      *reinterpret_cast<float4*>(&svv[t][d4]) = *reinterpret_cast<const float4*>(Vb + (int64_t)id * a.av_sn + d4);
    }
  } else {
    for (int i = tid; i < np * kD; i += kThreads) {
      const int t = i >> 7, d = i & 127;
      const int id = s_ids[t];
      skk[t][d] = Kb[(int64_t)id * a.ak_sn + d] * s_w[t];  // (k * w) (fc1_fused.py:39)
      svv[t][d] = Vb[(int64_t)id * a.av_sn + d];
    }
  }
  const float eg = expf(gu);
  __syncthreads();
#pragma unroll
  for (int r = 0; r < 16; ++r) {
    acc[r].x *= eg;
    acc[r].y *= eg;
    acc[r].z *= eg;
    acc[r].w *= eg;
  }
  for (int t = 0; t < np; ++t) {
    const float4 kk = *reinterpret_cast<const float4*>(&skk[t][k4]);
    // the thread's 16 vn entries are contiguous: four 128-bit shared loads
    float vr[16];
#pragma unroll
    for (int q = 0; q < 4; ++q) {
      const float4 v4 = *reinterpret_cast<const float4*>(&svv[t][v0 + 4 * q]);
      vr[4 * q] = v4.x;
      vr[4 * q + 1] = v4.y;
      vr[4 * q + 2] = v4.z;
      vr[4 * q + 3] = v4.w;
    }
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      const float vv = vr[r];
      acc[r].x = fmaf(vv, kk.x, acc[r].x);
      acc[r].y = fmaf(vv, kk.y, acc[r].y);
      acc[r].z = fmaf(vv, kk.z, acc[r].z);
      acc[r].w = fmaf(vv, kk.w, acc[r].w);
    }
  }
  if (vec) {
#pragma unroll
    for (int r = 0; r < 16; ++r) __stcs(reinterpret_cast<float4*>(So + (int64_t)(v0 + r) * a.so_sv + k4), acc[r]);
  } else {
#pragma unroll
    for (int r = 0; r < 16; ++r) {
      float* p = So + (int64_t)(v0 + r) * a.so_sv + (int64_t)k4 * a.so_sk;
      p[0] = acc[r].x;
      p[a.so_sk] = acc[r].y;
      p[2 * a.so_sk] = acc[r].z;
      p[3 * a.so_sk] = acc[r].w;
    }
  }
}

}  // namespace

extern "C" int dft_gdn_commit(const dft_commit_args* a, int32_t* dev_status, void* stream) {
  if (!a || !a->state_in || !a->state_out || !a->aux_k || !a->aux_vn || !a->aux_g || !a->anc || !a->path ||
      !a->ends)
    return DFT_ERR_INVALID;
  if (a->L <= 0 || a->B <= 0 || a->N <= 0 || a->Hk <= 0 || a->Hv <= 0 || a->P < 0 || a->E <= 0)
    return DFT_ERR_INVALID;
  if (a->Hv % a->Hk) return DFT_ERR_INVALID;
  // with a zero end stride every end node of a request writes the same output
  // tile (the in-place form): more than one end would race on it
  if (a->so_su == 0 && a->E > 1) return DFT_ERR_INVALID;
  if (a->Dk != kD || a->Dv != kD || a->P > kMaxPath || a->N > kMaxNodes) return DFT_ERR_UNSUPPORTED;
  const int64_t blocks = (int64_t)a->E * a->L * a->B * a->Hv;
  if (blocks > 0x7fffffffll) return DFT_ERR_UNSUPPORTED;
  if (a->P == 0) return DFT_ERR_UNSUPPORTED;
  const int cap = a->P < a->N ? a->P : a->N;
  const size_t sm = 2 * (size_t)cap * kD * sizeof(float);
  if (sm > 48 * 1024 &&
      cudaFuncSetAttribute(gdn_commit_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
    return DFT_ERR_CUDA;
  // the L2 prefetch needs 16-byte aligned rows
  const bool rows16 = ((uintptr_t)a->aux_k % 16 == 0) && ((uintptr_t)a->aux_vn % 16 == 0) && a->ak_sl % 4 == 0 &&
                      a->ak_sb % 4 == 0 && a->ak_sh % 4 == 0 && a->ak_sn % 4 == 0 && a->av_sl % 4 == 0 &&
                      a->av_sb % 4 == 0 && a->av_sh % 4 == 0 && a->av_sn % 4 == 0;
  int ahead = 0x7fffffff;
  if (rows16) {
    int dev = 0, sms = 148;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    ahead = 4 * sms;   // two CTAs per SM, two waves ahead
  }
  gdn_commit_kernel<<<(unsigned)blocks, kThreads, sm, reinterpret_cast<cudaStream_t>(stream)>>>(*a, dev_status, ahead);
  DFT_LAUNCH_CHECK();
  return DFT_OK;
}
