// Gated-DeltaNet tree verifier on the 5th-generation tensor cores (sm_100a).
//
// Reference: tree_gdn_split (tree_kernels.py:193-208) -> _tree_prepare,
// invert32, _tree_finish, three launches with q/k/G/beta/X round-tripping
// through HBM; the tree conv (fc1_conv.py:8-27) is a fourth launch.
//
// Here: one persistent CTA per SM loops over work units (request, k-head);
// a unit covers the R v-heads sharing that k-head.  Per unit:
//   A  the unit's activation tile (pre-conv x, or y) arrives by TMA, issued
//      at the end of the previous unit; tree conv + L2 norm in registers (one
//      thread per channel), k/q to a swizzled operand tile B = [k; q] (tf32),
//      gates and ancestor masks
//   M0 tcgen05 MMA  D0 = [k; q] k^T          -> k.k^T and q.k^T  (TMEM)
//   M1 tcgen05 MMA  D1_h = S0_h [k; q]^T     -> (k S0)^T, (q S0)^T per v-head,
//      S0_h streamed HBM -> shared by TMA (128B swizzle, no multicast); the
//      next unit's states are requested as soon as both M1 have retired
//   C  per v-head: A = strict-anc(beta k.k^T e^{G_i-G_j}), X = (I + A)^-1 by
//      forward substitution, Z = (q.k^T . D) X  -> operand tile [X; Z]
//   E1 R = beta (v - e^G (k S0)) by the thread owning TMEM lane v -> R^T tile
//   M2 tcgen05 MMA  D2_h = R^T [X; Z]^T (3xTF32) -> vn^T and (Z R)^T
//   E2 o = e^G (q S0) + Z R, vn, G stored
// Output tiles (k_hat, vn, o) are staged in shared memory and written with
// bulk async copies, one per row or tile.  The state is read once, at
// tensor-core rate, and everything else stays on chip.  Every wait is bounded (~1 s); on timeout the CTA raises
// DFT_DEV_TIMEOUT, drains what it issued (bounded), frees TMEM and exits.
#include "dft_common.cuh"

#include <cuda.h>

#include <cstring>
#include <mutex>

using namespace dft;

namespace {

constexpr int kD = 128;
constexpr int kNP = 32;            // nodes per tree, padded
constexpr int kThreads = 512;
constexpr uint32_t kTmemCols = 256;   // [0,32) k.k^T|q.k^T, [32,160) (kS0|qS0) per v-head, [160,224) vn|ZR

// shared memory map (from a 1024-byte aligned base)
constexpr uint32_t kS0Bytes = 64 * 1024;                 // one state tile: 4 K-blocks [128 x 128 B]
constexpr uint32_t OFF_S0 = 0;                           // R state tiles (TMA)
// B region (32 KB): activation tile (bf16) | [k; q] operand (4 K-blocks [64 x 128 B]) |
//                   R^T hi, lo | output staging (vn 16 KB, o)
constexpr uint32_t OFF_BOP = 2 * kS0Bytes;
// U region (32 KB): second half of an fp32 activation tile | k_hat staging |
//                   A, PD, X, [X;Z] hi, [X;Z] lo
constexpr uint32_t OFF_UNI = OFF_BOP + 32 * 1024;
constexpr uint32_t U_A = 0, U_PD = 4096, U_X = 8192, U_XZH = 16384, U_XZL = 24576;
constexpr uint32_t OFF_SMALL = OFF_UNI + 32 * 1024;
constexpr uint32_t kSmallBytes = 4096;
constexpr uint32_t kSmemBytes = OFF_SMALL + kSmallBytes + 1024;   // + alignment slack

struct Small {
  unsigned long long bar_tma[2];
  unsigned long long bar_x;
  unsigned long long bar_mma0, bar_mma1, bar_mma2, bar_drain;
  uint32_t tmem_base;
  int abort;
  uint32_t anc[kNP];               // bit j: j is i or an ancestor of i
  int cidx[kNP][3];                // conv columns of taps 0..2 (tap 3 is the node)
  float norm[2][4][kNP];           // per-warp partial sums of squares of q / k rows
  float rn[2][kNP];                // 1 / sqrt(sum + 1e-6) of q / k rows
  float G[2][kNP], beta[2][kNP], eG[2][kNP];
};
static_assert(sizeof(Small) <= kSmallBytes, "small region");

// ------------------------------------------------------------ PTX helpers --
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count));
}
__device__ __forceinline__ void mbar_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool mbar_try(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
// Bounded wait (~1 s of SM clock); false on timeout.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try(bar, parity)) {
    if (clock64() - t0 > 2000000000ll) return false;
  }
  return true;
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2, int c3,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

// UMMA shared-memory descriptor: K-major, 128-byte swizzle, 8-row groups 1 KiB apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t addr) {
  uint64_t d = (uint64_t)((addr >> 4) & 0x3FFFu);
  d |= (uint64_t)1 << 16;            // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;  // stride byte offset
  d |= (uint64_t)1 << 46;            // descriptor version (sm_100)
  d |= (uint64_t)2 << 61;            // SWIZZLE_128B
  return d;
}
// instruction descriptor: kind::tf32, D f32, A/B tf32 K-major, M x N
__host__ __device__ constexpr uint32_t idesc_tf32(int M, int N) {
  return (1u << 4) | (2u << 7) | (2u << 10) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}
__device__ __forceinline__ void mma_tf32(uint32_t dtmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                         uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::tf32 [%0], %1, %2, %3, p;\n\t}\n" ::"r"(dtmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate));
}
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// 32 TMEM lanes x 32 columns -> 32 registers per thread (thread = lane)
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  __syncwarp();  // .sync.aligned: the whole warp, converged
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}
__device__ __forceinline__ float tf32_rna(float x) {
  uint32_t r;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(r) : "f"(x));
  return __uint_as_float(r);
}
// byte offset of element (row r, k in [0, 32)) in a K-major SW128 tile of 128-byte rows
__device__ __forceinline__ uint32_t sw128_off(int r, int k) {
  return (uint32_t)(r * 128 + ((((k >> 2) ^ (r & 7)) << 4) | ((k & 3) << 2)));
}

struct TcArgs {
  dft_gdn_args g;
  dft_gdn_conv_args cv;
  int has_conv;
  int R;
  int vn_rows;     // 1: vn rows are 128 floats apart (one bulk copy per tile)
  int k_rows;      // 1: k_hat rows are 128 floats apart
};

__device__ __forceinline__ void bulk_store(void* gdst, uint32_t ssrc, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(gdst), "r"(ssrc), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_and_wait_read() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1, int c2,
                                            uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes "
      "[%0], [%1, {%2, %3, %4}], [%5];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void named_bar(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// anc row n of request b as a bit mask (bit j: j is n or an ancestor of n)
__device__ __forceinline__ uint32_t anc_mask(const float* anc, int b, int n, int N) {
  uint32_t m = 0;
  if (n >= N) return 0;
  const float* row = anc + ((int64_t)b * N + n) * N;
  if (N == kNP && (((uintptr_t)row) & 15) == 0) {
    float4 v[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) v[q] = __ldg(reinterpret_cast<const float4*>(row) + q);
#pragma unroll
    for (int q = 0; q < 8; ++q) {
      m |= (v[q].x > 0.5f ? 1u : 0u) << (4 * q);
      m |= (v[q].y > 0.5f ? 1u : 0u) << (4 * q + 1);
      m |= (v[q].z > 0.5f ? 1u : 0u) << (4 * q + 2);
      m |= (v[q].w > 0.5f ? 1u : 0u) << (4 * q + 3);
    }
  } else {
    for (int j = 0; j < N; ++j)
      if (__ldg(row + j) > 0.5f) m |= 1u << j;
  }
  return m;
}

// element (i, j) of the 32 x 32 A / PD tiles: XOR-swizzled columns so that a
// warp writing one row per lane hits 32 different banks
__device__ __forceinline__ int sq32(int i, int j) { return i * 32 + (j ^ i); }

template <typename T> __device__ __forceinline__ float roundT(float x) { return to_f32(from_f32<T>(x)); }

template <int R, typename T>
__global__ void __launch_bounds__(kThreads, 1)
    gdn_verify_tc(const __grid_constant__ CUtensorMap pool_map, const __grid_constant__ CUtensorMap act_map,
                  const TcArgs ta, int32_t* status) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem = (unsigned char*)(((uintptr_t)smem_raw + 1023) & ~(uintptr_t)1023);
  const uint32_t sbase = smem_u32(smem);
  Small& sm = *reinterpret_cast<Small*>(smem + OFF_SMALL);
  const dft_gdn_args& a = ta.g;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int N = a.N, Hk = a.Hk;
  const int KD = Hk * kD;
  const int units = a.B * Hk;
  constexpr uint32_t kBox = kNP * kD * sizeof(T);       // one activation box: 32 rows x 128 channels
  const uint32_t bar_tma0 = smem_u32(&sm.bar_tma[0]), bar_tma1 = smem_u32(&sm.bar_tma[1]);
  const uint32_t bar_x = smem_u32(&sm.bar_x);
  const uint32_t bar_m0 = smem_u32(&sm.bar_mma0), bar_m1 = smem_u32(&sm.bar_mma1), bar_m2 = smem_u32(&sm.bar_mma2);
  const uint32_t bar_dr = smem_u32(&sm.bar_drain);
  // one control thread issues every TMA and MMA; it sits in the last warp, whose
  // other lanes run no warp-collective tcgen05 op while it waits on a copy
  const bool ctl = tid == kThreads - 32;

  if (ctl) {
    mbar_init(bar_tma0, 1);
    mbar_init(bar_tma1, 1);
    mbar_init(bar_x, 1);
    mbar_init(bar_m0, 1);
    mbar_init(bar_m1, 1);
    mbar_init(bar_m2, 1);
    mbar_init(bar_dr, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    sm.abort = 0;
  }
  if (warp == 0) {
    __syncwarp();
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(&sm.tmem_base)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  auto slot_of = [&](int b) -> int {
    long long s = a.state_slots ? a.state_slots[b] : b;
    return s < 0 ? 0 : (int)s;
  };
  // both v-heads' states of unit u
  auto issue_states = [&](int u) {
    const int b = u / Hk, hk = u % Hk, slot = slot_of(b);
#pragma unroll
    for (int hl = 0; hl < R; ++hl) {
      const uint32_t bar = hl ? bar_tma1 : bar_tma0;
      mbar_expect_tx(bar, kS0Bytes);
#pragma unroll
      for (int kb = 0; kb < 4; ++kb)
        tma_load_4d(sbase + OFF_S0 + hl * kS0Bytes + kb * 16384, &pool_map, 32 * kb, 0, hk * R + hl, slot, bar);
    }
  };
  // the unit's activation tile: q, k and R v column blocks x 32 rows
  auto issue_act = [&](int u) {
    const int b = u / Hk, hk = u % Hk;
    mbar_expect_tx(bar_x, (2 + R) * kBox);
    tma_load_3d(sbase + OFF_BOP, &act_map, hk * kD, 0, b, bar_x);
    tma_load_3d(sbase + OFF_BOP + kBox, &act_map, KD + hk * kD, 0, b, bar_x);
#pragma unroll
    for (int hl = 0; hl < R; ++hl)
      tma_load_3d(sbase + OFF_BOP + (2 + hl) * kBox, &act_map, 2 * KD + (hk * R + hl) * kD, 0, b, bar_x);
  };
  int tma_pending = 0, tma_parity = 0;   // control thread: states requested but not yet consumed
  int x_pending = 0;
  if (ctl && (int)blockIdx.x < units) {
    issue_states(blockIdx.x);
    issue_act(blockIdx.x);
    tma_pending = 1;
    x_pending = 1;
  }

  // thread -> channel: t < 128 q, t < 256 k, then v of head (t - 256) / 128
  const int part = tid >> 7;
  const int d = tid & 127;
  const bool active = part < 2 + R;
  int it = 0;
  for (int u = blockIdx.x; u < units; u += gridDim.x, ++it) {
    const int b = u / Hk, hk = u % Hk;
    const uint32_t ph = it & 1;
    int col = 0;
    if (part == 0) col = hk * kD + d;
    else if (part == 1) col = KD + hk * kD + d;
    else col = 2 * KD + (hk * R + (part - 2)) * kD + d;
    // ------------------------------------------------ A0: per-node setup (warps 14, 15)
    float st0 = 0.f, st1 = 0.f, st2 = 0.f, bias = 0.f, w0 = 0.f, w1 = 0.f, w2 = 0.f, w3 = 0.f;
    if (active && ta.has_conv) {
      const dft_gdn_conv_args& cv = ta.cv;
      const long long cslot = cv.conv_slots ? cv.conv_slots[b] : b;
      const int64_t cb = cslot * cv.cs_ss + (int64_t)col * cv.cs_sc;
      st0 = load_any(cv.conv_state, cv.cs_dtype, cb);
      st1 = load_any(cv.conv_state, cv.cs_dtype, cb + cv.cs_st);
      st2 = load_any(cv.conv_state, cv.cs_dtype, cb + 2 * cv.cs_st);
      w0 = load_any(cv.weight, cv.w_dtype, (int64_t)col * 4);
      w1 = load_any(cv.weight, cv.w_dtype, (int64_t)col * 4 + 1);
      w2 = load_any(cv.weight, cv.w_dtype, (int64_t)col * 4 + 2);
      w3 = load_any(cv.weight, cv.w_dtype, (int64_t)col * 4 + 3);
      bias = cv.bias ? load_any(cv.bias, cv.w_dtype, col) : 0.f;
    }
    if (warp == 15) {
      const int n = lane;
      sm.anc[n] = anc_mask(a.anc, b, n, N);
      if (ta.has_conv) {
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          long long c = n < N ? ta.cv.cidx[((int64_t)b * N + n) * 4 + j] : 3 + n;
          if (c < 0 || c >= 3 + N) {
            if (n < N) raise_status(status, DFT_DEV_BAD_INDEX);
            c = 3 + n;
          }
          sm.cidx[n][j] = (int)c;
        }
        const long long c3 = n < N ? ta.cv.cidx[((int64_t)b * N + n) * 4 + 3] : 3 + n;
        if (n < N && c3 != 3 + n) raise_status(status, DFT_DEV_BAD_INDEX);   // tap 3 is the node itself
      }
    } else if (warp == 14) {
      // gates of the R v-heads: g, beta, G = sum over ancestors (tree_kernels.py:146-153)
      const int n = lane;
      const uint32_t m = anc_mask(a.anc, b, n, N);
#pragma unroll
      for (int hl = 0; hl < R; ++hl) {
        const int h = hk * R + hl;
        float g = 0.f, beta = 0.f;
        if (n < N) {
          const int64_t ab = (int64_t)b * a.ab_sb + (int64_t)n * a.ab_sn + h;
          const float ar = load_any(a.a, a.ab_dtype, ab) + load_any(a.dt_bias, a.dtb_dtype, h);
          const float sp = ar > 20.f ? ar : logf(1.f + expf(fminf(ar, 20.f)));
          const float dec = a.neg_exp_A ? a.neg_exp_A[h] : -expf(a.A_log[h]);
          g = dec * sp;
          beta = 1.f / (1.f + expf(-load_any(a.bg, a.ab_dtype, ab)));
        }
        float G = 0.f;
#pragma unroll
        for (int j = 0; j < kNP; ++j) {
          const float gj = __shfl_sync(0xffffffffu, g, j);
          if ((m >> j) & 1u) G += gj;
        }
        sm.G[hl][n] = G;
        sm.beta[hl][n] = beta;
        sm.eG[hl][n] = expf(G);
        if (a.aux_g && n < N) a.aux_g[(int64_t)b * a.ag_sb + (int64_t)h * a.ag_sh + n] = G;
      }
    }
    // the activation tile (requested at the end of the previous unit)
    if (!mbar_wait(bar_x, ph)) atomicExch(&sm.abort, 1);
    if (ctl) x_pending = 0;
    __syncthreads();
    if (sm.abort) break;
    // ------------------------------------------------ A1: tree conv (thread = channel)
    float yv[kNP];
    if (active) {
      const T* tile = reinterpret_cast<const T*>(smem + OFF_BOP + part * kBox) + d;   // [n][128]
      if (ta.has_conv) {
#pragma unroll
        for (int n = 0; n < kNP; ++n) {
          float tap[3];
#pragma unroll
          for (int j = 0; j < 3; ++j) {
            const int c = sm.cidx[n][j];
            tap[j] = c < 3 ? (c == 0 ? st0 : (c == 1 ? st1 : st2)) : to_f32(tile[(c - 3) * kD]);
          }
          // fc1_conv.py:20 rounds each product and sum in order j = 0..3
          float acc = __fmul_rn(tap[0], w0);
          acc = __fadd_rn(acc, __fmul_rn(tap[1], w1));
          acc = __fadd_rn(acc, __fmul_rn(tap[2], w2));
          acc = __fadd_rn(acc, __fmul_rn(to_f32(tile[n * kD]), w3));
          acc = __fadd_rn(acc, bias);
          // SiLU, then the reference stores y in x's dtype before the verifier reads it
          const float yy = roundT<T>(__fdividef(acc, 1.f + __expf(-acc)));
          yv[n] = n < N ? yy : 0.f;
        }
      } else {
#pragma unroll
        for (int n = 0; n < kNP; ++n) yv[n] = to_f32(tile[n * kD]);
      }
    } else {
#pragma unroll
      for (int n = 0; n < kNP; ++n) yv[n] = 0.f;
    }
    // ------------------------------------------------ A2: q/k row norms
    if (part < 2) {
#pragma unroll
      for (int n = 0; n < kNP; ++n) {
        const float s = warp_sum(yv[n] * yv[n]);
        if (lane == 0) sm.norm[part][warp & 3][n] = s;
      }
    }
    __syncthreads();   // also: every thread is done reading the activation tile
    if (tid < 2 * kNP) {
      const int pp = tid >> 5, n = tid & 31;
      const float ss = (sm.norm[pp][0][n] + sm.norm[pp][1][n]) + (sm.norm[pp][2][n] + sm.norm[pp][3][n]);
      sm.rn[pp][n] = 1.f / sqrtf(ss + 1e-6f);   // tree_kernels.py:144-145
    }
    __syncthreads();
    // ------------------------------------------------ A3: k -> rows 0..31, q -> rows 32..63 (tf32); k_hat staged
    if (part < 2) {
      const int kb = d >> 5, kk = d & 31;
      unsigned char* bop = smem + OFF_BOP + kb * 8192;
      float* kst = reinterpret_cast<float*>(smem + OFF_UNI) + d;   // k_hat staging [n][128]
#pragma unroll
      for (int n = 0; n < kNP; ++n) {
        float v = yv[n] * sm.rn[part][n];
        if (part == 0) v = v * a.scale;
        *reinterpret_cast<float*>(bop + sw128_off(part == 0 ? 32 + n : n, kk)) = tf32_rna(v);
        if (part == 1) kst[n * kD] = v;
      }
      if (part == 1 && a.aux_k) {
        fence_async_smem();
        named_bar(3, 128);
        if (d < 32) {
          // lane n of the first k warp writes row n (or the whole tile when rows are contiguous)
          const int n = d;
          const int heads = a.aux_k_per_v ? R : 1;
          for (int hh = 0; hh < heads; ++hh) {
            float* g = a.aux_k + (int64_t)b * a.ak_sb + (int64_t)(a.aux_k_per_v ? hk * R + hh : hk) * a.ak_sh;
            if (ta.k_rows) {
              if (n == 0) bulk_store(g, smem_u32(kst - d), N * kD * 4);
            } else if (n < N) {
              bulk_store(g + (int64_t)n * a.ak_sn, smem_u32(kst - d + n * kD), kD * 4);
            }
          }
          bulk_commit_and_wait_read();
        }
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // ------------------------------------------------ M0, M1 (one thread issues)
    if (ctl) {
      const uint32_t id0 = idesc_tf32(128, 32), id1 = idesc_tf32(128, 64);
#pragma unroll
      for (int kb = 0; kb < 4; ++kb) {
        const uint64_t db = sw128_desc(sbase + OFF_BOP + kb * 8192);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) mma_tf32(tmem + 0, db + 2 * ks, db + 2 * ks, id0, (kb | ks) != 0);
      }
      mma_commit(bar_m0);
#pragma unroll
      for (int hl = 0; hl < R; ++hl) {
        if (!mbar_wait(hl ? bar_tma1 : bar_tma0, ph)) {
          atomicExch(&sm.abort, 1);
          break;
        }
        tc_fence_after();
#pragma unroll
        for (int kb = 0; kb < 4; ++kb) {
          const uint64_t da = sw128_desc(sbase + OFF_S0 + hl * kS0Bytes + kb * 16384);
          const uint64_t db = sw128_desc(sbase + OFF_BOP + kb * 8192);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            mma_tf32(tmem + 32 + 64 * hl, da + 2 * ks, db + 2 * ks, id1, (kb | ks) != 0);
        }
      }
      tma_pending = 0;
      mma_commit(bar_m1);
    }
    // ------------------------------------------------ C + E per v-head
    for (int hl = 0; hl < R; ++hl) {
      // A and PD rows from k.k^T (lanes 0..31) and q.k^T (lanes 32..63)
      if (warp < 2) {
        if (!mbar_wait(bar_m0, ph)) atomicExch(&sm.abort, 1);
        tc_fence_after();
        float kk[32];
        tmem_ld32(tmem + ((uint32_t)(32 * warp) << 16) + 0, kk);
        const int i = lane;
        const uint32_t mi = sm.anc[i];
        const float Gi = sm.G[hl][i], bi = sm.beta[hl][i];
        float* dst = reinterpret_cast<float*>(smem + OFF_UNI + (warp == 0 ? U_A : U_PD));
#pragma unroll
        for (int j = 0; j < 32; ++j) {
          const bool anc = (mi >> j) & 1u;
          const float D = anc ? __expf(Gi - sm.G[hl][j]) : 0.f;
          dst[sq32(i, j)] = warp == 0 ? ((anc && j != i) ? bi * kk[j] * D : 0.f) : (anc ? kk[j] * D : 0.f);
        }
      }
      __syncthreads();
      if (sm.abort) break;
      // X = (I + A)^-1: one column per lane of warp 2, column kept in registers
      if (warp == 2) {
        const float* A = reinterpret_cast<const float*>(smem + OFF_UNI + U_A);
        float* X = reinterpret_cast<float*>(smem + OFF_UNI + U_X);
        const int c = lane;
        float xc[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
#pragma unroll
          for (int m = 0; m < i; m += 4) {
            s0 = fmaf(A[sq32(i, m)], xc[m], s0);
            if (m + 1 < i) s1 = fmaf(A[sq32(i, m + 1)], xc[m + 1], s1);
            if (m + 2 < i) s2 = fmaf(A[sq32(i, m + 2)], xc[m + 2], s2);
            if (m + 3 < i) s3 = fmaf(A[sq32(i, m + 3)], xc[m + 3], s3);
          }
          xc[i] = (i == c ? 1.f : 0.f) - ((s0 + s1) + (s2 + s3));
          X[i * 32 + c] = xc[i];
        }
      }
      __syncthreads();
      // [X; Z] operand (hi / lo tf32 split): rows 0..31 X, rows 32..63 Z = PD X
      {
        const float* PD = reinterpret_cast<const float*>(smem + OFF_UNI + U_PD);
        const float* X = reinterpret_cast<const float*>(smem + OFF_UNI + U_X);
        unsigned char* xzh = smem + OFF_UNI + U_XZH;
        unsigned char* xzl = smem + OFF_UNI + U_XZL;
        const int t = tid & 255, n = t >> 3, c = t & 7;   // row n, 16-byte chunk c (columns 4c..4c+3)
        float4 v;
        int row;
        if (tid < 256) {
          float4 z = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
          for (int j = 0; j < 32; ++j) {
            const float pd = PD[sq32(n, j)];
            const float4 xr = *reinterpret_cast<const float4*>(X + j * 32 + 4 * c);
            z.x = fmaf(pd, xr.x, z.x);
            z.y = fmaf(pd, xr.y, z.y);
            z.z = fmaf(pd, xr.z, z.z);
            z.w = fmaf(pd, xr.w, z.w);
          }
          v = z;
          row = 32 + n;
        } else {
          v = *reinterpret_cast<const float4*>(X + n * 32 + 4 * c);
          row = n;
        }
        float4 hi, lo;
        hi.x = tf32_rna(v.x); lo.x = tf32_rna(v.x - hi.x);
        hi.y = tf32_rna(v.y); lo.y = tf32_rna(v.y - hi.y);
        hi.z = tf32_rna(v.z); lo.z = tf32_rna(v.z - hi.z);
        hi.w = tf32_rna(v.w); lo.w = tf32_rna(v.w - hi.w);
        const uint32_t off = (uint32_t)(row * 128 + ((c ^ (row & 7)) << 4));
        *reinterpret_cast<float4*>(xzh + off) = hi;
        *reinterpret_cast<float4*>(xzl + off) = lo;
      }
      // E1: R = beta (v - e^G (k S0)) by the threads of this head's v part
      const bool epi = part == 2 + hl;
      if (epi) {
        if (!mbar_wait(bar_m1, ph)) atomicExch(&sm.abort, 1);
        tc_fence_after();
        const uint32_t taddr = tmem + ((uint32_t)(32 * (warp & 3)) << 16) + 32 + 64 * hl;
        float ks_[kNP];
        tmem_ld32(taddr, ks_);
        unsigned char* rth = smem + OFF_BOP;
        unsigned char* rtl = smem + OFF_BOP + 16384;
        const int v = d;
        // row v of R^T: eight 16-byte chunks, swizzled (chunk c at c ^ (v & 7))
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          float4 hi, lo;
          float* phi = &hi.x;
          float* plo = &lo.x;
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int n = 4 * c + e;
            const float rr = sm.beta[hl][n] * (yv[n] - sm.eG[hl][n] * ks_[n]);
            phi[e] = tf32_rna(rr);
            plo[e] = tf32_rna(rr - phi[e]);
          }
          const uint32_t off = (uint32_t)(v * 128 + ((c ^ (v & 7)) << 4));
          *reinterpret_cast<float4*>(rth + off) = hi;
          *reinterpret_cast<float4*>(rtl + off) = lo;
        }
      }
      // the states of this unit are consumed: request the next unit's
      if (ctl && hl == 0 && !sm.abort) {
        if (!mbar_wait(bar_m1, ph)) atomicExch(&sm.abort, 1);
        const int nu = u + gridDim.x;
        if (nu < units && !sm.abort) {
          issue_states(nu);
          tma_pending = 1;
          tma_parity = (it + 1) & 1;
        }
      }
      fence_async_smem();
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      if (sm.abort) break;
      // M2: D2 = R^T [X; Z]^T, 3xTF32 (hi.hi + hi.lo + lo.hi), TMEM columns 160..223
      if (ctl) {
        const uint32_t id2 = idesc_tf32(128, 64);
        const uint32_t dcol = tmem + 160;
        const uint64_t ah = sw128_desc(sbase + OFF_BOP), al = sw128_desc(sbase + OFF_BOP + 16384);
        const uint64_t bh = sw128_desc(sbase + OFF_UNI + U_XZH), bl = sw128_desc(sbase + OFF_UNI + U_XZL);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) mma_tf32(dcol, ah + 2 * ks, bh + 2 * ks, id2, ks != 0);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) mma_tf32(dcol, ah + 2 * ks, bl + 2 * ks, id2, 1);
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) mma_tf32(dcol, al + 2 * ks, bh + 2 * ks, id2, 1);
        mma_commit(bar_m2);
      }
      // E2: vn and o = e^G (q S0) + Z R, staged in the (now free) B region, bulk-stored
      if (epi) {
        if (!mbar_wait(bar_m2, (it * R + hl) & 1)) atomicExch(&sm.abort, 1);
        tc_fence_after();
        const uint32_t lanes = (uint32_t)(32 * (warp & 3)) << 16;
        const int h = hk * R + hl, v = d;
        float* vst = reinterpret_cast<float*>(smem + OFF_BOP);                  // [n][128] f32
        T* ost = reinterpret_cast<T*>(smem + OFF_BOP + 16384);                  // [n][128] T
        {
          float vn[32];
          tmem_ld32(tmem + lanes + 160, vn);
#pragma unroll
          for (int n = 0; n < kNP; ++n) vst[n * kD + v] = vn[n];
        }
        {
          float zr[32], qs[32];
          tmem_ld32(tmem + lanes + 192, zr);
          tmem_ld32(tmem + lanes + 32 + 64 * hl + 32, qs);
#pragma unroll
          for (int n = 0; n < kNP; ++n) ost[n * kD + v] = from_f32<T>(sm.eG[hl][n] * qs[n] + zr[n]);
        }
        fence_async_smem();
        named_bar(1 + hl, 128);
        if (d < 32) {
          const int n = d;
          if (a.aux_vn) {
            float* g = a.aux_vn + (int64_t)b * a.av_sb + (int64_t)h * a.av_sh;
            if (ta.vn_rows) {
              if (n == 0) bulk_store(g, smem_u32(vst), N * kD * 4);
            } else if (n < N) {
              bulk_store(g + (int64_t)n * a.av_sn, smem_u32(vst + n * kD), kD * 4);
            }
          }
          if (n < N) {
            T* g = reinterpret_cast<T*>(a.o) + (int64_t)b * a.o_sb + (int64_t)n * a.o_sn + (int64_t)h * a.o_sh;
            bulk_store(g, smem_u32(ost + n * kD), kD * sizeof(T));
          }
          bulk_commit_and_wait_read();
        }
      } else if (ctl) {
        if (!mbar_wait(bar_m2, (it * R + hl) & 1)) atomicExch(&sm.abort, 1);
      }
      tc_fence_before();
      __syncthreads();
      tc_fence_after();
      if (sm.abort) break;
    }
    if (sm.abort) break;
    // the B / U regions are free again: request the next unit's activation tile
    if (ctl) {
      const int nu = u + gridDim.x;
      if (nu < units) {
        issue_act(nu);
        x_pending = 1;
      }
    }
  }
  // ------------------------------------------------ teardown
  __syncthreads();
  if (sm.abort) {
    if (ctl) {
      raise_status(status, DFT_DEV_TIMEOUT);
      // drain what this CTA issued before freeing its shared memory / TMEM (bounded)
      if (tma_pending) {
        mbar_wait(bar_tma0, tma_parity);
        if (R > 1) mbar_wait(bar_tma1, tma_parity);
      }
      if (x_pending) mbar_wait(bar_x, it & 1);
      mma_commit(bar_dr);   // arrives once every MMA this thread issued has retired
      mbar_wait(bar_dr, 0);
    }
    __syncthreads();
  }
  tc_fence_after();
  __syncwarp();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda at link time)
typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
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

int sm_count() {
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

}  // namespace

// The tcgen05 path applies for N <= 32, Dk = Dv = 128, R = Hv / Hk in {1, 2},
// float / bfloat16 activations with o in the same dtype, a pool with unit k
// stride and 16-byte multiple strides and a known slot count, and outputs
// whose rows are 16-byte aligned (bulk copies).
bool dft_gdn_tc_applicable(const dft_gdn_args* a) {
  if (a->force_simt) return false;
  const int dt = a->conv ? a->conv->x_dtype : a->y_dtype;
  if ((dt != DFT_F32 && dt != DFT_BF16) || a->o_dtype != dt) return false;
  const int es = dt == DFT_F32 ? 4 : 2;
  if (a->N > kNP || a->Dk != kD || a->Dv != kD) return false;
  const int R = a->Hv / a->Hk;
  if (R != 1 && R != 2) return false;
  if (a->p_sk != 1 || a->p_nslots <= 0) return false;
  if ((a->p_sv * 4) % 16 || (a->p_sh * 4) % 16 || (a->p_ss * 4) % 16) return false;
  if (!al16(a->pool)) return false;
  // activation tile by TMA: unit channel stride, 16-byte row strides
  const void* act = a->conv ? a->conv->x : a->y;
  const int64_t sn = a->conv ? a->conv->x_sn : a->y_sn, sb = a->conv ? a->conv->x_sb : a->y_sb;
  if (!al16(act) || (sn * es) % 16 || (sb * es) % 16 || sn <= 0 || sb <= 0) return false;
  // bulk-copied output rows
  if (!al16(a->o) || (a->o_sb * es) % 16 || (a->o_sn * es) % 16 || (a->o_sh * es) % 16) return false;
  if (a->aux_vn && (!al16(a->aux_vn) || a->av_sb % 4 || a->av_sh % 4 || a->av_sn % 4)) return false;
  if (a->aux_k && (!al16(a->aux_k) || a->ak_sb % 4 || a->ak_sh % 4 || a->ak_sn % 4)) return false;
  if (a->Hv > 65535 || a->B > 65535) return false;
  return encode_fn() != nullptr;
}

int dft_gdn_tc_launch(const dft_gdn_args* a, int32_t* status, cudaStream_t st) {
  CUtensorMap pool_map, act_map;
  {
    const cuuint64_t dims[4] = {(cuuint64_t)kD, (cuuint64_t)kD, (cuuint64_t)a->Hv, (cuuint64_t)a->p_nslots};
    const int64_t ss = a->p_ss > 0 ? a->p_ss : (int64_t)a->Hv * a->p_sh;
    const cuuint64_t strides[3] = {(cuuint64_t)(a->p_sv * 4), (cuuint64_t)(a->p_sh * 4), (cuuint64_t)(ss * 4)};
    const cuuint32_t box[4] = {32, 128, 1, 1};
    const cuuint32_t estr[4] = {1, 1, 1, 1};
    if (encode_fn()(&pool_map, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(a->pool), dims, strides, box,
                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return DFT_ERR_UNSUPPORTED;
  }
  const int dt = a->conv ? a->conv->x_dtype : a->y_dtype;
  const int es = dt == DFT_F32 ? 4 : 2;
  {
    // activation (pre-conv x or y) as [B][N][C]: rows >= N of a 32-row box read as zeros
    const void* act = a->conv ? a->conv->x : a->y;
    const int64_t sn = a->conv ? a->conv->x_sn : a->y_sn, sb = a->conv ? a->conv->x_sb : a->y_sb;
    const int64_t C = 2 * (int64_t)a->Hk * a->Dk + (int64_t)a->Hv * a->Dv;
    const cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)a->N, (cuuint64_t)a->B};
    const cuuint64_t strides[2] = {(cuuint64_t)(sn * es), (cuuint64_t)(sb * es)};
    const cuuint32_t box[3] = {128, (cuuint32_t)kNP, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (encode_fn()(&act_map, dt == DFT_F32 ? CU_TENSOR_MAP_DATA_TYPE_FLOAT32 : CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                    const_cast<void*>(act), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return DFT_ERR_UNSUPPORTED;
  }
  TcArgs ta;
  ta.g = *a;
  ta.has_conv = a->conv != nullptr;
  if (a->conv) ta.cv = *a->conv;
  else memset(&ta.cv, 0, sizeof(ta.cv));
  ta.R = a->Hv / a->Hk;
  ta.vn_rows = a->av_sn == kD;
  ta.k_rows = a->ak_sn == kD;
  const int units = a->B * a->Hk;
  const int grid = units < sm_count() ? units : sm_count();
  auto go = [&](auto kernel) -> int {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmemBytes) != cudaSuccess)
      return DFT_ERR_CUDA;
    kernel<<<grid, kThreads, kSmemBytes, st>>>(pool_map, act_map, ta, status);
    return DFT_OK;
  };
  int rc;
  if (ta.R == 2) rc = dt == DFT_BF16 ? go(gdn_verify_tc<2, __nv_bfloat16>) : go(gdn_verify_tc<2, float>);
  else rc = dt == DFT_BF16 ? go(gdn_verify_tc<1, __nv_bfloat16>) : go(gdn_verify_tc<1, float>);
  if (rc) return rc;
  DFT_LAUNCH_CHECK();
  return DFT_OK;
}
