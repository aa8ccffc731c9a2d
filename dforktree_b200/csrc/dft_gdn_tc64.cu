// Gated-DeltaNet tree verifier for trees of 33..64 nodes on the 5th-generation
// tensor cores (sm_100a) -- the plugin's default tree of 64 nodes
// (fc1_fused.py:4, FC1_TREE_N).
//
// Reference: tree_gdn_split (tree_kernels.py:193-208) -> _tree_prepare,
// invert32 (fc1_block_inverse.py:10-83), _tree_finish; the tree conv
// (fc1_conv.py:8-27) before it.
//
// One persistent CTA per SM loops over work units (request, v-head); the
// 32-node kernel's layout (dft_gdn_tc.cu) with every node dimension doubled:
//   [k; q] is a full 128-row tf32 operand, D0 = [k; q] k^T is 128 x 64,
//   D1 = S0 [k; q]^T and D2 = R^T [X; Z]^T are 128 x 128 (TMEM: 448 of 512
//   columns), the state tile streams HBM -> shared by TMA (128B swizzle, no
//   multicast) while the previous unit finishes.
// The triangular solve is the part that does not scale by doubling: a
// 64-step substitution per column would dominate the unit.  Here it runs by
// depth level instead: row i of X = (I + A)^-1 is
//     X[i] = e_i - sum_{m strict ancestor of i} A[i][m] X[m],
// so every row of one depth level is independent; eight warps take the rows
// of a level (one row per warp, lane = column pair, a loop over the row's
// ancestors), with one named barrier per level.  Z = PD X needs no solve:
// Z[n] = sum_{j ancestor-or-self of n} PD[n][j] X[j], all rows at once.
// X lives in the state tile's slot once M1 has consumed the state.
// Per unit:
//   F  tree conv in place of the unit's bf16 tile (q, k, v: 3 + 64 rows),
//      gathered by cp.async and converted by warps 8-13 as soon as the
//      previous unit's E1 has read v (alongside that unit's C2)
//   N  L2 norms -> tf32 [k; q] operand (k rows 0-63, q rows 64-127), k_hat rows
//   M0 D0 = [k; q] k^T     M1 D1 = S0 [k; q]^T
//   C1 A = strict-anc(beta k.k^T e^{G_i-G_j}), PD = anc(q.k^T e^{G_i-G_j})
//   C2 X by depth level, Z = PD X -> [X; Z] operand (3xTF32 hi / lo)
//   E1 R = beta (v - e^G (k S0)) -> R^T hi / lo in TMEM (alongside C1 / C2)
//   M2 D2 = R^T [X; Z]^T   -> vn^T, (Z R)^T, issued once every warp has
//      arrived on an mbarrier (operands ready) rather than at a CTA barrier
//   E2 o = e^G (q S0) + Z R, vn -> global memory, by warps 0-7 after their C2
//      (warps 8-13 are converting the next unit's tile meanwhile)
// Every wait is bounded (~1 s); on timeout the CTA raises DFT_DEV_TIMEOUT,
// drains what it issued (bounded), frees TMEM and exits.
#include "dft_common.cuh"
#include "dft_tc.cuh"
#include "dft_gdn_tile.cuh"

#include <cuda.h>

#include <cstring>
#include <mutex>

using namespace dft;
using namespace dft::tc;
using namespace dft::gtile;

namespace {

constexpr int kD = 128;
constexpr int kNP = 64;            // nodes per tree, padded
constexpr int kThreads = 512;
constexpr uint32_t kTmemCols = 512;
// TMEM columns: [0, 64) k.k^T (lanes 0-63) | q.k^T (lanes 64-127);
// [64, 192) (k S0)^T | (q S0)^T; [192, 320) R^T hi | lo (M2's A operand,
// lane v = row v); [320, 448) vn^T | (Z R)^T
constexpr uint32_t COL_M0 = 0, COL_M1 = 64, COL_RT = 192, COL_M2 = 320;

// shared memory map (from a 1024-byte aligned base)
constexpr uint32_t kS0Bytes = 64 * 1024;   // state tile: 4 K-blocks [128 x 128 B]; X (fp32 [64][64]) once M1 retired
constexpr uint32_t OFF_S0 = 0;
constexpr uint32_t OFF_KQ = 64 * 1024;     // [k; q] (4 K-blocks [128 x 128 B]); then [X; Z] hi (2 K-blocks), lo (+32 KB)
constexpr uint32_t OFF_U = 128 * 1024;     // A (+0), PD (+16 KB): fp32 [64][64], 16-byte chunks XOR-swizzled
constexpr uint32_t U_A = 0, U_PD = 16384;
constexpr uint32_t OFF_SMALL = 160 * 1024;
constexpr uint32_t kSmallBytes = 4096;
constexpr uint32_t OFF_ACT = OFF_SMALL + kSmallBytes;   // 3 parts x (conv rows + 64 node rows) x 128 bf16
constexpr uint32_t kMaxSmem = 227 * 1024;

struct Small {
  unsigned long long bar_s, bar_x, bar_m0, bar_m1, bar_m2, bar_dr;
  unsigned long long bar_r;        // M2's operands ready: one arrival per warp
  uint32_t tmem_base;
  int abort;
  // per-unit inputs, double-buffered: unit u uses buffer (its ordinal) % 2
  // while the next unit's are prepared in the other
  unsigned long long anc[2][kNP];  // bit j: j is i or an ancestor of i
  uint32_t taps[2][kNP];           // tile rows of conv taps 0..2 (one byte each; tap 3 is the node)
  __align__(16) float G[2][kNP];
  __align__(16) float beta[2][kNP];
  __align__(16) float eG[2][kNP];
  uint8_t order[2][kNP];           // nodes by depth, ascending index within a depth
  uint8_t lstart[2][kNP + 2];      // first position of depth d in order[] (d = 0 .. maxdepth + 1)
  int maxdepth[2];
  int s_issued;                    // state loads requested (control thread)
};
static_assert(sizeof(Small) <= kSmallBytes, "small region");

// element (i, j) of the 64 x 64 A / PD tiles: 16-byte chunks of a row
// XOR-swizzled by i mod 16
__device__ __forceinline__ int sq64(int i, int j) { return i * 64 + ((((j >> 2) ^ i) & 15) << 2) + (j & 3); }



// four consecutive bf16 channels of a tile row
__device__ __forceinline__ float4 ld4_bf16(const unsigned char* p) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u), __uint_as_float(u.y << 16),
                     __uint_as_float(u.y & 0xFFFF0000u));
}


// first channel of activation part p (q and k of k-head hk, v of v-head h)
__device__ __forceinline__ int part_channel(int p, int h, int hk, int Hk) {
  const int KD = Hk * kD;
  return p == 0 ? hk * kD : (p == 1 ? KD + hk * kD : 2 * KD + h * kD);
}

// ancestor rows of request b as 64-bit masks (bit j: j is n or an ancestor of
// n); lane n receives row n in m0 and row n + 32 in m1.  Eight rows per step,
// two columns per lane, sixteen loads in flight.
__device__ __forceinline__ void anc_masks64(const float* anc, int b, int N, int lane, unsigned long long& m0,
                                            unsigned long long& m1) {
  m0 = m1 = 0ull;
  const float* base = anc + (int64_t)b * N * N;
#pragma unroll 1
  for (int r0 = 0; r0 < N; r0 += 8) {
    float v[8][2];
#pragma unroll
    for (int e = 0; e < 8; ++e)
#pragma unroll
      for (int c = 0; c < 2; ++c) {
        const int col = lane + 32 * c;
        v[e][c] = (r0 + e < N && col < N) ? __ldg(base + (int64_t)(r0 + e) * N + col) : 0.f;
      }
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const unsigned long long row = (unsigned long long)__ballot_sync(0xffffffffu, v[e][0] > 0.5f) |
                                     ((unsigned long long)__ballot_sync(0xffffffffu, v[e][1] > 0.5f) << 32);
      const int r = r0 + e;
      if (lane == (r & 31)) {
        if (r < 32) m0 = row;
        else m1 = row;
      }
    }
  }
}

// Conv taps of unit u into buffer buf (one warp): the tile rows of taps 0..2
// of every node, one byte each (tap 3 is the node itself).  Cheap, so that
// the next unit's conv can start as soon as this unit's E1 is done.
__device__ __forceinline__ void prep_taps(const dft_gdn_args& a, const dft_gdn_conv_args& cv, Small& sm,
                                          int32_t* status, int u, int buf, int lane) {
  const int N = a.N, b = u / a.Hv;
  int64_t c4[2][4] = {{0, 0, 0, 0}, {0, 0, 0, 0}};
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int n = lane + 32 * c;
    if (n < N) {
      const int64_t* ci = cv.cidx + ((int64_t)b * N + n) * 4;
#pragma unroll
      for (int j = 0; j < 4; ++j) c4[c][j] = __ldg(reinterpret_cast<const long long*>(ci) + j);
    }
  }
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int n = lane + 32 * c;
    uint32_t packed = 0;
    if (n < N) {
#pragma unroll
      for (int j = 0; j < 3; ++j) {
        int64_t t = c4[c][j];
        if (t < 0 || t >= 3 + N) {
          raise_status(status, DFT_DEV_BAD_INDEX);
          t = 3 + n;
        }
        packed |= (uint32_t)t << (8 * j);
      }
      if (c4[c][3] != 3 + n) raise_status(status, DFT_DEV_BAD_INDEX);   // tap 3 is the node itself
    }
    sm.taps[buf][n] = packed;
  }
  __syncwarp();
}

// Masks, depth-level order and gates of unit u into buffer buf (one warp):
// ancestor masks; nodes ordered by depth (counting sort, stable by index);
// gates g, beta, G = sum of g over the ancestors in ascending order
// (tree_kernels.py:146-153), e^G, and G to aux_g.  Every global load is
// issued before any of their values is used.
__device__ __forceinline__ void prep_masks_gates(const dft_gdn_args& a, Small& sm, int u, int buf, int lane) {
  const int N = a.N, Hv = a.Hv;
  const int b = u / Hv, h = u % Hv;
  uint32_t ra[2] = {0u, 0u}, rb[2] = {0u, 0u};
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int n = lane + 32 * c;
    if (n < N) {
      const int64_t ab = (int64_t)b * a.ab_sb + (int64_t)n * a.ab_sn + h;
      ra[c] = ld_bits(a.a, a.ab_dtype, ab);
      rb[c] = ld_bits(a.bg, a.ab_dtype, ab);
    }
  }
  const uint32_t rd = ld_bits(a.dt_bias, a.dtb_dtype, h);
  const float dec = a.neg_exp_A ? __ldg(a.neg_exp_A + h) : -expf(__ldg(a.A_log + h));
  unsigned long long m[2];
  anc_masks64(a.anc, b, N, lane, m[0], m[1]);
  sm.anc[buf][lane] = m[0];
  sm.anc[buf][lane + 32] = m[1];
  // order[lstart[d] .. lstart[d + 1]) are the nodes of depth d; padding
  // nodes (no mask) are left out
  const int d0 = __popcll(m[0]) - 1, d1 = __popcll(m[1]) - 1;
  int maxd = d0 > d1 ? d0 : d1;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) maxd = max(maxd, __shfl_xor_sync(0xffffffffu, maxd, o));
  const uint32_t lt = (1u << lane) - 1u;
  int start = 0;
#pragma unroll 1
  for (int d = 0; d <= maxd; ++d) {
    const uint32_t b0 = __ballot_sync(0xffffffffu, d0 == d), b1 = __ballot_sync(0xffffffffu, d1 == d);
    if (d0 == d) sm.order[buf][start + __popc(b0 & lt)] = (uint8_t)lane;
    if (d1 == d) sm.order[buf][start + __popc(b0) + __popc(b1 & lt)] = (uint8_t)(lane + 32);
    if (lane == 0) sm.lstart[buf][d] = (uint8_t)start;
    start += __popc(b0) + __popc(b1);
  }
  if (lane == 0) {
    sm.lstart[buf][maxd + 1] = (uint8_t)start;
    sm.maxdepth[buf] = maxd;
  }
  float g[2], beta[2];
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    g[c] = 0.f;
    beta[c] = 0.f;
    if (lane + 32 * c < N) {
      const float ar = bits_f32(ra[c], a.ab_dtype) + bits_f32(rd, a.dtb_dtype);
      const float sp = ar > 20.f ? ar : logf(1.f + expf(fminf(ar, 20.f)));
      g[c] = dec * sp;
      beta[c] = 1.f / (1.f + expf(-bits_f32(rb[c], a.ab_dtype)));
    }
  }
  float G[2] = {0.f, 0.f};
#pragma unroll
  for (int hf = 0; hf < 2; ++hf) {
#pragma unroll 8
    for (int j = 0; j < 32; ++j) {
      const float gj = __shfl_sync(0xffffffffu, g[hf], j);
      const int bit = 32 * hf + j;
#pragma unroll
      for (int c = 0; c < 2; ++c)
        if ((m[c] >> bit) & 1ull) G[c] += gj;
    }
  }
#pragma unroll
  for (int c = 0; c < 2; ++c) {
    const int n = lane + 32 * c;
    sm.G[buf][n] = G[c];
    sm.beta[buf][n] = beta[c];
    sm.eG[buf][n] = expf(G[c]);
    if (a.aux_g && n < N) a.aux_g[(int64_t)b * a.ag_sb + (int64_t)h * a.ag_sh + n] = G[c];
  }
  __syncwarp();
}

template <bool CONV>
__global__ void __launch_bounds__(kThreads, 1)
    gdn_verify_tc64(const __grid_constant__ CUtensorMap pool_map, const __grid_constant__ CUtensorMap act_map,
                    const TcArgs ta, int32_t* status) {
  using T = __nv_bfloat16;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  Small& sm = *reinterpret_cast<Small*>(smem + OFF_SMALL);
  unsigned char* act = smem + OFF_ACT;
  const dft_gdn_args& a = ta.g;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int N = a.N, Hk = a.Hk, Hv = a.Hv, ratio = a.Hv / a.Hk;
  const int units = a.B * Hv;
  constexpr int kOff = CONV ? 3 : 0;                   // conv-state rows ahead of the node rows
  constexpr int kRowB = kD * 2;                        // bytes per tile row
  constexpr int kPartB = (kOff + kNP) * kRowB;         // bytes per activation part
  constexpr uint32_t kBox = kNP * kRowB;               // one TMA box: 64 node rows
  constexpr int kConvThreads = 64 * 3;                 // channel pairs of q, k, v
  const uint32_t bar_s = smem_u32(&sm.bar_s), bar_x = smem_u32(&sm.bar_x), bar_m0 = smem_u32(&sm.bar_m0);
  const uint32_t bar_m1 = smem_u32(&sm.bar_m1), bar_m2 = smem_u32(&sm.bar_m2), bar_dr = smem_u32(&sm.bar_dr);
  const uint32_t bar_r = smem_u32(&sm.bar_r);
  // lane 0 of the last warp issues every TMA and MMA; the warp reconverges
  // (__syncwarp) after each control block, so that every CTA barrier is
  // reached by whole warps
  const bool ctl = tid == kThreads - 32;
  const bool ctl_warp = warp == kThreads / 32 - 1;

  if (ctl_warp) {
    if (lane == 0) {
      mbar_init(bar_s, 1);
      mbar_init(bar_x, 1);
      mbar_init(bar_m0, 1);
      mbar_init(bar_m1, 1);
      mbar_init(bar_m2, 1);
      mbar_init(bar_dr, 1);
      mbar_init(bar_r, kThreads / 32);
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      sm.abort = 0;
      sm.s_issued = 0;
    }
    __syncwarp();
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

  const uint64_t once = l2_evict_first();
  // state of unit u's v-head into the state slot (free once the previous
  // unit's M1 has retired and its X has been consumed)
  auto issue_state = [&](int u) {
    const int b = u / Hv, h = u % Hv;
    const long long s = a.state_slots ? a.state_slots[b] : b;
    const int slot = s < 0 ? 0 : (int)s;
    mbar_expect_tx(bar_s, kS0Bytes);
#pragma unroll
    for (int kb = 0; kb < 4; ++kb) tma_load_4d(sbase + OFF_S0 + kb * 16384, &pool_map, 32 * kb, 0, h, slot, bar_s, once);
  };
  // the unit's activation tile: q, k, v column blocks x 64 node rows
  auto issue_act = [&](int u) {
    const int b = u / Hv, h = u % Hv, hk = h / ratio;
    mbar_expect_tx(bar_x, 3 * kBox);
#pragma unroll
    for (int p = 0; p < 3; ++p)
      tma_load_3d(sbase + OFF_ACT + p * kPartB + kOff * kRowB, &act_map, part_channel(p, h, hk, Hk), 0, b, bar_x,
                  once);
  };
  // control-thread bookkeeping for the drain on timeout
  int s_issued = 0, s_used = 0, x_issued = 0, x_used = 0;
  if (ctl_warp) {
    if (lane == 0 && (int)blockIdx.x < units) {
      issue_state(blockIdx.x);
      s_issued = 1;
    }
    __syncwarp();
  }

  // conv: warps 8-13, thread 256 + t -> channel pair (part t / 64, channels
  // 2 (t % 64) + {0, 1}); its weights, bias and conv state are fetched one unit
  // ahead (raw bits).  The next unit's gather and conv run once this unit's E1
  // has read v, alongside C2.
  const int ctid = tid - 256;
  const int cpart = ctid >> 6;
  const int cpair = (ctid & 63) * 2;
  const bool conv_thr = CONV && tid >= 256 && ctid < kConvThreads;
  uint4 pw = make_uint4(0u, 0u, 0u, 0u);
  uint32_t pb = 0u;
  unsigned short ps[6] = {0, 0, 0, 0, 0, 0};   // conv state (tap j, channel e) at 2 j + e
  auto load_conv = [&](int u) {
    const dft_gdn_conv_args& cv = ta.cv;
    const int b = u / Hv, h = u % Hv, hk = h / ratio;
    const int col = part_channel(cpart, h, hk, Hk) + cpair;
    pw = ldg_keep_v4(reinterpret_cast<const uint16_t*>(cv.weight) + (int64_t)col * 4);
    pb = cv.bias ? ldg_keep_u32(reinterpret_cast<const uint16_t*>(cv.bias) + col) : 0u;
    const long long cslot = cv.conv_slots ? cv.conv_slots[b] : b;
    const uint16_t* cs = reinterpret_cast<const uint16_t*>(cv.conv_state);
    const int64_t c0 = cslot * cv.cs_ss + (int64_t)col * cv.cs_sc, c1 = c0 + cv.cs_sc;
#pragma unroll
    for (int j = 0; j < 3; ++j) {
      ps[2 * j] = ldg_keep_u16(cs + c0 + j * cv.cs_st);
      ps[2 * j + 1] = ldg_keep_u16(cs + c1 + j * cv.cs_st);
    }
  };
  if (conv_thr && (int)blockIdx.x < units) load_conv(blockIdx.x);
  if (CONV && warp == 14 && (int)blockIdx.x < units) prep_taps(a, ta.cv, sm, status, blockIdx.x, 0, lane);
  // activations (x or y, a, bg) and every global write come after the
  // previous kernel has completed; the next launch may then be scheduled
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (ctl && !CONV && (int)blockIdx.x < units) {
    issue_act(blockIdx.x);
    x_issued = 1;
  }
  if (warp == 14 && (int)blockIdx.x < units) prep_masks_gates(a, sm, blockIdx.x, 0, lane);

  // tree conv in place (fc1_conv.py:8-27) of unit cu from taps buffer cbuf,
  // by the conv threads: one channel pair per thread, nodes from last to first
  // (a node's taps are its ancestors, lower indices, still unconverted)
  auto do_conv = [&](int cu, int cbuf) {
    const f32x2 w0 = pk2(__uint_as_float(pw.x << 16), __uint_as_float(pw.z << 16));
    const f32x2 w1 = pk2(__uint_as_float(pw.x & 0xFFFF0000u), __uint_as_float(pw.z & 0xFFFF0000u));
    const f32x2 w2 = pk2(__uint_as_float(pw.y << 16), __uint_as_float(pw.w << 16));
    const f32x2 w3 = pk2(__uint_as_float(pw.y & 0xFFFF0000u), __uint_as_float(pw.w & 0xFFFF0000u));
    const f32x2 bias2 = bf16x2_to_f32x2(pb);
    const bool has_bias = ta.cv.bias != nullptr;
    unsigned char* colp = act + cpart * kPartB + cpair * 2;
#pragma unroll
    for (int j = 0; j < 3; ++j) st_s32(colp + j * kRowB, (uint32_t)ps[2 * j] | ((uint32_t)ps[2 * j + 1] << 16));
    {
      const int nu = cu + gridDim.x;
      if (nu < units) load_conv(nu);   // in flight until that unit's conv
    }
    auto load = [&](int n) -> uint4 {
      const uint32_t tp = sm.taps[cbuf][n];
      return make_uint4(ld_s32(colp + (int)(tp & 0xFFu) * kRowB), ld_s32(colp + (int)((tp >> 8) & 0xFFu) * kRowB),
                        ld_s32(colp + (int)((tp >> 16) & 0xFFu) * kRowB), ld_s32(colp + (3 + n) * kRowB));
    };
    // products and sums rounded in order j = 0..3 (fc1_conv.py:20), bias, SiLU, bf16
    auto node = [&](uint4 in) -> uint32_t {
      f32x2 acc = mul2(bf16x2_to_f32x2(in.x), w0);
      acc = add2(acc, mul2(bf16x2_to_f32x2(in.y), w1));
      acc = add2(acc, mul2(bf16x2_to_f32x2(in.z), w2));
      acc = add2(acc, mul2(bf16x2_to_f32x2(in.w), w3));
      if (has_bias) acc = add2(acc, bias2);
      return f32x2_to_bf16x2(silu_hw2(acc));
    };
    int n = N - 1;
#pragma unroll 1
    for (; n >= 3; n -= 4) {
      const uint32_t ya = node(load(n)), yb = node(load(n - 1)), yc = node(load(n - 2)), yd = node(load(n - 3));
      st_s32(colp + (3 + n) * kRowB, ya);
      st_s32(colp + (2 + n) * kRowB, yb);
      st_s32(colp + (1 + n) * kRowB, yc);
      st_s32(colp + n * kRowB, yd);
    }
#pragma unroll 1
    for (; n >= 0; --n) st_s32(colp + (3 + n) * kRowB, node(load(n)));
  };

  // the pre-conv rows of unit gu into the activation tile, by the conv threads
  // (16-byte cp.async, rows >= N zero-filled); gather_wait completes them
  auto gather_tile = [&](int gu) {
    const int nb = gu / Hv, nh = gu % Hv, nhk = nh / ratio;
    const unsigned char* xb = static_cast<const unsigned char*>(ta.cv.x) + (int64_t)nb * ta.cv.x_sb * 2;
#pragma unroll 4
    for (int i = 0; i < 16; ++i) {
      const int id = ctid + kConvThreads * i;           // 0 .. 3071
      const int p = id >> 10, row = (id >> 4) & 63, c16 = id & 15;
      const bool in = row < N;
      const unsigned char* src =
          xb + ((int64_t)(in ? row : 0) * ta.cv.x_sn + part_channel(p, nh, nhk, Hk)) * 2 + c16 * 16;
      cp_async16(sbase + OFF_ACT + p * kPartB + (kOff + row) * kRowB + c16 * 16, src, in ? 16u : 0u, once);
    }
  };
  auto gather_wait = [&]() {
    cp_async_wait_all();
    named_bar(1, kConvThreads);
  };
  if (conv_thr && (int)blockIdx.x < units) gather_tile(blockIdx.x);

  int it = 0;
  for (int u = blockIdx.x; u < units; u += gridDim.x, ++it) {
    const int b = u / Hv, h = u % Hv, hk = h / ratio;
    const uint32_t ph = it & 1;
    const int cb = it & 1;   // this unit's buffer of per-unit inputs
    // ------------------------------------------------ F: the activation tile
    if (it == 0) {
      if (!CONV) {
        if (!mbar_wait(bar_x, ph)) atomicExch(&sm.abort, 1);
        if (ctl) ++x_used;
      }
      __syncwarp();
      __syncthreads();
      if (sm.abort) break;
      if (conv_thr) {
        gather_wait();
        do_conv(u, cb);
      }
    } else if (!CONV && ctl) {
      if (!mbar_wait(bar_x, ph)) atomicExch(&sm.abort, 1);
      ++x_used;
    }
    __syncwarp();
    __syncthreads();
    if (sm.abort) break;
    // ------------------------------------------------ N: norms, [k; q] operand, k_hat rows
    {
      // warp w: nodes w, w + 16, w + 32, w + 48, q and k, as eight independent chains
      const int kb = lane >> 3, ch = lane & 7;
      float4 v[4][2];
      float ss[4][2];
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int n = warp + 16 * r;
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          v[r][p] = n < N ? ld4_bf16(act + p * kPartB + (kOff + n) * kRowB + lane * 8) : make_float4(0.f, 0.f, 0.f, 0.f);
          ss[r][p] = (v[r][p].x * v[r][p].x + v[r][p].y * v[r][p].y) + (v[r][p].z * v[r][p].z + v[r][p].w * v[r][p].w);
        }
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
#pragma unroll
        for (int r = 0; r < 4; ++r)
#pragma unroll
          for (int p = 0; p < 2; ++p) ss[r][p] += __shfl_xor_sync(0xffffffffu, ss[r][p], o);
      }
      const bool write_k = a.aux_k && (a.aux_k_per_v || h % ratio == 0);
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const int n = warp + 16 * r;
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          float4 y = v[r][p];
          if (n < N) {
            const float rn = rsqrtf(ss[r][p] + 1e-6f);   // tl.rsqrt, tree_kernels.py:144-145
            y.x *= rn;
            y.y *= rn;
            y.z *= rn;
            y.w *= rn;
            if (p == 0) {
              y.x *= a.scale;
              y.y *= a.scale;
              y.z *= a.scale;
              y.w *= a.scale;
            } else if (write_k) {
              float* g = a.aux_k + (int64_t)b * a.ak_sb + (int64_t)(a.aux_k_per_v ? h : hk) * a.ak_sh +
                         (int64_t)n * a.ak_sn + lane * 4;
              *reinterpret_cast<float4*>(g) = y;
            }
          }
          const int row = p == 0 ? 64 + n : n;   // k rows 0..63, q rows 64..127
          const float4 t = make_float4(tf32_rna(y.x), tf32_rna(y.y), tf32_rna(y.z), tf32_rna(y.w));
          *reinterpret_cast<float4*>(smem + OFF_KQ + kb * 16384 + row * 128 + ((ch ^ (row & 7)) << 4)) = t;
        }
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // ------------------------------------------------ M0, M1 (one thread issues)
    if (ctl_warp) {
      if (lane == 0) {
        const uint32_t id0 = idesc_tf32(128, 64), id1 = idesc_tf32(128, 128);
#pragma unroll 1
        for (int kb = 0; kb < 4; ++kb) {
          const uint64_t db = sw128_desc(sbase + OFF_KQ + kb * 16384);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) mma_tf32(tmem + COL_M0, db + 2 * ks, db + 2 * ks, id0, (kb | ks) != 0);
        }
        mma_commit(bar_m0);
        if (!mbar_wait(bar_s, s_used & 1)) atomicExch(&sm.abort, 1);
        ++s_used;
        tc_fence_after();
#pragma unroll 1
        for (int kb = 0; kb < 4; ++kb) {
          const uint64_t da = sw128_desc(sbase + OFF_S0 + kb * 16384);
          const uint64_t db = sw128_desc(sbase + OFF_KQ + kb * 16384);
#pragma unroll
          for (int ks = 0; ks < 4; ++ks) mma_tf32(tmem + COL_M1, da + 2 * ks, db + 2 * ks, id1, (kb | ks) != 0);
        }
        mma_commit(bar_m1);
      }
      __syncwarp();
    }
    // ------------------------------------------------ the next unit's conv taps (warp 14)
    if (CONV && warp == 14) {
      const int nu = u + gridDim.x;
      if (nu < units) prep_taps(a, ta.cv, sm, status, nu, cb ^ 1, lane);
    }
    // ------------------------------------------------ C1, C2 (warps 0-7)
    if (warp < 8) {
      // C1: warp w reads TMEM lanes 32 (w % 4): k.k^T rows (w % 4 < 2) -> A,
      // q.k^T rows -> PD; columns 32 (w / 4) .. + 31
      {
        const int q4 = warp & 3, half = warp >> 2;
        const bool pd = q4 >= 2;
        if (!mbar_wait(bar_m0, ph)) atomicExch(&sm.abort, 1);
        tc_fence_after();
        float kk[32];
        tmem_ld32(tmem + ((uint32_t)(32 * q4) << 16) + COL_M0 + 32 * half, kk);
        const int i = 32 * (q4 & 1) + lane;
        const unsigned long long keep = pd ? sm.anc[cb][i] : sm.anc[cb][i] & ~(1ull << i);
        const float Gi = sm.G[cb][i], ci = pd ? 1.f : sm.beta[cb][i];
        float* dst = reinterpret_cast<float*>(smem + OFF_U + (pd ? U_PD : U_A));
        // e^{G_i - G_j} = 2^((G_i - G_j) log2 e), the differences and products in packed pairs
        const f32x2 gi2 = pk2(Gi, Gi), l2e = pk2(-kNegLog2e, -kNegLog2e), ci2 = pk2(ci, ci);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const int j0 = 32 * half + 4 * c;
          const float4 gj = *reinterpret_cast<const float4*>(&sm.G[cb][j0]);
          float a0, a1, a2, a3, p0, p1, p2, p3;
          upk2(mul2(sub2(gi2, pk2(gj.x, gj.y)), l2e), a0, a1);
          upk2(mul2(sub2(gi2, pk2(gj.z, gj.w)), l2e), a2, a3);
          upk2(mul2(mul2(ci2, pk2(kk[4 * c], kk[4 * c + 1])), pk2(ex2_approx(a0), ex2_approx(a1))), p0, p1);
          upk2(mul2(mul2(ci2, pk2(kk[4 * c + 2], kk[4 * c + 3])), pk2(ex2_approx(a2), ex2_approx(a3))), p2, p3);
          float4 o;
          o.x = ((keep >> j0) & 1ull) ? p0 : 0.f;
          o.y = ((keep >> (j0 + 1)) & 1ull) ? p1 : 0.f;
          o.z = ((keep >> (j0 + 2)) & 1ull) ? p2 : 0.f;
          o.w = ((keep >> (j0 + 3)) & 1ull) ? p3 : 0.f;
          *reinterpret_cast<float4*>(dst + sq64(i, j0)) = o;
        }
      }
      named_bar(2, 256);   // A and PD written
      // C2: X by depth level into the state slot (free once M1 has retired;
      // [k; q] is then free for the [X; Z] operand as well).  Warp w takes
      // rows w, w + 8, .. of a level; lane c owns columns c and c + 32.  Right
      // after its X row n the warp forms Z row n = sum over n's ancestors-or-self
      // j of PD[n][j] X[j] (rows of earlier levels, and its own X row in
      // registers) and writes both as [X; Z] operand rows n and 64 + n (hi / lo
      // tf32 split; one 128-byte row per K-block and store).
      if (!mbar_wait(bar_m1, ph)) atomicExch(&sm.abort, 1);
      float* X = reinterpret_cast<float*>(smem + OFF_S0);           // X[i][c] at i * 64 + c
      const float* A = reinterpret_cast<const float*>(smem + OFF_U + U_A);
      const float* PD = reinterpret_cast<const float*>(smem + OFF_U + U_PD);
      unsigned char* xzh = smem + OFF_KQ;
      unsigned char* xzl = xzh + 32768;
      auto put_row = [&](int row, float v0, float v1) {
#pragma unroll
        for (int kb2 = 0; kb2 < 2; ++kb2) {
          const float val = kb2 ? v1 : v0;
          const uint32_t off = (uint32_t)(kb2 * 16384 + row * 128 + ((((lane >> 2) ^ row) & 7) << 4) + (lane & 3) * 4);
          const float hi = tf32_rna(val);
          *reinterpret_cast<float*>(xzh + off) = hi;
          *reinterpret_cast<float*>(xzl + off) = tf32_rna(val - hi);
        }
      };
      // operand rows of padding nodes are zero
      for (int n = N + warp; n < kNP; n += 8) {
        put_row(n, 0.f, 0.f);
        put_row(64 + n, 0.f, 0.f);
      }
      const int maxd = sm.maxdepth[cb];
#pragma unroll 1
      for (int d = 0; d <= maxd; ++d) {
        const int l0 = sm.lstart[cb][d], l1 = sm.lstart[cb][d + 1];
#pragma unroll 1
        for (int k = l0 + warp; k < l1; k += 8) {
          const int i = sm.order[cb][k];
          float x0 = lane == i ? 1.f : 0.f, x1 = lane + 32 == i ? 1.f : 0.f;
          // strict ancestors, ascending (the rows of the previous levels)
          const unsigned long long sanc = sm.anc[cb][i] & ((1ull << i) - 1ull);
          unsigned long long msk = sanc;
#pragma unroll 1
          while (msk) {
            const int m = __ffsll((long long)msk) - 1;
            msk &= msk - 1ull;
            const float am = A[sq64(i, m)];
            x0 = fmaf(-am, X[m * 64 + lane], x0);
            x1 = fmaf(-am, X[m * 64 + 32 + lane], x1);
          }
          X[i * 64 + lane] = x0;
          X[i * 64 + 32 + lane] = x1;
          float z0 = 0.f, z1 = 0.f;
          msk = sanc;
#pragma unroll 1
          while (msk) {
            const int j = __ffsll((long long)msk) - 1;
            msk &= msk - 1ull;
            const float pj = PD[sq64(i, j)];
            z0 = fmaf(pj, X[j * 64 + lane], z0);
            z1 = fmaf(pj, X[j * 64 + 32 + lane], z1);
          }
          const float pii = PD[sq64(i, i)];
          z0 = fmaf(pii, x0, z0);
          z1 = fmaf(pii, x1, z1);
          put_row(i, x0, x1);
          put_row(64 + i, z0, z1);
        }
        named_bar(3, 256);   // level d written
      }
      // the operand rows, for the tensor cores; then this warp's arrival for M2
      fence_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_r);
    }
    // ------------------------------------------------ E1 (warps 8-15), alongside C1 / C2
    // R = beta (v - e^G (k S0)) by the thread owning TMEM lane v; warps 8-11
    // take nodes 0-31, warps 12-15 nodes 32-63.  Row v of R^T (hi / lo) goes
    // to TMEM lane v as M2's A operand.
    if (warp >= 8) {
      if (!mbar_wait(bar_m1, ph)) atomicExch(&sm.abort, 1);
      tc_fence_after();
      const uint32_t lanes = (uint32_t)(32 * (warp & 3)) << 16;
      const int nh = (warp >> 2) & 1;
      float ks_[32];
      tmem_ld32(tmem + lanes + COL_M1 + 32 * nh, ks_);
      const int v = tid & 127;
      const T* yv = reinterpret_cast<const T*>(act + 2 * kPartB + kOff * kRowB) + v;
#pragma unroll
      for (int c16 = 0; c16 < 2; ++c16) {
        uint32_t hi[16], lo[16];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const int n0 = 32 * nh + 16 * c16 + 4 * c;
          const float4 be4 = *reinterpret_cast<const float4*>(&sm.beta[cb][n0]);
          const float4 eg4 = *reinterpret_cast<const float4*>(&sm.eG[cb][n0]);
          const float* be = &be4.x;
          const float* eg = &eg4.x;
#pragma unroll
          for (int e = 0; e < 4; e += 2) {
            const int n = n0 + e, kx = 16 * c16 + 4 * c + e;
            // rr = beta (v - e^G (k S0)) for nodes n, n + 1 in packed pairs
            const f32x2 d = fma2(pk2(-eg[e], -eg[e + 1]), pk2(ks_[kx], ks_[kx + 1]),
                                 pk2(to_f32(yv[n * kD]), to_f32(yv[(n + 1) * kD])));
            float r0, r1;
            upk2(mul2(pk2(be[e], be[e + 1]), d), r0, r1);
            const float h0 = tf32_rna(r0), h1 = tf32_rna(r1);
            float l0, l1;
            upk2(sub2(pk2(r0, r1), pk2(h0, h1)), l0, l1);
            hi[4 * c + e] = __float_as_uint(h0);
            hi[4 * c + e + 1] = __float_as_uint(h1);
            lo[4 * c + e] = __float_as_uint(tf32_rna(l0));
            lo[4 * c + e + 1] = __float_as_uint(tf32_rna(l1));
          }
        }
        tmem_st16(tmem + lanes + COL_RT + 32 * nh + 16 * c16, hi);
        tmem_st16(tmem + lanes + COL_RT + 64 + 32 * nh + 16 * c16, lo);
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(bar_r);
      // every E1 warp has read v and the next unit's taps are prepared (warp 14):
      // the activation tile takes the next unit's rows (warps 8-13), while
      // warp 14 prepares the next unit's masks, depth order and gates (first
      // read by that unit's C1)
      named_bar(4, 256);
      const int nu = u + gridDim.x;
      if (conv_thr && nu < units) {
        gather_tile(nu);
        gather_wait();
        do_conv(nu, cb ^ 1);
      }
      if (warp == 14 && nu < units) prep_masks_gates(a, sm, nu, cb ^ 1, lane);
    }
    if (ctl_warp) {
      if (lane == 0) {
        const int nu = u + gridDim.x;
        // M2's operands: [X; Z] (warps 0-7) and R^T (warps 8-15)
        if (!mbar_wait(bar_r, ph)) atomicExch(&sm.abort, 1);
        tc_fence_after();
        if (!CONV && nu < units) {
          issue_act(nu);   // the tile is consumed (E1 has read v)
          ++x_issued;
        }
        // M2: D2 = R^T [X; Z]^T, 3xTF32 (hi.hi + hi.lo + lo.hi); K = 64 nodes in
        // 8 steps, two K-blocks of the operand
        const uint32_t id2 = idesc_tf32(128, 128);
        const uint32_t dcol = tmem + COL_M2;
        const uint32_t ah = tmem + COL_RT, al = ah + 64;
        const uint64_t bh0 = sw128_desc(sbase + OFF_KQ), bl0 = sw128_desc(sbase + OFF_KQ + 32768);
        // descriptor start addresses are in 16-byte units: one K-block is 1024 of them
#pragma unroll
        for (int ks = 0; ks < 8; ++ks)
          mma_tf32_ts(dcol, ah + 8 * ks, bh0 + 1024 * (ks >> 2) + 2 * (ks & 3), id2, ks != 0);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) mma_tf32_ts(dcol, ah + 8 * ks, bl0 + 1024 * (ks >> 2) + 2 * (ks & 3), id2, 1);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) mma_tf32_ts(dcol, al + 8 * ks, bh0 + 1024 * (ks >> 2) + 2 * (ks & 3), id2, 1);
        mma_commit(bar_m2);
        // X (in the state slot) is consumed: the slot takes the next unit's state
        if (nu < units) {
          issue_state(nu);
          ++s_issued;
        }
      }
      __syncwarp();
    }
    // ------------------------------------------------ E2: vn and o = e^G (q S0) + Z R (warps 0-7,
    // after their C2; warps 8-13 are converting the next unit's tile meanwhile)
    if (warp < 8) {
      if (!mbar_wait(bar_m2, ph)) atomicExch(&sm.abort, 1);
      tc_fence_after();
      const uint32_t lanes = (uint32_t)(32 * (warp & 3)) << 16;
      const int nh = (warp >> 2) & 1;
      const int v = tid & 127;
      float* gv = a.aux_vn ? a.aux_vn + (int64_t)b * a.av_sb + (int64_t)h * a.av_sh + v : nullptr;
      T* go = reinterpret_cast<T*>(a.o) + (int64_t)b * a.o_sb + (int64_t)h * a.o_sh + v;
#pragma unroll 1
      for (int c16 = 0; c16 < 2; ++c16) {
        const int n0 = 32 * nh + 16 * c16;
        float vn[16], zr[16], qs[16];
        tmem_ld16(tmem + lanes + COL_M2 + n0, vn);
        tmem_ld16(tmem + lanes + COL_M2 + 64 + n0, zr);
        tmem_ld16(tmem + lanes + COL_M1 + 64 + n0, qs);
#pragma unroll
        for (int e4 = 0; e4 < 16; e4 += 4) {
          const float4 eg4 = *reinterpret_cast<const float4*>(&sm.eG[cb][n0 + e4]);
          const float* eg = &eg4.x;
#pragma unroll
          for (int e = e4; e < e4 + 4; ++e) {
            const int n = n0 + e;
            if (n < N) {
              if (gv) gv[(int64_t)n * a.av_sn] = vn[e];
              go[(int64_t)n * a.o_sn] = __float2bfloat16_rn(eg[e - e4] * qs[e] + zr[e]);
            }
          }
        }
      }
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (sm.abort) break;
  }
  // ------------------------------------------------ teardown
  __syncthreads();
  if (sm.abort) {
    if (ctl_warp) {
      if (lane == 0) {
        raise_status(status, DFT_DEV_TIMEOUT);
        // drain what this CTA issued before freeing its shared memory / TMEM (bounded)
        for (; s_used < s_issued; ++s_used) mbar_wait(bar_s, s_used & 1);
        for (; x_used < x_issued; ++x_used) mbar_wait(bar_x, x_used & 1);
        mma_commit(bar_dr);   // arrives once every MMA this thread issued has retired
        mbar_wait(bar_dr, 0);
      }
      __syncwarp();
    }
    __syncthreads();
  }
  tc_fence_after();
  __syncwarp();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}


// dynamic shared memory of one launch: fixed regions + activation tile + alignment slack
uint32_t smem_bytes(bool conv) { return OFF_ACT + 3u * (uint32_t)((conv ? 3 : 0) + kNP) * kD * 2 + 1024; }

}  // namespace

// The 64-node tcgen05 path applies for 32 < N <= 64, Dk = Dv = 128, any
// Hv / Hk, bfloat16 activations and o (the fused tree conv: bfloat16 x, conv
// state and weights), a pool with unit k stride, 16-byte multiple strides and
// a known slot count, and 16-byte aligned output rows.
bool dft_gdn_tc64_applicable(const dft_gdn_args* a) {
  if (a->force_simt) return false;
  if (a->N <= 32 || a->N > kNP || a->Dk != kD || a->Dv != kD) return false;
  const int dt = a->conv ? a->conv->x_dtype : a->y_dtype;
  if (dt != DFT_BF16 || a->o_dtype != dt) return false;
  if (a->conv && (a->conv->cs_dtype != DFT_BF16 || a->conv->w_dtype != DFT_BF16 ||
                  !al16(a->conv->weight) || ((uintptr_t)a->conv->bias & 3)))
    return false;
  const int es = 2;
  if (smem_bytes(a->conv != nullptr) > kMaxSmem) return false;
  if (a->p_sk != 1 || a->p_nslots <= 0) return false;
  if ((a->p_sv * 4) % 16 || (a->p_sh * 4) % 16 || (a->p_ss * 4) % 16) return false;
  if (!al16(a->pool)) return false;
  const void* act = a->conv ? a->conv->x : a->y;
  const int64_t sn = a->conv ? a->conv->x_sn : a->y_sn, sb = a->conv ? a->conv->x_sb : a->y_sb;
  if (!al16(act) || (sn * es) % 16 || (sb * es) % 16 || sn <= 0 || sb <= 0) return false;
  if (!al16(a->o) || (a->o_sb * es) % 16 || (a->o_sn * es) % 16 || (a->o_sh * es) % 16) return false;
  if (a->aux_vn && (!al16(a->aux_vn) || a->av_sb % 4 || a->av_sh % 4 || a->av_sn % 4)) return false;
  if (a->aux_k && (!al16(a->aux_k) || a->ak_sb % 4 || a->ak_sh % 4 || a->ak_sn % 4)) return false;
  if (a->Hv > 65535 || a->B > 65535 || (int64_t)a->B * a->Hv > (1ll << 30)) return false;
  return encode_fn() != nullptr;
}

int dft_gdn_tc64_launch(const dft_gdn_args* a, int32_t* status, cudaStream_t st) {
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
  const int es = 2;
  {
    // activation (pre-conv x, or y) as [B][N][C]: rows >= N of a 64-row box read as zeros
    const void* act = a->conv ? a->conv->x : a->y;
    const int64_t sn = a->conv ? a->conv->x_sn : a->y_sn, sb = a->conv ? a->conv->x_sb : a->y_sb;
    const int64_t C = 2 * (int64_t)a->Hk * a->Dk + (int64_t)a->Hv * a->Dv;
    const cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)a->N, (cuuint64_t)a->B};
    const cuuint64_t strides[2] = {(cuuint64_t)(sn * es), (cuuint64_t)(sb * es)};
    const cuuint32_t box[3] = {128, (cuuint32_t)kNP, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (encode_fn()(&act_map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(act), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return DFT_ERR_UNSUPPORTED;
  }
  TcArgs ta;
  ta.g = *a;
  if (a->conv) ta.cv = *a->conv;
  else memset(&ta.cv, 0, sizeof(ta.cv));
  const bool conv = a->conv != nullptr;
  const uint32_t smem = smem_bytes(conv);
  const int units = a->B * a->Hv;
  const int grid = units < sm_count() ? units : sm_count();
  auto go = [&](auto kernel) -> int {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return DFT_ERR_CUDA;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = a->overlap_prev ? 1 : 0;
    if (cudaLaunchKernelEx(&cfg, kernel, pool_map, act_map, ta, status) != cudaSuccess) return DFT_ERR_CUDA;
    return DFT_OK;
  };
  const int rc = conv ? go(gdn_verify_tc64<true>) : go(gdn_verify_tc64<false>);
  if (rc) return rc;
  DFT_LAUNCH_CHECK();
  return DFT_OK;
}
