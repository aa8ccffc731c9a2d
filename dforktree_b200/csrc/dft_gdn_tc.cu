// Gated-DeltaNet tree verifier on the 5th-generation tensor cores (sm_100a).
//
// Reference: tree_gdn_split (tree_kernels.py:193-208) -> _tree_prepare,
// invert32, _tree_finish, three launches with q/k/G/beta/X round-tripping
// through HBM; the tree conv (fc1_conv.py:8-27) is a fourth launch.
//
// Here: one persistent CTA per SM loops over work units (request, k-head);
// a unit covers the R <= 2 v-heads sharing that k-head, and both heads run
// side by side on disjoint warps and buffers.  Per unit:
//   F  the unit's bf16 activation tile (pre-conv x, or y) is in shared memory
//      and already converted: the first unit's arrives by TMA and is
//      converted at the top of the loop; every later unit's is prefetched
//      into L2 by warp 7 during the previous unit's C1, gathered from there by
//      the conv threads (16-byte cp.async) and converted at the end of the
//      previous unit, while warps 8+ run that unit's M2 and E2.  Tree conv in
//      place, one thread per channel pair in packed fp32x2 arithmetic, nodes
//      from last to first (a node's taps are its ancestors, lower indices);
//      then one warp per node pair: L2 norms of q / k, the swizzled tf32
//      operand [k; q] and the fp32 k_hat rows (stored to aux_k).  The next
//      unit's gates and ancestor masks are computed by warps 10, 11, 14
//      during this unit's C1 (their loads ahead of the next states' copies)
//   M0 tcgen05 MMA  D0 = [k; q] k^T          -> k.k^T and q.k^T  (TMEM)
//   M1 tcgen05 MMA  D1_h = S0_h [k; q]^T     -> (k S0)^T, (q S0)^T per v-head,
//      head 1's issued right behind head 0's; each head's state streams HBM ->
//      its own shared slot by TMA (128B swizzle, no multicast): head 0's for
//      the next unit with this unit's M2, head 1's at the top of its unit
//   C  per v-head: A = strict-anc(beta k.k^T e^{G_i-G_j}) and PD = q.k^T . D;
//      X = (I + A)^-1 by forward substitution and Z = PD X by backward
//      substitution of Z (I + A) = PD, on two warps at once -> operand tile
//      [X; Z] (3xTF32 hi / lo), written over [k; q] once every M1 has retired
//   E1 R = beta (v - e^G (k S0)) by the thread owning TMEM lane v -> row v of
//      R^T (hi / lo) stored back to TMEM lane v (alongside C's solves)
//   M2 tcgen05 MMA  D2_h = R^T [X; Z]^T (3xTF32, A from TMEM) -> vn^T, (Z R)^T
//   E2 o = e^G (q S0) + Z R and vn from TMEM straight to global memory (per
//      node row, one warp writes 32 consecutive elements)
// The state is read once, at tensor-core rate, and everything else stays on
// chip.  Every wait is bounded (~1 s); on timeout the CTA raises
// DFT_DEV_TIMEOUT, drains what it issued (bounded), frees TMEM and exits.
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

// address of the h-th of consecutive 8-byte mbarriers
__device__ __forceinline__ uint32_t bar_at(uint32_t base, int h) { return base + 8u * (uint32_t)h; }

constexpr int kD = 128;
constexpr int kNP = 32;            // nodes per tree, padded
constexpr int kThreads = 512;
constexpr uint32_t kTmemCols = 512;
// TMEM columns: [0,32) k.k^T (lanes 0-31) | q.k^T (lanes 32-63); v-head h:
// [32 + 64h, 96 + 64h) (k S0)^T | (q S0)^T, [160 + 64h, 224 + 64h) vn^T | (Z R)^T
// and [288 + 64h, 352 + 64h) R^T hi | lo (M2's A operand, lane v = row v)
constexpr uint32_t COL_M0 = 0, COL_M1 = 32, COL_M2 = 160, COL_RT = 288;

// shared memory map (from a 1024-byte aligned base)
constexpr uint32_t kS0Bytes = 64 * 1024;   // one state tile: 4 K-blocks [128 x 128 B]
constexpr uint32_t OFF_S0 = 0;
constexpr uint32_t OFF_KQ = 64 * 1024;     // [k; q] operand (4 K-blocks [64 x 128 B]); then [X; Z] hi, lo of head h at +16 KB h
constexpr uint32_t OFF_S1 = 96 * 1024;     // head 1's state tile (TMA)
constexpr uint32_t OFF_U = 160 * 1024;     // head h at +12 KB h: A, PD, A' (4 KB each; A'[p][q] = A[31-q][31-p])
constexpr uint32_t U_A = 0, U_PD = 4096, U_AT = 8192, kUHead = 12288;
constexpr uint32_t OFF_SMALL = 184 * 1024;
constexpr uint32_t kSmallBytes = 4096;
constexpr uint32_t OFF_ACT = 188 * 1024;   // (2 + R) parts x (conv rows + 32 node rows) x 128 bf16 channels
constexpr uint32_t kMaxSmem = 227 * 1024;

struct Small {
  unsigned long long bar_s, bar_s1, bar_x, bar_m0, bar_m1[2], bar_m2[2], bar_dr;
  uint32_t tmem_base;
  int abort;
  // per-unit inputs, double-buffered: unit u uses buffer (its ordinal) % 2
  // while the next unit's are prepared in the other
  uint32_t anc[2][kNP];            // bit j: j is i or an ancestor of i
  // byte offsets, within one activation part, of the rows that conv taps
  // 0..2 and 3 (the node itself) read: conv-state rows 0..2, node rows 3..
  __align__(16) uint4 taps[2][kNP];
  __align__(16) float G[2][2][kNP];   // [buffer][v-head][node]
  __align__(16) float beta[2][2][kNP];
  __align__(16) float eG[2][2][kNP];
  int s1_issued;                   // head-1 state loads requested (any thread that issues one)
};
static_assert(sizeof(Small) <= kSmallBytes, "small region");


// ancestor rows of request b as bit masks (bit j: j is n or an ancestor of
// n); lane n receives row n.  One coalesced row read per step.
__device__ __forceinline__ uint32_t anc_mask_warp(const float* anc, int b, int N, int lane) {
  uint32_t mine = 0;
  const float* base = anc + (int64_t)b * N * N;
  // eight rows per step, all four steps in flight (one memory latency)
#pragma unroll
  for (int n0 = 0; n0 < kNP; n0 += 8) {
    float v[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) v[e] = (n0 + e < N && lane < N) ? __ldg(base + (int64_t)(n0 + e) * N + lane) : 0.f;
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      const uint32_t row = __ballot_sync(0xffffffffu, v[e] > 0.5f);
      if (lane == n0 + e) mine = row;
    }
  }
  return mine;
}

// element (i, j) of the 32 x 32 A / PD tiles: 16-byte chunks of a row
// XOR-swizzled by i mod 8, so that a warp storing one row chunk per lane
// covers all banks in the minimum number of wavefronts
__device__ __forceinline__ int sq32(int i, int j) { return i * 32 + ((((j >> 2) ^ i) & 7) << 2) + (j & 3); }





// four consecutive channels of a tile row
__device__ __forceinline__ float4 ld4(const unsigned char* p, __nv_bfloat16) {
  const uint2 u = *reinterpret_cast<const uint2*>(p);
  return make_float4(__uint_as_float(u.x << 16), __uint_as_float(u.x & 0xFFFF0000u), __uint_as_float(u.y << 16),
                     __uint_as_float(u.y & 0xFFFF0000u));
}

// first channel of activation part p (q, k, v of head hk*R + p - 2) of k-head hk
__device__ __forceinline__ int part_channel(int p, int hk, int Hk, int R) {
  const int KD = Hk * kD;
  return p == 0 ? hk * kD : (p == 1 ? KD + hk * kD : 2 * KD + (hk * R + p - 2) * kD);
}

// Per-unit masks and gates of unit u into buffer buf, by three warps (role 2:
// ancestor masks and conv taps; roles 0, 1: gates of v-head role).  Every
// global load is issued before any of their values is used.
template <int R, bool CONV>
__device__ __forceinline__ void prep_unit(const dft_gdn_args& a, const dft_gdn_conv_args& cv, Small& sm,
                                          int32_t* status, int u, int buf, int role, int lane) {
  const int N = a.N, Hk = a.Hk;
  const int b = u / Hk, hk = u % Hk;
  const int n = lane;
  const int hl = role, h = hk * R + hl;
  const bool gate = role < 2 && hl < R && n < N;
  // gate inputs (raw bits) and conv columns first
  uint32_t ra = 0, rb = 0, rd = 0;
  float dec = 0.f;
  if (gate) {
    const int64_t ab = (int64_t)b * a.ab_sb + (int64_t)n * a.ab_sn + h;
    ra = ld_bits(a.a, a.ab_dtype, ab);
    rb = ld_bits(a.bg, a.ab_dtype, ab);
    rd = ld_bits(a.dt_bias, a.dtb_dtype, h);
    dec = a.neg_exp_A ? __ldg(a.neg_exp_A + h) : -expf(__ldg(a.A_log + h));
  }
  int64_t c4[4] = {0, 0, 0, 0};
  if (CONV && role == 2 && n < N) {
    const int64_t* ci = cv.cidx + ((int64_t)b * N + n) * 4;
#pragma unroll
    for (int j = 0; j < 4; ++j) c4[j] = __ldg(reinterpret_cast<const long long*>(ci) + j);
  }
  const uint32_t m = anc_mask_warp(a.anc, b, N, lane);
  if (role == 2) {
    sm.anc[buf][n] = m;
    if (CONV) {
      uint32_t row[3] = {0u, 0u, 0u};
      if (n < N) {
#pragma unroll
        for (int j = 0; j < 3; ++j) {
          int64_t c = c4[j];
          if (c < 0 || c >= 3 + N) {
            raise_status(status, DFT_DEV_BAD_INDEX);
            c = 3 + n;
          }
          row[j] = (uint32_t)c;
        }
        if (c4[3] != 3 + n) raise_status(status, DFT_DEV_BAD_INDEX);   // tap 3 is the node itself
      }
      constexpr uint32_t kRowBytes = kD * 2;
      sm.taps[buf][n] = make_uint4(row[0] * kRowBytes, row[1] * kRowBytes, row[2] * kRowBytes, (3u + n) * kRowBytes);
    }
  } else if (hl < R) {
    // g, beta, G = sum of g over the ancestors in ascending order (tree_kernels.py:146-153)
    float g = 0.f, beta = 0.f;
    if (gate) {
      const float ar = bits_f32(ra, a.ab_dtype) + bits_f32(rd, a.dtb_dtype);
      const float sp = ar > 20.f ? ar : logf(1.f + expf(fminf(ar, 20.f)));
      g = dec * sp;
      beta = 1.f / (1.f + expf(-bits_f32(rb, a.ab_dtype)));
    }
    float G = 0.f;
#pragma unroll 8
    for (int j = 0; j < kNP; ++j) {
      const float gj = __shfl_sync(0xffffffffu, g, j);
      if ((m >> j) & 1u) G += gj;
    }
    sm.G[buf][hl][n] = G;
    sm.beta[buf][hl][n] = beta;
    sm.eG[buf][hl][n] = expf(G);
    if (a.aux_g && n < N) a.aux_g[(int64_t)b * a.ag_sb + (int64_t)h * a.ag_sh + n] = G;
  }
  __syncwarp();
}

template <int R, bool CONV>
__global__ void __launch_bounds__(kThreads, 1)
    gdn_verify_tc(const __grid_constant__ CUtensorMap pool_map, const __grid_constant__ CUtensorMap act_map,
                  const TcArgs ta, int32_t* status) {
  using T = __nv_bfloat16;
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // 1024-byte aligned base, offset within the shared array (keeps the shared
  // address space visible to the compiler: LDS / STS rather than generic access)
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const uint32_t sbase = smem_u32(smem);
  Small& sm = *reinterpret_cast<Small*>(smem + OFF_SMALL);
  unsigned char* act = smem + OFF_ACT;
  const dft_gdn_args& a = ta.g;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int N = a.N, Hk = a.Hk;
  const int units = a.B * Hk;
  constexpr int kOff = CONV ? 3 : 0;                   // conv-state rows ahead of the node rows
  constexpr int kRowB = kD * 2;                        // bytes per tile row
  constexpr int kPartB = (kOff + kNP) * kRowB;         // bytes per activation part
  constexpr uint32_t kBox = kNP * kRowB;               // one TMA box: 32 node rows
  const uint32_t bar_s = smem_u32(&sm.bar_s), bar_s1 = smem_u32(&sm.bar_s1), bar_x = smem_u32(&sm.bar_x);
  const uint32_t bar_m0 = smem_u32(&sm.bar_m0), bar_dr = smem_u32(&sm.bar_dr);
  // per-head mbarriers are consecutive 8-byte words: head h's is base + 8 h
  // (an address, not a local array that a runtime head index would put in
  // local memory)
  const uint32_t bar_m1_0 = smem_u32(&sm.bar_m1[0]), bar_m2_0 = smem_u32(&sm.bar_m2[0]);
  // lane 0 of the last warp issues every TMA and MMA; the warp reconverges
  // (__syncwarp) after each control block, so that every CTA barrier is
  // reached by whole warps
  const bool ctl = tid == kThreads - 32;
  const bool ctl_warp = warp == kThreads / 32 - 1;

  if (ctl_warp) {
    if (lane == 0) {
      mbar_init(bar_s, 1);
      mbar_init(bar_s1, 1);
      mbar_init(bar_x, 1);
      mbar_init(bar_m0, 1);
      mbar_init(bar_at(bar_m1_0, 0), 1);
      mbar_init(bar_at(bar_m1_0, 1), 1);
      mbar_init(bar_at(bar_m2_0, 0), 1);
      mbar_init(bar_at(bar_m2_0, 1), 1);
      mbar_init(bar_dr, 1);
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      sm.abort = 0;
      sm.s1_issued = 0;
    }
    __syncwarp();   // the control warp reconverges before the next CTA barrier
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
  // state of v-head hl of unit u into that head's slot (free once the previous
  // unit's M1 of the head has retired)
  auto issue_state = [&](int u, int hl) {
    const int b = u / Hk, hk = u % Hk;
    const long long s = a.state_slots ? a.state_slots[b] : b;
    const int slot = s < 0 ? 0 : (int)s;
    const uint32_t bar = hl ? bar_s1 : bar_s, dst = sbase + (hl ? OFF_S1 : OFF_S0);
    mbar_expect_tx(bar, kS0Bytes);
#pragma unroll
    for (int kb = 0; kb < 4; ++kb) tma_load_4d(dst + kb * 16384, &pool_map, 32 * kb, 0, hk * R + hl, slot, bar, once);
  };
  // the unit's activation tile: q, k and R v column blocks x 32 node rows
  auto issue_act = [&](int u) {
    const int b = u / Hk, hk = u % Hk;
    mbar_expect_tx(bar_x, (2 + R) * kBox);
#pragma unroll
    for (int p = 0; p < 2 + R; ++p)
      tma_load_3d(sbase + OFF_ACT + p * kPartB + kOff * kRowB, &act_map, part_channel(p, hk, Hk, R), 0, b, bar_x,
                  once);
  };
  // control-thread bookkeeping for the drain on timeout
  int s_issued = 0, s_used = 0, s1_used = 0, x_issued = 0, x_used = 0;
  // Up to the grid-dependency wait below, the CTA reads only what the previous
  // kernel in the stream does not write (dft_gdn_args.overlap_prev): states,
  // conv state and weights, ancestor masks, conv columns.  Launched without
  // the programmatic attribute, the wait returns at once.
  if (ctl_warp) {
    if (lane == 0 && (int)blockIdx.x < units) {
      issue_state(blockIdx.x, 0);
      s_issued = 1;
      if (R == 2) {
        issue_state(blockIdx.x, 1);
        sm.s1_issued = 1;
      }
    }
    __syncwarp();   // the control warp reconverges before the next CTA barrier
  }

  // conv: thread -> channel pair (part tid / 64, channels 2 (tid % 64) + {0, 1});
  // its weights, bias and conv state are fetched one unit ahead (raw bits)
  const int cpart = tid >> 6;
  const int cpair = (tid & 63) * 2;
  const bool conv_thr = CONV && tid < 64 * (2 + R);
  uint4 pw = make_uint4(0u, 0u, 0u, 0u);
  uint32_t pb = 0u;
  // conv state of tap j, channels (col, col + 1) as one bf16 pair (scalars, not an
  // array: the lambdas capture it by reference)
  uint32_t ps0 = 0u, ps1 = 0u, ps2 = 0u;
  auto load_conv = [&](int u) {
    const dft_gdn_conv_args& cv = ta.cv;
    const int b = u / Hk, hk = u % Hk;
    const int col = part_channel(cpart, hk, Hk, R) + cpair;
    // bf16 weights [C][4]: channels col, col + 1 are 16 contiguous bytes.  The
    // loads are volatile so that they issue here, a unit ahead of their use,
    // rather than being re-issued next to it
    pw = ldg_keep_v4(reinterpret_cast<const uint16_t*>(cv.weight) + (int64_t)col * 4);
    pb = cv.bias ? ldg_keep_u32(reinterpret_cast<const uint16_t*>(cv.bias) + col) : 0u;
    const long long cslot = cv.conv_slots ? cv.conv_slots[b] : b;
    const uint16_t* cs = reinterpret_cast<const uint16_t*>(cv.conv_state);
    const int64_t c0 = cslot * cv.cs_ss + (int64_t)col * cv.cs_sc, c1 = c0 + cv.cs_sc;
    // raw loads only: nothing here waits for them (they are consumed a unit later)
    ps0 = (uint32_t)ldg_keep_u16(cs + c0) | ((uint32_t)ldg_keep_u16(cs + c1) << 16);
    ps1 = (uint32_t)ldg_keep_u16(cs + c0 + cv.cs_st) | ((uint32_t)ldg_keep_u16(cs + c1 + cv.cs_st) << 16);
    ps2 = (uint32_t)ldg_keep_u16(cs + c0 + 2 * cv.cs_st) | ((uint32_t)ldg_keep_u16(cs + c1 + 2 * cv.cs_st) << 16);
  };
  if (conv_thr && (int)blockIdx.x < units) load_conv(blockIdx.x);
  if (warp == 15 && (int)blockIdx.x < units) prep_unit<R, CONV>(a, ta.cv, sm, status, blockIdx.x, 0, 2, lane);
  // activations (x or y, a, bg) and every global write come after the
  // previous kernel has completed; the next launch may then be scheduled (its
  // CTAs take an SM as soon as this kernel's CTA there exits)
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (ctl && !CONV && (int)blockIdx.x < units) {
    issue_act(blockIdx.x);   // with the fused conv the conv threads gather it
    x_issued = 1;
  }
  if ((warp == 13 || warp == 14) && (int)blockIdx.x < units)
    prep_unit<R, CONV>(a, ta.cv, sm, status, blockIdx.x, 0, warp - 13, lane);

  // F2, tree conv in place (fc1_conv.py:8-27) of unit cu from taps buffer cbuf,
  // by the conv threads (warps 0 .. 2 + R - 1): the first unit's at the top of
  // the loop, every later unit's at the end of the previous unit, alongside
  // that unit's M2 and E2 (the activation tile is free once E1 has read v)
  auto do_conv = [&](int cu, int cbuf) {
      const f32x2 w0 = pk2(__uint_as_float(pw.x << 16), __uint_as_float(pw.z << 16));
      const f32x2 w1 = pk2(__uint_as_float(pw.x & 0xFFFF0000u), __uint_as_float(pw.z & 0xFFFF0000u));
      const f32x2 w2 = pk2(__uint_as_float(pw.y << 16), __uint_as_float(pw.w << 16));
      const f32x2 w3 = pk2(__uint_as_float(pw.y & 0xFFFF0000u), __uint_as_float(pw.w & 0xFFFF0000u));
      const f32x2 bias2 = bf16x2_to_f32x2(pb);
      const bool has_bias = ta.cv.bias != nullptr;
      unsigned char* colp = act + cpart * kPartB + cpair * 2;   // this thread's channel pair, row 0
      st_s32(colp, ps0);
      st_s32(colp + kRowB, ps1);
      st_s32(colp + 2 * kRowB, ps2);
      {
        const int nu = cu + gridDim.x;
        if (nu < units) load_conv(nu);   // in flight until that unit's conv
      }
      // one node: its three taps and itself (raw bf16 pairs), then products and
      // sums rounded in order j = 0..3 (fc1_conv.py:20), bias, SiLU, bf16
      auto load = [&](int n) -> uint4 {
        const uint4 tp = sm.taps[cbuf][n];   // one 16-byte broadcast load: the four row offsets
        return make_uint4(ld_s32(colp + tp.x), ld_s32(colp + tp.y), ld_s32(colp + tp.z), ld_s32(colp + tp.w));
      };
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
  // (16-byte cp.async, rows >= N zero-filled); gather_wait completes them for
  // all conv threads.  The first unit's go out right after the grid-dependency
  // wait, alongside its gate preparation
  auto gather_tile = [&](int gu) {
    constexpr int kConvThreads = 64 * (2 + R);
    const int nb = gu / Hk, nhk = gu % Hk;
    const unsigned char* xb = static_cast<const unsigned char*>(ta.cv.x) + (int64_t)nb * ta.cv.x_sb * 2;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int id = tid + kConvThreads * i;
      const int p = id >> 9, row = (id >> 4) & 31, c16 = id & 15;
      const bool in = row < N;
      const unsigned char* src =
          xb + ((int64_t)(in ? row : 0) * ta.cv.x_sn + part_channel(p, nhk, Hk, R)) * 2 + c16 * 16;
      cp_async16(sbase + OFF_ACT + p * kPartB + (kOff + row) * kRowB + c16 * 16, src, in ? 16u : 0u, once);
    }
  };
  auto gather_wait = [&]() {
    cp_async_wait_all();
    named_bar(1, 64 * (2 + R));
  };
  if (conv_thr && (int)blockIdx.x < units) gather_tile(blockIdx.x);

  int it = 0;
  for (int u = blockIdx.x; u < units; u += gridDim.x, ++it) {
    const int b = u / Hk, hk = u % Hk;
    const uint32_t ph = it & 1;
    const int cb = it & 1;   // this unit's buffer of per-unit inputs
    // ------------------------------------------------ F1: the activation tile
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
      // the tile (y, no conv) streamed by TMA since the previous unit's E1
      if (!mbar_wait(bar_x, ph)) atomicExch(&sm.abort, 1);
      ++x_used;
    }
    __syncwarp();
    __syncthreads();
    if (sm.abort) break;
    if (R == 2 && ctl && it > 0) {
      // head 1's state for this unit (its slot is free since the previous
      // unit's M1): streamed during the norms and C1, whose shared-memory
      // traffic is light, and needed only at this unit's second M1
      issue_state(u, 1);
      ++sm.s1_issued;
    }
    // ------------------------------------------------ F3: norms, [k; q] operand, k_hat rows
    {
      // warp w: nodes w and w + 16, q and k, as four independent chains
      const int kb = lane >> 3, ch = lane & 7;                         // K-block, 16-byte chunk of channels 4 lane..
      float4 v[2][2];
      float ss[2][2];
#pragma unroll
      for (int r = 0; r < 2; ++r) {
        const int n = warp + 16 * r;
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          v[r][p] = n < N ? ld4(act + p * kPartB + (kOff + n) * kRowB + lane * 8, T()) : make_float4(0.f, 0.f, 0.f, 0.f);
          ss[r][p] = (v[r][p].x * v[r][p].x + v[r][p].y * v[r][p].y) + (v[r][p].z * v[r][p].z + v[r][p].w * v[r][p].w);
        }
      }
#pragma unroll
      for (int o = 16; o >= 1; o >>= 1) {
#pragma unroll
        for (int r = 0; r < 2; ++r)
#pragma unroll
          for (int p = 0; p < 2; ++p) ss[r][p] += __shfl_xor_sync(0xffffffffu, ss[r][p], o);
      }
#pragma unroll
      for (int r = 0; r < 2; ++r) {
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
            } else if (a.aux_k) {
              // k_hat row n -> aux_k: 16 bytes per lane, one coalesced 512-byte row per warp
              const int heads = a.aux_k_per_v ? R : 1;
              for (int hh = 0; hh < heads; ++hh) {
                float* g = a.aux_k + (int64_t)b * a.ak_sb + (int64_t)(a.aux_k_per_v ? hk * R + hh : hk) * a.ak_sh +
                           (int64_t)n * a.ak_sn + lane * 4;
                *reinterpret_cast<float4*>(g) = y;
              }
            }
          }
          const int row = p == 0 ? 32 + n : n;   // k rows 0..31, q rows 32..63
          const float4 t = make_float4(tf32_rna(y.x), tf32_rna(y.y), tf32_rna(y.z), tf32_rna(y.w));
          *reinterpret_cast<float4*>(smem + OFF_KQ + kb * 8192 + row * 128 + ((ch ^ (row & 7)) << 4)) = t;
        }
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // ------------------------------------------------ M0, M1 of every head (one thread issues)
    if (ctl_warp) {
      if (lane == 0) {
        const uint32_t id0 = idesc_tf32(128, 32), id1 = idesc_tf32(128, 64);
  #pragma unroll 1
        for (int kb = 0; kb < 4; ++kb) {
          const uint64_t db = sw128_desc(sbase + OFF_KQ + kb * 8192);
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
          const uint64_t db = sw128_desc(sbase + OFF_KQ + kb * 8192);
  #pragma unroll
          for (int ks = 0; ks < 4; ++ks) mma_tf32(tmem + COL_M1, da + 2 * ks, db + 2 * ks, id1, (kb | ks) != 0);
        }
        mma_commit(bar_at(bar_m1_0, 0));
        if (R == 2) {
          // head 1's M1 (its state streamed into its own slot since the previous unit's M1)
          if (!mbar_wait(bar_s1, s1_used & 1)) atomicExch(&sm.abort, 1);
          ++s1_used;
          tc_fence_after();
  #pragma unroll 1
          for (int kb = 0; kb < 4; ++kb) {
            const uint64_t da = sw128_desc(sbase + OFF_S1 + kb * 16384);
            const uint64_t db = sw128_desc(sbase + OFF_KQ + kb * 8192);
  #pragma unroll
            for (int ks = 0; ks < 4; ++ks) mma_tf32(tmem + COL_M1 + 64, da + 2 * ks, db + 2 * ks, id1, (kb | ks) != 0);
          }
          mma_commit(bar_at(bar_m1_0, 1));
        }
      }
      __syncwarp();   // the control warp reconverges before the next CTA barrier
    }
    // ------------------------------------------------ the next unit's masks and gates (warps 10, 11, 14)
    // by warps idle until E1, early in the unit: their loads go out before the
    // next unit's state copies are queued behind them
    if (warp == 10 || warp == 11 || warp == 14) {
      const int nu = u + gridDim.x;
      if (nu < units) prep_unit<R, CONV>(a, ta.cv, sm, status, nu, cb ^ 1, warp == 14 ? 2 : warp - 10, lane);
    }
    // ------------------------------------------------ the next unit's pre-conv rows into L2 (warp 7, idle until E1)
    // so that the conv threads' gather at the end of this unit reads L2, not DRAM
    if (CONV && warp == 7) {
      const int nu = u + gridDim.x;
      if (nu < units && lane < N) {
        const int nb = nu / Hk, nhk = nu % Hk;
        const unsigned char* xr =
            static_cast<const unsigned char*>(ta.cv.x) + ((int64_t)nb * ta.cv.x_sb + (int64_t)lane * ta.cv.x_sn) * 2;
#pragma unroll
        for (int p = 0; p < 2 + R; ++p) prefetch_l2(xr + part_channel(p, nhk, Hk, R) * 2, 256u);
      }
    }
    // ------------------------------------------------ C1: A and PD of every head (8 warps)
    // warp w: rows from TMEM lanes 32 (w % 4) (k.k^T for w % 4 == 0, q.k^T for 1),
    // head (w / 4) % 2, columns 16 (w / 8) .. + 15
    if ((warp & 3) < 2 && ((warp >> 2) & 1) < R) {
      const int hh = (warp >> 2) & 1, half = warp >> 3;
      const bool pd = warp & 1;
      if (!mbar_wait(bar_m0, ph)) atomicExch(&sm.abort, 1);
      tc_fence_after();
      float kk[16];
      tmem_ld16(tmem + ((uint32_t)(32 * (warp & 3)) << 16) + COL_M0 + 16 * half, kk);
      // A: strict ancestors, beta_i k.k^T e^{G_i-G_j}; PD: ancestors, q.k^T e^{G_i-G_j}
      const int i = lane;
      const uint32_t keep = pd ? sm.anc[cb][i] : sm.anc[cb][i] & ~(1u << i);
      const float Gi = sm.G[cb][hh][i], ci = pd ? 1.f : sm.beta[cb][hh][i];
      float* dst = reinterpret_cast<float*>(smem + OFF_U + hh * kUHead + (pd ? U_PD : U_A));
      // e^{G_i - G_j} = 2^((G_i - G_j) log2 e), the differences and products in packed pairs
      const f32x2 gi2 = pk2(Gi, Gi), l2e = pk2(-kNegLog2e, -kNegLog2e), ci2 = pk2(ci, ci);
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        const int j0 = 16 * half + 4 * c;
        const float4 gj = *reinterpret_cast<const float4*>(&sm.G[cb][hh][j0]);
        float a0, a1, a2, a3, p0, p1, p2, p3;
        upk2(mul2(sub2(gi2, pk2(gj.x, gj.y)), l2e), a0, a1);
        upk2(mul2(sub2(gi2, pk2(gj.z, gj.w)), l2e), a2, a3);
        upk2(mul2(mul2(ci2, pk2(kk[4 * c], kk[4 * c + 1])), pk2(ex2_approx(a0), ex2_approx(a1))), p0, p1);
        upk2(mul2(mul2(ci2, pk2(kk[4 * c + 2], kk[4 * c + 3])), pk2(ex2_approx(a2), ex2_approx(a3))), p2, p3);
        float4 o;
        o.x = ((keep >> j0) & 1u) ? p0 : 0.f;
        o.y = ((keep >> (j0 + 1)) & 1u) ? p1 : 0.f;
        o.z = ((keep >> (j0 + 2)) & 1u) ? p2 : 0.f;
        o.w = ((keep >> (j0 + 3)) & 1u) ? p3 : 0.f;
        *reinterpret_cast<float4*>(dst + sq32(i, j0)) = o;
        if (!pd) {
          // A'[31 - j][31 - i] = A[i][j]: lane i writes column 31 - i of four rows
          float* at = reinterpret_cast<float*>(smem + OFF_U + hh * kUHead + U_AT);
          at[sq32(31 - j0, 31 - i)] = o.x;
          at[sq32(30 - j0, 31 - i)] = o.y;
          at[sq32(29 - j0, 31 - i)] = o.z;
          at[sq32(28 - j0, 31 - i)] = o.w;
        }
      }
      // head hh's A / PD / A' are written: release its two solver warps
      // (named barrier 2 + hh: the C1 warps of the head arrive, the two solver
      // warps wait; no other warp waits for C1).  Head 1's solvers are its C1
      // warps 4 and 5 themselves: they wait rather than arrive
      if (!(R == 2 && (warp == 4 || warp == 5)))
        asm volatile("bar.arrive %0, %1;" ::"r"(2 + hh), "r"(hh ? 128 : 192) : "memory");
    }
    // ------------------------------------------------ X, Z per head (warps 2, 3 / 4, 5)
    // Both are unit lower-triangular solves r_i = init_i - sum_{m < i} L[i][m] r_m,
    // one column / row per lane, in registers:
    //   X = (I + A)^-1:  L = A,  init = e_c (lane c = column c of X)
    //   Z = PD X, i.e. Z (I + A) = PD:  L = A' (A'[p][q] = A[31-q][31-p]),
    //   init = row n of PD reversed, z_j = r_{31-j} (lane n = row n of Z)
    // They go into the [X; Z] operand (hi / lo tf32 split) over [k; q] once
    // every M1 has retired.
    // The four solver warps sit on the four SM sub-partitions (warp % 4):
    // head 0's on warps 2, 3, head 1's on warps 4, 5 once their C1 part is done.
    if (warp == 2 || warp == 3 || (R == 2 && (warp == 4 || warp == 5))) {
      const int hh = warp >= 4 ? 1 : 0;
      const bool zw = warp & 1;
      named_bar(2 + hh, hh ? 128 : 192);   // head hh's C1 is done
      const float* L = reinterpret_cast<const float*>(smem + OFF_U + hh * kUHead + (zw ? U_AT : U_A));
      // r_i in packed pairs rp[i / 2] = (r_{2k}, r_{2k+1}): each fma.rn.f32x2
      // performs the two lanes' FMAs of the scalar chains s0 / s1 and s2 / s3
      // (same operands, same order, same rounding)
      f32x2 rp[16];
      if (!zw) {
#pragma unroll
        for (int k = 0; k < 16; ++k) rp[k] = pk2(2 * k == lane ? 1.f : 0.f, 2 * k + 1 == lane ? 1.f : 0.f);
      } else {
        const float* PD = reinterpret_cast<const float*>(smem + OFF_U + hh * kUHead + U_PD);
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          const float4 q = *reinterpret_cast<const float4*>(PD + sq32(lane, 4 * c));
          rp[15 - 2 * c] = pk2(q.y, q.x);   // r[30 - 4c], r[31 - 4c]
          rp[14 - 2 * c] = pk2(q.w, q.z);   // r[28 - 4c], r[29 - 4c]
        }
      }
      // row i of L in 16-byte chunks: entries at and above the diagonal are
      // zero (L is strictly lower triangular), so whole chunks can be used
#pragma unroll
      for (int i = 1; i < 32; ++i) {
        f32x2 s01 = 0ull, s23 = 0ull;
#pragma unroll
        for (int m = 0; m < i; m += 4) {
          const float4 l4 = *reinterpret_cast<const float4*>(L + sq32(i, m));
          s01 = fma2(pk2(l4.x, l4.y), rp[m >> 1], s01);
          s23 = fma2(pk2(l4.z, l4.w), rp[(m >> 1) + 1], s23);
        }
        float s0, s1, s2, s3, lo, hi;
        upk2(s01, s0, s1);
        upk2(s23, s2, s3);
        upk2(rp[i >> 1], lo, hi);
        if (i & 1) hi = hi - ((s0 + s1) + (s2 + s3));
        else lo = lo - ((s0 + s1) + (s2 + s3));
        rp[i >> 1] = pk2(lo, hi);
      }
      float r[32];
#pragma unroll
      for (int k = 0; k < 16; ++k) upk2(rp[k], r[2 * k], r[2 * k + 1]);
      if (!mbar_wait(bar_at(bar_m1_0, R - 1), ph)) atomicExch(&sm.abort, 1);   // [k; q] is free
      unsigned char* xzh = smem + OFF_KQ + hh * 16384;
      unsigned char* xzl = xzh + 8192;
      if (!zw) {
        // lane c writes column c of every X row i (a full 128-byte row per step)
        const int c = lane;
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const uint32_t off = (uint32_t)(i * 128 + ((((c >> 2) ^ i) & 7) << 4) + (c & 3) * 4);
          const float hi = tf32_rna(r[i]);
          *reinterpret_cast<float*>(xzh + off) = hi;
          *reinterpret_cast<float*>(xzl + off) = tf32_rna(r[i] - hi);
        }
      } else {
        // lane n writes Z row n (z_j = r_{31-j}) as operand row 32 + n
        const int row = 32 + lane;
#pragma unroll
        for (int c = 0; c < 8; ++c) {
          float4 hi, lo;
          hi.x = tf32_rna(r[31 - 4 * c]); lo.x = tf32_rna(r[31 - 4 * c] - hi.x);
          hi.y = tf32_rna(r[30 - 4 * c]); lo.y = tf32_rna(r[30 - 4 * c] - hi.y);
          hi.z = tf32_rna(r[29 - 4 * c]); lo.z = tf32_rna(r[29 - 4 * c] - hi.z);
          hi.w = tf32_rna(r[28 - 4 * c]); lo.w = tf32_rna(r[28 - 4 * c] - hi.w);
          const uint32_t off = (uint32_t)(row * 128 + ((c ^ (row & 7)) << 4));
          *reinterpret_cast<float4*>(xzh + off) = hi;
          *reinterpret_cast<float4*>(xzl + off) = lo;
        }
      }
    }
    if (ctl_warp) {
      if (lane == 0) {

      }
      __syncwarp();   // the control warp reconverges before its E1 (warp-collective TMEM loads)
    }
    // ------------------------------------------------ E1 (warps 8-15), alongside the X / Z solves
    if (warp >= 8 && ((warp - 8) >> 2) < R) {
      // E1: R = beta (v - e^G (k S0)) by the four warps owning head hh's TMEM
      // lanes; row v of R^T (hi / lo tf32 split) goes to TMEM lane v as M2's A
      const int hh = (warp - 8) >> 2;
      if (!mbar_wait(bar_at(bar_m1_0, hh), ph)) atomicExch(&sm.abort, 1);   // (k S0) of head hh ready
      tc_fence_after();
      const uint32_t lanes = (uint32_t)(32 * (warp & 3)) << 16;
      float ks_[kNP];
      tmem_ld32(tmem + lanes + COL_M1 + 64 * hh, ks_);
      const int v = tid & 127;
      const T* yv = reinterpret_cast<const T*>(act + (2 + hh) * kPartB + kOff * kRowB) + v;
#pragma unroll
      for (int half = 0; half < 2; ++half) {
        uint32_t hi[16], lo[16];
#pragma unroll
        for (int c = 0; c < 4; ++c) {
          const float4 be4 = *reinterpret_cast<const float4*>(&sm.beta[cb][hh][16 * half + 4 * c]);
          const float4 eg4 = *reinterpret_cast<const float4*>(&sm.eG[cb][hh][16 * half + 4 * c]);
#pragma unroll
          for (int e = 0; e < 4; e += 2) {
            const int n = 16 * half + 4 * c + e;
            const float be0 = e ? be4.z : be4.x, be1 = e ? be4.w : be4.y;
            const float eg0 = e ? eg4.z : eg4.x, eg1 = e ? eg4.w : eg4.y;
            // rr = beta (v - e^G (k S0)) for nodes n, n + 1 in packed pairs
            const f32x2 d = fma2(pk2(-eg0, -eg1), pk2(ks_[n], ks_[n + 1]), pk2(to_f32(yv[n * kD]), to_f32(yv[(n + 1) * kD])));
            float r0, r1;
            upk2(mul2(pk2(be0, be1), d), r0, r1);
            const float h0 = tf32_rna(r0), h1 = tf32_rna(r1);
            float l0, l1;
            upk2(sub2(pk2(r0, r1), pk2(h0, h1)), l0, l1);
            hi[4 * c + e] = __float_as_uint(h0);
            hi[4 * c + e + 1] = __float_as_uint(h1);
            lo[4 * c + e] = __float_as_uint(tf32_rna(l0));
            lo[4 * c + e + 1] = __float_as_uint(tf32_rna(l1));
          }
        }
        tmem_st16(tmem + lanes + COL_RT + 64 * hh + 16 * half, hi);
        tmem_st16(tmem + lanes + COL_RT + 64 * hh + 32 + 16 * half, lo);
      }
    }
    fence_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    if (sm.abort) break;
    if (ctl_warp) {
      if (lane == 0) {
        // the tile is consumed: request the next unit's (with the fused conv the
        // conv threads gather it themselves at the end of this unit)
        const int nu = u + gridDim.x;
        if (!CONV && nu < units) {
          issue_act(nu);
          ++x_issued;
        }
        // M2 per head: D2 = R^T [X; Z]^T, 3xTF32 (hi.hi + hi.lo + lo.hi)
        const uint32_t id2 = idesc_tf32(128, 64);
  #pragma unroll 1
        for (int hh = 0; hh < R; ++hh) {
          const uint32_t dcol = tmem + COL_M2 + 64 * hh;
          const uint32_t ah = tmem + COL_RT + 64 * hh, al = ah + 32;   // R^T hi / lo in TMEM, 8 columns per K step
          const uint64_t bh = sw128_desc(sbase + OFF_KQ + hh * 16384), bl = sw128_desc(sbase + OFF_KQ + hh * 16384 + 8192);
  #pragma unroll
          for (int ks = 0; ks < 4; ++ks) mma_tf32_ts(dcol, ah + 8 * ks, bh + 2 * ks, id2, ks != 0);
  #pragma unroll
          for (int ks = 0; ks < 4; ++ks) mma_tf32_ts(dcol, ah + 8 * ks, bl + 2 * ks, id2, 1);
  #pragma unroll
          for (int ks = 0; ks < 4; ++ks) mma_tf32_ts(dcol, al + 8 * ks, bh + 2 * ks, id2, 1);
          mma_commit(bar_at(bar_m2_0, hh));
        }
        {
          // every M1 of this unit has retired (the solvers waited for it): the
          // head-0 slot takes the next unit's state.  Issued here rather than
          // right after M1, so that the copy's shared-memory writes do not meet
          // the solves' and E1's traffic; head 1's goes out at the top of the
          // next unit (measured: 1.5 % and 4.5 % faster than both after M1)
          const int nu = u + gridDim.x;
          if (nu < units) {
            if (!mbar_wait(bar_at(bar_m1_0, R - 1), ph)) atomicExch(&sm.abort, 1);
            issue_state(nu, 0);
            ++s_issued;
          }
        }
      }
      __syncwarp();   // the control warp reconverges before the next CTA barrier
    }
    // ------------------------------------------------ E2: vn and o = e^G (q S0) + Z R
    // thread v holds column v: for each node row a warp writes 32 consecutive
    // elements (128 bytes of vn, 64 bytes of o); no shared-memory staging
    if (warp >= 8 && ((warp - 8) >> 2) < R) {
      const int hh = (warp - 8) >> 2;
      if (!mbar_wait(bar_at(bar_m2_0, hh), ph)) atomicExch(&sm.abort, 1);
      tc_fence_after();
      const uint32_t lanes = (uint32_t)(32 * (warp & 3)) << 16;
      const int h = hk * R + hh, v = tid & 127;
      // per-node output pointers advance by the node strides (one 64-bit add
      // per store rather than an index multiply); vn and o rows of nodes >= N
      // are not written
      char* gvp = a.aux_vn ? reinterpret_cast<char*>(a.aux_vn + (int64_t)b * a.av_sb + (int64_t)h * a.av_sh + v) : nullptr;
      char* gop = reinterpret_cast<char*>(reinterpret_cast<T*>(a.o) + (int64_t)b * a.o_sb + (int64_t)h * a.o_sh + v);
      const int64_t vstep = a.av_sn * (int64_t)sizeof(float), ostep = a.o_sn * (int64_t)sizeof(T);
#pragma unroll 1
      for (int half = 0; half < 2; ++half) {
        float vn[16], zr[16], qs[16];
        tmem_ld16(tmem + lanes + COL_M2 + 64 * hh + 16 * half, vn);
        tmem_ld16(tmem + lanes + COL_M2 + 64 * hh + 32 + 16 * half, zr);
        tmem_ld16(tmem + lanes + COL_M1 + 64 * hh + 32 + 16 * half, qs);
        const int nv = N - 16 * half;   // nodes of this half that exist (uniform)
        float ov[16];
#pragma unroll
        for (int e4 = 0; e4 < 16; e4 += 4) {
          const float4 eg4 = *reinterpret_cast<const float4*>(&sm.eG[cb][hh][16 * half + e4]);
          ov[e4] = eg4.x * qs[e4] + zr[e4];
          ov[e4 + 1] = eg4.y * qs[e4 + 1] + zr[e4 + 1];
          ov[e4 + 2] = eg4.z * qs[e4 + 2] + zr[e4 + 2];
          ov[e4 + 3] = eg4.w * qs[e4 + 3] + zr[e4 + 3];
        }
        if (nv >= 16) {
          if (gvp) {
#pragma unroll
            for (int e = 0; e < 16; ++e, gvp += vstep) *reinterpret_cast<float*>(gvp) = vn[e];
          }
#pragma unroll
          for (int e = 0; e < 16; ++e, gop += ostep) *reinterpret_cast<T*>(gop) = __float2bfloat16_rn(ov[e]);
        } else {
#pragma unroll
          for (int e = 0; e < 16; ++e) {
            if (e < nv) {
              if (gvp) *reinterpret_cast<float*>(gvp + e * vstep) = vn[e];
              *reinterpret_cast<T*>(gop + e * ostep) = __float2bfloat16_rn(ov[e]);
            }
          }
        }
      }
    }
    // ------------------------------------------------ the next unit's tile and conv (warps 0 .. 2 + R - 1)
    // The conv threads gather the next unit's pre-conv rows with 16-byte
    // cp.async (a DRAM round trip, not queued behind shared-memory traffic as
    // a TMA write is here), then convert them while warps 8+ run M2 and E2.
    if (conv_thr) {
      const int nu = u + gridDim.x;
      if (nu < units) {
        gather_tile(nu);
        gather_wait();
        do_conv(nu, cb ^ 1);
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
        for (; s1_used < sm.s1_issued; ++s1_used) mbar_wait(bar_s1, s1_used & 1);
        for (; x_used < x_issued; ++x_used) mbar_wait(bar_x, x_used & 1);
        mma_commit(bar_dr);   // arrives once every MMA this thread issued has retired
        mbar_wait(bar_dr, 0);
      }
      __syncwarp();   // the control warp reconverges before the next CTA barrier
    }
    __syncthreads();
  }
  tc_fence_after();
  __syncwarp();
  if (warp == 0) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
}


// dynamic shared memory of one launch: fixed regions + activation tile + alignment slack
uint32_t smem_bytes(int R, bool conv) {
  const uint32_t act = (uint32_t)(2 + R) * (uint32_t)((conv ? 3 : 0) + kNP) * kD * 2;
  return OFF_ACT + act + 1024;
}

}  // namespace

// The tcgen05 path applies for N <= 32, Dk = Dv = 128, R = Hv / Hk in {1, 2},
// bfloat16 activations and o (the fused tree conv: bfloat16 x, conv state and
// weights), a pool with unit k stride, 16-byte multiple strides and a known
// slot count, and 16-byte aligned output rows.
bool dft_gdn_tc_applicable(const dft_gdn_args* a) {
  if (a->force_simt) return false;
  const int dt = a->conv ? a->conv->x_dtype : a->y_dtype;
  if (dt != DFT_BF16 || a->o_dtype != dt) return false;
  if (a->conv && (a->conv->cs_dtype != DFT_BF16 || a->conv->w_dtype != DFT_BF16 ||
                  !al16(a->conv->weight) || ((uintptr_t)a->conv->bias & 3)))
    return false;
  const int es = 2;
  if (a->N > kNP || a->Dk != kD || a->Dv != kD) return false;
  const int R = a->Hv / a->Hk;
  if (R != 1 && R != 2) return false;
  if (smem_bytes(R, a->conv != nullptr) > kMaxSmem) return false;
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
  const int es = 2;
  {
    // activation (pre-conv x, or y) as [B][N][C]: rows >= N of a 32-row box read as zeros
    const void* act = a->conv ? a->conv->x : a->y;
    const int64_t sn = a->conv ? a->conv->x_sn : a->y_sn, sb = a->conv ? a->conv->x_sb : a->y_sb;
    const int64_t C = 2 * (int64_t)a->Hk * a->Dk + (int64_t)a->Hv * a->Dv;
    const cuuint64_t dims[3] = {(cuuint64_t)C, (cuuint64_t)a->N, (cuuint64_t)a->B};
    const cuuint64_t strides[2] = {(cuuint64_t)(sn * es), (cuuint64_t)(sb * es)};
    const cuuint32_t box[3] = {128, (cuuint32_t)kNP, 1};
    const cuuint32_t estr[3] = {1, 1, 1};
    if (encode_fn()(&act_map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3,
                    const_cast<void*>(act), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return DFT_ERR_UNSUPPORTED;
  }
  TcArgs ta;
  ta.g = *a;
  if (a->conv) ta.cv = *a->conv;
  else memset(&ta.cv, 0, sizeof(ta.cv));
  const int R = a->Hv / a->Hk;
  const bool conv = a->conv != nullptr;
  const uint32_t smem = smem_bytes(R, conv);
  const int units = a->B * a->Hk;
  const int grid = units < sm_count() ? units : sm_count();
  auto go = [&](auto kernel) -> int {
    if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem) != cudaSuccess)
      return DFT_ERR_CUDA;
    // overlap_prev: programmatic dependent launch (the kernel's own
    // griddepcontrol.wait orders its activation reads and its writes)
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
  int rc;
  if (conv) rc = R == 2 ? go(gdn_verify_tc<2, true>) : go(gdn_verify_tc<1, true>);
  else rc = R == 2 ? go(gdn_verify_tc<2, false>) : go(gdn_verify_tc<1, false>);
  if (rc) return rc;
  DFT_LAUNCH_CHECK();
  return DFT_OK;
}
