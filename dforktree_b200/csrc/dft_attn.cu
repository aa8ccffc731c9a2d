// Tree-masked attention verify for the gated full-attention layers (sm_100a).
//
// Reference: the plugin verifies a 32-node draft tree through SGLang's
// flashinfer prefill wrapper with a custom mask (fc1_branch64.py:39 builds
// mask = [ones(n, prefix) | anc], fc1_plan.py:16-33 plans one request with
// page size 1 and the host-known KV length).  Per request and q-head:
//   o[n] = softmax_j( q[n] . k[j] * sm_scale  |  j < prefix or anc[n][j - prefix] ) . v[j]
// with grouped-query heads (q-head hq reads kv-head hq / G).
//
// Here: one CTA per work unit (request b, kv-head h, key split s).  The G
// q-heads of kv-head h and the N tree nodes form one 128-row query tile
// (row = node * G + head), so one tcgen05 MMA of M = 128 serves the whole
// group.  Both A operands live in tensor memory, so shared memory holds only
// the K / V stream:
//   Q   loaded once per unit by the softmax threads (one row each) and stored
//       to TMEM as packed bf16
//   K,V 64-key tiles gathered through the page table (page size 1) with
//       16-byte cp.async into the 128B-swizzled layout: three stages, four
//       producer warps, the next tile's slot indices fetched a tile ahead
//       (paged rows rule out tiled TMA)
//   S   = Q K^T    tcgen05 kind::f16, A from TMEM, M=128 N=64 K=256, fp32 in TMEM
//   P   = exp2(S * scale*log2e - m) with the tree mask, one thread per row
//       (TMEM lane); the running max moves (and O is rescaled in TMEM) only
//       when it grows by more than 8; P written back as bf16 over its own S
//   O  += P V      tcgen05 kind::f16, A = P from TMEM, V as an MN-major smem
//       operand, M=128 N=256 K=64
// S / P are double-buffered in TMEM (O 256 columns, Q 128, S/P 2 x 64), so
// the S MMA of tile t+1 runs while the softmax of tile t does.  Splits write
// (O, m, l) partials that a second kernel merges; a single split writes o
// directly.  Every wait is bounded (~1 s); on timeout the CTA raises
// DFT_DEV_TIMEOUT, drains its copies and MMAs (bounded), frees TMEM and exits.
#include "dft_common.cuh"
#include "dft_tc.cuh"

#include <cstring>

using namespace dft;
using namespace dft::tc;

namespace {

constexpr int kD = 256;        // head dim (tensor-core path)
constexpr int kRows = 128;     // query rows per unit (nodes x group)
constexpr int kKeys = 64;      // keys per tile
constexpr int kStages = 3;     // K/V tiles in shared memory
constexpr int kThreads = 416;  // warps 0-7 softmax / epilogue, 8 control + MMA, 9-12 KV producers
constexpr int kSoftmax = 256;  // two threads per query row (columns split in halves)
constexpr int kCtlWarp = 8, kProdWarp0 = 9;
constexpr int kProducers = 128;
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t COL_O = 0, COL_Q = 256, COL_S = 384;  // S/P buffer b at COL_S + 64 b

constexpr uint32_t kKVChunk = kKeys * 128;  // 8 KB: 64 keys x 64 dims
constexpr uint32_t kKVTile = 4 * kKVChunk;  // 32 KB
constexpr uint32_t kStageBytes = 2 * kKVTile;  // K then V
constexpr uint32_t OFF_SMALL = kStages * kStageBytes;
constexpr uint32_t kSmallBytes = 4096;
constexpr uint32_t kSmem = OFF_SMALL + kSmallBytes + 1024;  // + alignment slack

struct Small {
  uint64_t q_ready;
  uint64_t kv_full[kStages], kv_empty[kStages];
  uint64_t s_full[2], p_full[2];
  uint64_t o_done, o_full, o_free, mma_done;
  uint32_t tmem_base;
  int abort;
  float xmax[2][2][kRows];  // [tile parity][half][row] tile max exchange between a row's two threads
  float lsum[2][kRows];     // [half][row] final row sums
  int okx[2][2][4];         // [tile parity][half][row warp] wait outcomes, shared by a row's two warps
  int okr[2][2][4];         // the same for the rescale's wait
  int oke[2][4];            // [half][row warp] the epilogue's wait
};
static_assert(sizeof(Small) <= kSmallBytes, "small region");

struct AttnParams {
  dft_tree_attn_args a;
  int G;          // q-heads per kv-head
  int splits;     // key splits per (request, kv-head)
  int tps;        // tiles per split
  float* ws_o;    // [units][128][256] partial O (splits > 1)
  float* ws_ml;   // [units][128][2]   partial (m, l)
};

__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
__device__ __forceinline__ uint32_t pack_bf16(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

__device__ __forceinline__ void set_abort(Small& sm, int32_t* status) {
  *reinterpret_cast<volatile int*>(&sm.abort) = 1;
  raise_status(status, DFT_DEV_TIMEOUT);
}

// Work unit u = (request b, kv-head h, key split s) and its key tiles.
struct Unit {
  int b, h, s, len, plen, t0, T;
  int64_t kv_start;
  bool bad;
};
__device__ __forceinline__ Unit unit_info(const AttnParams& P, int u) {
  const dft_tree_attn_args& a = P.a;
  Unit U;
  U.s = u % P.splits;
  U.h = (u / P.splits) % a.Hkv;
  U.b = u / (P.splits * a.Hkv);
  // keys of request b: kv_indices[start, start + len); the last N are the tree nodes
  U.kv_start = a.kv_indptr[U.b];
  U.len = (int)(a.kv_indptr[U.b + 1] - U.kv_start);
  U.bad = U.len < a.N || U.len > a.max_kv_len;
  if (U.bad) U.len = 0;
  U.plen = U.len - a.N;
  const int n_tiles = (U.len + kKeys - 1) / kKeys;
  U.t0 = U.s * P.tps;
  const int t1 = min(U.t0 + P.tps, n_tiles);
  U.T = t1 > U.t0 ? t1 - U.t0 : 0;
  return U;
}

// Persistent: CTA c takes units c, c + grid, ...  Tile, buffer and barrier
// phases run on per-CTA counters across units (g: key tiles, ui: units with
// keys), so the next unit's loads, Q and S MMAs start while this unit's last
// P V and epilogue finish.
__global__ void __launch_bounds__(kThreads, 1)
    tree_attn_kernel(const __grid_constant__ AttnParams P, int units, int32_t* status) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  unsigned char* smem = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  Small& sm = *reinterpret_cast<Small*>(smem + OFF_SMALL);
  const volatile int* abort_flag = &sm.abort;
  const dft_tree_attn_args& a = P.a;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const uint32_t sbase = smem_u32(smem);

  if (warp == kCtlWarp) {
    if (lane == 0) {
      mbar_init(smem_u32(&sm.q_ready), kSoftmax);
      for (int i = 0; i < kStages; ++i) {
        mbar_init(smem_u32(&sm.kv_full[i]), kProducers);
        mbar_init(smem_u32(&sm.kv_empty[i]), 1);
      }
      for (int i = 0; i < 2; ++i) {
        mbar_init(smem_u32(&sm.s_full[i]), 1);
        mbar_init(smem_u32(&sm.p_full[i]), kSoftmax);
      }
      mbar_init(smem_u32(&sm.o_done), 1);
      mbar_init(smem_u32(&sm.o_full), 1);
      mbar_init(smem_u32(&sm.o_free), kSoftmax);
      mbar_init(smem_u32(&sm.mma_done), 1);
      sm.abort = 0;
      asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    }
    __syncwarp();
    tmem_alloc(smem_u32(&sm.tmem_base), kTmemCols);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = sm.tmem_base;

  if (warp == kCtlWarp) {
    // ------------------------------------------------------ control: MMAs
    if (lane == 0) {
      const uint32_t id_s = idesc_bf16(128, kKeys, false), id_o = idesc_bf16(128, kD, true);
      int g = 0, ui = 0;
      bool ok = true;
      for (int unit = blockIdx.x; ok && unit < units; unit += gridDim.x) {
        const Unit U = unit_info(P, unit);
        if (U.bad) raise_status(status, DFT_DEV_BAD_INDEX);
        if (U.T == 0) continue;
        ok = mbar_wait_or_abort(smem_u32(&sm.q_ready), ui & 1, abort_flag);
        for (int t = 0; ok && t <= U.T; ++t) {
          if (t < U.T) {
            const int gt = g + t, st = gt % kStages, sb = gt & 1;
            ok = mbar_wait_or_abort(smem_u32(&sm.kv_full[st]), (gt / kStages) & 1, abort_flag);
            // S/P buffer sb is free once P V of tile gt-2 has retired.  For a
            // unit's first tile that wait happened before the previous unit's
            // last P V was issued: o_done's parity tells phases apart only
            // while P V gt-1 is not yet issued.
            if (ok && t >= 1 && gt >= 2) ok = mbar_wait_or_abort(smem_u32(&sm.o_done), (gt - 2) & 1, abort_flag);
            if (!ok) break;
            tc_fence_after();
            fence_async_smem();  // cp.async (generic proxy) writes -> tensor-core reads
            const uint32_t kb = sbase + st * kStageBytes;
#pragma unroll
            for (int k = 0; k < 16; ++k) {
              const uint64_t bd = sw128_desc(kb + (k >> 2) * kKVChunk + (k & 3) * 32);
              mma_bf16_ts(tmem + COL_S + 64 * sb, tmem + COL_Q + 8 * k, bd, id_s, k > 0);
            }
            mma_commit(smem_u32(&sm.s_full[sb]));
          }
          if (t >= 1) {
            const int gu = g + t - 1, pb = gu & 1;
            ok = mbar_wait_or_abort(smem_u32(&sm.p_full[pb]), (gu >> 1) & 1, abort_flag);
            // the first P V of a unit overwrites O: the previous unit's epilogue has read it
            if (ok && t == 1 && ui > 0) ok = mbar_wait_or_abort(smem_u32(&sm.o_free), (ui - 1) & 1, abort_flag);
            // before a unit's last P V, P V gu-1 has retired (frees the next unit's first S/P buffer)
            if (ok && t == U.T && gu >= 1) ok = mbar_wait_or_abort(smem_u32(&sm.o_done), (gu - 1) & 1, abort_flag);
            if (!ok) break;
            tc_fence_after();
            const uint32_t vb = sbase + (gu % kStages) * kStageBytes + kKVTile;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              // V [keys x dims] is MN-major: 64-dim chunks 8 KB apart, 8-key groups 1 KB apart
              const uint64_t bd = sw128_desc(vb + k * 16 * 128, kKVChunk, 1024);
              mma_bf16_ts(tmem + COL_O, tmem + COL_S + 64 * pb + 8 * k, bd, id_o, (t > 1 || k > 0) ? 1u : 0u);
            }
            mma_commit(smem_u32(&sm.kv_empty[gu % kStages]));
            mma_commit(smem_u32(&sm.o_done));
            if (t == U.T) mma_commit(smem_u32(&sm.o_full));
          }
        }
        g += U.T;
        ++ui;
      }
      if (!ok && !*abort_flag) set_abort(sm, status);
      // every MMA issued above has retired before TMEM is freed
      mma_commit(smem_u32(&sm.mma_done));
      if (!mbar_wait(smem_u32(&sm.mma_done), 0)) raise_status(status, DFT_DEV_TIMEOUT);
    }
    __syncwarp();
  } else if (warp >= kProdWarp0) {
    // ------------------------------------------- producers: paged K/V gather
    const int pw = warp - kProdWarp0;
    const uint64_t pol = l2_evict_first();
    const unsigned char* kc = static_cast<const unsigned char*>(a.k_cache);
    const unsigned char* vc = static_cast<const unsigned char*>(a.v_cache);
    const uint32_t dst_lane = (uint32_t)(lane >> 3) * kKVChunk;
    int g = 0;
    bool ok = true;
    for (int unit = blockIdx.x; ok && unit < units; unit += gridDim.x) {
      const Unit U = unit_info(P, unit);
      if (U.T == 0) continue;
      const int64_t head_off = (int64_t)U.h * a.kv_sh * 2 + (int64_t)lane * 16;
      // lane i < 16 holds the slot of key 4 i + pw of a tile (-1 past the end)
      auto fetch_slots = [&](int tile) -> int {
        const int j = tile * kKeys + 4 * lane + pw;
        return (lane < kKeys / 4 && j < U.len) ? a.kv_indices[U.kv_start + j] : -1;
      };
      int cur = fetch_slots(U.t0);
      for (int t = 0; t < U.T; ++t) {
        const int gt = g + t, st = gt % kStages;
        const int nxt = t + 1 < U.T ? fetch_slots(U.t0 + t + 1) : -1;  // in flight during this tile
        if (gt >= kStages) {
          ok = mbar_wait_or_abort(smem_u32(&sm.kv_empty[st]), (gt / kStages - 1) & 1, abort_flag);
          if (!ok) break;
        }
        const int j0 = (U.t0 + t) * kKeys;
        if (lane < kKeys / 4 && j0 + 4 * lane + pw < U.len && (cur < 0 || (int64_t)cur >= a.n_slots))
          raise_status(status, DFT_DEV_BAD_INDEX);
        const uint32_t kb = sbase + st * kStageBytes, vb = kb + kKVTile;
#pragma unroll
        for (int kk = 0; kk < kKeys / 4; ++kk) {
          const int r = kk * 4 + pw;
          const int slot = __shfl_sync(0xffffffffu, cur, kk);
          const bool valid = j0 + r < U.len && slot >= 0 && (int64_t)slot < a.n_slots;
          const int64_t off = (int64_t)(valid ? slot : 0) * a.kv_st * 2 + head_off;
          const uint32_t dst = dst_lane + (uint32_t)r * 128 + ((((uint32_t)lane & 7) ^ ((uint32_t)r & 7)) << 4);
          cp_async16(kb + dst, valid ? kc + off : kc, valid ? 16u : 0u, pol);
          cp_async16(vb + dst, valid ? vc + off : vc, valid ? 16u : 0u, pol);
        }
        cp_async_arrive_noinc(smem_u32(&sm.kv_full[st]));
        cur = nxt;
      }
      g += U.T;
    }
    cp_async_wait_all();
    if (!ok && !*abort_flag) set_abort(sm, status);
  } else {
    // ---------------------- softmax / epilogue: two threads per row, one half each
    const int r = (warp & 3) * 32 + lane;  // TMEM lane (query row)
    const int hf = warp >> 2;              // S columns [32 hf, 32 hf + 32), O / Q columns by halves
    const int pair_bar = 1 + (warp & 3);   // named barrier of warps w and w + 4 (same rows)
    const int wq = warp & 3;
    const int n = r / P.G, g_ = r % P.G;
    const bool row_ok = n < a.N;
    const uint32_t lane_base = (uint32_t)((warp & 3) * 32) << 16;
    const float sc = a.sm_scale * 1.4426950408889634f;
    // Q row half of unit U -> TMEM (packed bf16, 64 columns; rows past the tree
    // are zero), then the unit's ancestor row of node n as a bit mask
    auto load_q = [&](const Unit& U, uint64_t& mask) {
      const uint4* qrow = reinterpret_cast<const uint4*>(
          static_cast<const unsigned char*>(a.q) +
          ((int64_t)U.b * a.q_sb + (int64_t)(row_ok ? n : 0) * a.q_sn + (int64_t)(U.h * P.G + g_) * a.q_sh) * 2 +
          hf * 256);
      const float* arow = a.anc + (int64_t)U.b * a.anc_sb + (int64_t)(row_ok ? n : 0) * a.N;
      float av[64];
#pragma unroll
      for (int m = 0; m < 64; ++m) av[m] = (row_ok && m < a.N) ? __ldg(arow + m) : 0.f;
#pragma unroll 1
      for (int c = 0; c < 2; ++c) {
        float v[32];
#pragma unroll
        for (int q = 0; q < 8; ++q) {
          const uint4 w = row_ok ? __ldg(qrow + 8 * c + q) : make_uint4(0u, 0u, 0u, 0u);
          v[4 * q] = __uint_as_float(w.x);
          v[4 * q + 1] = __uint_as_float(w.y);
          v[4 * q + 2] = __uint_as_float(w.z);
          v[4 * q + 3] = __uint_as_float(w.w);
        }
        tmem_st32(tmem + lane_base + COL_Q + 64 * hf + 32 * c, v);
      }
      tc_fence_before();
      mbar_arrive(smem_u32(&sm.q_ready));
      mask = 0;
#pragma unroll
      for (int m = 0; m < 64; ++m) mask |= (uint64_t)(av[m] > 0.5f) << m;
    };
    // the first unit with keys, and from then on always the next one
    auto next_live = [&](int from) {
      for (int u = from; u < units; u += gridDim.x)
        if (unit_info(P, u).T > 0) return u;
      return units;
    };
    uint64_t mask_next = 0;
    int qu = next_live(blockIdx.x);  // the unit whose Q is in TMEM
    if (qu < units) load_q(unit_info(P, qu), mask_next);
    int g = 0, ui = 0;
    bool ok = true;
    for (int unit = blockIdx.x; ok && unit < units; unit += gridDim.x) {
      const Unit U = unit_info(P, unit);
      if (U.T == 0) {
        if (P.splits > 1) {
          const int64_t prow = (int64_t)unit * kRows + r;
          float4* dst = reinterpret_cast<float4*>(P.ws_o + prow * kD + 128 * hf);
#pragma unroll 4
          for (int q = 0; q < 32; ++q) dst[q] = make_float4(0.f, 0.f, 0.f, 0.f);
          if (hf == 0) {
            P.ws_ml[2 * prow] = -INFINITY;
            P.ws_ml[2 * prow + 1] = 0.f;
          }
        }
        continue;
      }
      const uint64_t mask = mask_next;  // bit m: tree node m is n or an ancestor of n
      // A row's two warps meet at the same named barriers in the same order;
      // every early exit is decided from outcomes both have exchanged there.
      float m_used = -INFINITY, l = 0.f;
      for (int t = 0; t < U.T; ++t) {
        const int gt = g + t, sb = gt & 1;
        const bool got =
            __all_sync(0xffffffffu, mbar_wait_or_abort(smem_u32(&sm.s_full[sb]), (gt >> 1) & 1, abort_flag));
        float x[32];
        if (got) {
          tc_fence_after();
          tmem_ld32(tmem + lane_base + COL_S + 64 * sb + 32 * hf, x);
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) x[i] = 0.f;
        }
        const int j0 = (U.t0 + t) * kKeys + 32 * hf;
        // keys of a tile inside the prefix need no mask: x stays raw, P = 2^(x sc - m)
        const bool plain = (U.t0 + t + 1) * kKeys <= U.plen;  // block-uniform
        float tmax = -INFINITY;
        if (plain) {
#pragma unroll
          for (int i = 0; i < 32; ++i) tmax = fmaxf(tmax, x[i]);
          tmax *= sc;
        } else {
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            const int j = j0 + i;
            float y = x[i] * sc;
            if (j >= U.len) y = -INFINITY;
            else if (j >= U.plen && !((mask >> (j - U.plen)) & 1ull)) y = -INFINITY;
            x[i] = y;
            tmax = fmaxf(tmax, y);
          }
        }
        sm.xmax[sb][hf][r] = tmax;
        if (lane == 0) sm.okx[sb][hf][wq] = got;
        // the barrier also orders this half's S reads before the other half's P
        // stores (half 1 writes P over S columns 16..31, which half 0 reads)
        tc_fence_before();
        named_bar(pair_bar, 64);
        tc_fence_after();
        tmax = fmaxf(tmax, sm.xmax[sb][hf ^ 1][r]);
        ok = got && sm.okx[sb][hf ^ 1][wq];
        if (!ok) break;
        // a row moves its reference max only when the tile max exceeds it by
        // more than 8 (P <= 2^8 otherwise); O then scales by 2^(old - new)
        const bool grow = tmax > m_used + 8.f;
        if (__any_sync(0xffffffffu, grow)) {
          const float m_new = grow ? tmax : m_used;
          if (t > 0) {
            // O holds P V of this unit's earlier tiles: wait for the last, then rescale this half row
            const bool done = __all_sync(0xffffffffu,
                                         mbar_wait_or_abort(smem_u32(&sm.o_done), (gt - 1) & 1, abort_flag));
            if (lane == 0) sm.okr[sb][hf][wq] = done;
            named_bar(pair_bar, 64);
            ok = done && sm.okr[sb][hf ^ 1][wq];
            if (!ok) break;
            tc_fence_after();
            const float alpha = grow ? ex2(m_used - m_new) : 1.f;
#pragma unroll 1
            for (int c = 0; c < 4; ++c) {
              float v[32];
              tmem_ld32(tmem + lane_base + COL_O + 128 * hf + 32 * c, v);
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] *= alpha;
              tmem_st32(tmem + lane_base + COL_O + 128 * hf + 32 * c, v);
            }
            l *= alpha;
          }
          m_used = m_new;
        }
        uint32_t pk[16];
        f32x2 sum2 = pk2(0.f, 0.f);
        if (plain) {
          const f32x2 sc2 = pk2(sc, sc), nm2 = pk2(-m_used, -m_used);
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            float e0, e1;
            upk2(fma2(pk2(x[2 * i], x[2 * i + 1]), sc2, nm2), e0, e1);
            const f32x2 p2 = pk2(ex2(e0), ex2(e1));
            sum2 = add2(sum2, p2);
            pk[i] = f32x2_to_bf16x2(p2);
          }
        } else {
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const float p0 = x[2 * i] == -INFINITY ? 0.f : ex2(x[2 * i] - m_used);
            const float p1 = x[2 * i + 1] == -INFINITY ? 0.f : ex2(x[2 * i + 1] - m_used);
            const f32x2 p2 = pk2(p0, p1);
            sum2 = add2(sum2, p2);
            pk[i] = f32x2_to_bf16x2(p2);
          }
        }
        float s0, s1;
        upk2(sum2, s0, s1);
        l += s0 + s1;
        // P (bf16 pairs) over columns [16 hf, 16 hf + 16) of its own S buffer
        tmem_st16(tmem + lane_base + COL_S + 64 * sb + 16 * hf, pk);
        tc_fence_before();
        mbar_arrive(smem_u32(&sm.p_full[sb]));
      }
      if (!ok) break;
      g += U.T;
      // every S MMA of this unit has been consumed: the next unit's Q may go in
      qu = next_live(unit + gridDim.x);
      if (qu < units) load_q(unit_info(P, qu), mask_next);
      // ---- epilogue: wait for this unit's last P V, then O (or its partial) out
      const bool got = __all_sync(0xffffffffu, mbar_wait_or_abort(smem_u32(&sm.o_full), ui & 1, abort_flag));
      tc_fence_after();
      sm.lsum[hf][r] = l;
      if (lane == 0) sm.oke[hf][wq] = got;
      named_bar(pair_bar, 64);
      l = sm.lsum[0][r] + sm.lsum[1][r];
      ok = got && sm.oke[hf ^ 1][wq];
      if (ok) {
        if (P.splits == 1) {
          const float inv = l > 0.f ? 1.f / l : 0.f;
          unsigned char* orow = static_cast<unsigned char*>(a.o) +
                                ((int64_t)U.b * a.o_sb + (int64_t)n * a.o_sn + (int64_t)(U.h * P.G + g_) * a.o_sh) * 2 +
                                hf * 256;
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float v[32];
            tmem_ld32(tmem + lane_base + COL_O + 128 * hf + 32 * c, v);
            if (row_ok) {
              uint4* dst = reinterpret_cast<uint4*>(orow + c * 64);
#pragma unroll
              for (int q = 0; q < 4; ++q)
                dst[q] = make_uint4(pack_bf16(v[8 * q] * inv, v[8 * q + 1] * inv),
                                    pack_bf16(v[8 * q + 2] * inv, v[8 * q + 3] * inv),
                                    pack_bf16(v[8 * q + 4] * inv, v[8 * q + 5] * inv),
                                    pack_bf16(v[8 * q + 6] * inv, v[8 * q + 7] * inv));
            }
          }
        } else {
          const int64_t prow = (int64_t)unit * kRows + r;
          float4* dst = reinterpret_cast<float4*>(P.ws_o + prow * kD + 128 * hf);
          const bool mine = l > 0.f;
#pragma unroll 1
          for (int c = 0; c < 4; ++c) {
            float v[32];
            tmem_ld32(tmem + lane_base + COL_O + 128 * hf + 32 * c, v);
#pragma unroll
            for (int q = 0; q < 8; ++q)
              dst[8 * c + q] = mine ? make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3])
                                    : make_float4(0.f, 0.f, 0.f, 0.f);
          }
          if (hf == 0) {
            P.ws_ml[2 * prow] = mine ? m_used : -INFINITY;
            P.ws_ml[2 * prow + 1] = mine ? l : 0.f;
          }
        }
        // O may now be overwritten by the next unit's first P V
        tc_fence_before();
        mbar_arrive(smem_u32(&sm.o_free));
      }
      ++ui;
    }
    if (!ok && !*abort_flag) set_abort(sm, status);
  }
  tc_fence_before();
  __syncthreads();
  if (warp == kCtlWarp) {
    tc_fence_after();
    tmem_dealloc(tmem, kTmemCols);
  }
}

// Merge the split partials of one output row (request b, node n, q-head hq):
// o = sum_s 2^(m_s - M) O_s / sum_s 2^(m_s - M) l_s.  64 threads x 4 dims.
__global__ void __launch_bounds__(64) tree_attn_combine(const __grid_constant__ AttnParams P) {
  const dft_tree_attn_args& a = P.a;
  const int nh = blockIdx.x, b = blockIdx.y;
  const int n = nh / a.Hq, hq = nh % a.Hq;
  const int h = hq / P.G, g = hq % P.G;
  const int r = n * P.G + g;
  const int64_t u0 = ((int64_t)b * a.Hkv + h) * P.splits;
  float M = -INFINITY;
  for (int s = 0; s < P.splits; ++s) M = fmaxf(M, P.ws_ml[2 * ((u0 + s) * kRows + r)]);
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  float L = 0.f;
  for (int s = 0; s < P.splits; ++s) {
    const int64_t prow = (u0 + s) * kRows + r;
    const float ls = P.ws_ml[2 * prow + 1];
    if (!(ls > 0.f)) continue;
    const float w = ex2(P.ws_ml[2 * prow] - M);
    const float4 v = reinterpret_cast<const float4*>(P.ws_o + prow * kD)[threadIdx.x];
    acc.x += w * v.x;
    acc.y += w * v.y;
    acc.z += w * v.z;
    acc.w += w * v.w;
    L += w * ls;
  }
  const float inv = L > 0.f ? 1.f / L : 0.f;
  unsigned char* orow = static_cast<unsigned char*>(a.o) +
                        ((int64_t)b * a.o_sb + (int64_t)n * a.o_sn + (int64_t)hq * a.o_sh) * 2;
  reinterpret_cast<uint2*>(orow)[threadIdx.x] = make_uint2(pack_bf16(acc.x * inv, acc.y * inv), pack_bf16(acc.z * inv, acc.w * inv));
}

// ------------------------------------------------------------------ host --
int sm_count() {
  int dev = 0, n = 0;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n > 0 ? n : 148;
}

inline bool al16(const void* p) { return ((uintptr_t)p & 15) == 0; }

int check_args(const dft_tree_attn_args* a) {
  if (!a || !a->q || !a->k_cache || !a->v_cache || !a->kv_indptr || !a->kv_indices || !a->anc || !a->o)
    return DFT_ERR_INVALID;
  if (a->B <= 0 || a->N <= 0 || a->Hq <= 0 || a->Hkv <= 0 || a->Hq % a->Hkv || a->max_kv_len < a->N ||
      a->n_slots <= 0 || a->B > 65535)
    return DFT_ERR_INVALID;
  const int G = a->Hq / a->Hkv;
  if (a->D != kD || (G != 1 && G != 2 && G != 4 && G != 8) || a->N * G > kRows || a->N > 64)
    return DFT_ERR_UNSUPPORTED;
  if (!al16(a->q) || !al16(a->k_cache) || !al16(a->v_cache) || !al16(a->o)) return DFT_ERR_UNSUPPORTED;
  if ((a->q_sh * 2) % 16 || (a->q_sn * 2) % 16 || (a->q_sb * 2) % 16 || (a->kv_st * 2) % 16 ||
      (a->kv_sh * 2) % 16 || (a->o_sh * 2) % 16 || (a->o_sn * 2) % 16 || (a->o_sb * 2) % 16)
    return DFT_ERR_UNSUPPORTED;
  if (a->q_sh < kD || a->q_sn <= 0 || a->q_sb <= 0) return DFT_ERR_UNSUPPORTED;
  return DFT_OK;
}

// Key splits per (request, kv-head).  A unit costs its key tiles plus a fixed
// part (Q load, first tiles' latency, O readout: about 8 tiles' time), and
// splits > 1 add the partials' merge (about 12 tiles' time); the persistent
// CTAs take ceil(units / SMs) units each.  The split count minimising
//   ceil(pairs * sp / SMs) * (ceil(tiles / sp) + 8) + (sp > 1 ? 12 : 0)
// is taken (ties: fewer splits).  Measured at batch 64 with 4K prefixes
// (256 pairs, 65 tiles): 1 split 0.222 ms per layer, 2: 0.276, 3: 0.298,
// 4: 0.293 (the earlier rule, fill the last wave to >= 90 %, chose 4).  A few
// requests with long prefixes still split (4 pairs, 65 tiles: 8 splits).
void plan(const dft_tree_attn_args* a, int* splits, int* tps) {
  const int64_t tiles = (a->max_kv_len + kKeys - 1) / kKeys;
  const int64_t pairs = (int64_t)a->B * a->Hkv;
  const int64_t sms = sm_count();
  constexpr int64_t kUnitFixed = 8, kMerge = 12;
  int best = 1;
  int64_t best_cost = -1;
  for (int sp = 1; sp <= 8 && sp <= tiles; ++sp) {
    const int64_t per = (pairs * sp + sms - 1) / sms;
    const int64_t cost = per * ((tiles + sp - 1) / sp + kUnitFixed) + (sp > 1 ? kMerge : 0);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best = sp;
    }
  }
  *splits = best;
  *tps = (int)((tiles + best - 1) / best);
}

}  // namespace

extern "C" int64_t dft_tree_attn_workspace_bytes(const dft_tree_attn_args* a) {
  if (check_args(a)) return -1;
  int splits, tps;
  plan(a, &splits, &tps);
  if (splits == 1) return 0;
  const int64_t units = (int64_t)a->B * a->Hkv * splits;
  return units * kRows * (kD + 2) * (int64_t)sizeof(float);
}

extern "C" int dft_tree_attn(const dft_tree_attn_args* a, void* workspace, int32_t* dev_status, void* stream) {
  const int rc = check_args(a);
  if (rc) return rc;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  AttnParams P;
  memset(&P, 0, sizeof(P));
  P.a = *a;
  P.G = a->Hq / a->Hkv;
  plan(a, &P.splits, &P.tps);
  const int64_t units = (int64_t)a->B * a->Hkv * P.splits;
  if (P.splits > 1) {
    if (!workspace || !al16(workspace)) return DFT_ERR_INVALID;
    P.ws_o = static_cast<float*>(workspace);
    P.ws_ml = P.ws_o + units * kRows * kD;
  }
  if (units > 0x7FFFFFFF) return DFT_ERR_UNSUPPORTED;
  if (cudaFuncSetAttribute(tree_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kSmem) != cudaSuccess)
    return DFT_ERR_CUDA;
  const int64_t grid = units < sm_count() ? units : sm_count();
  tree_attn_kernel<<<(unsigned)grid, kThreads, kSmem, st>>>(P, (int)units, dev_status);
  DFT_LAUNCH_CHECK();
  if (P.splits > 1) {
    dim3 grid((unsigned)(a->N * a->Hq), (unsigned)a->B);
    tree_attn_combine<<<grid, 64, 0, st>>>(P);
    DFT_LAUNCH_CHECK();
  }
  return DFT_OK;
}
