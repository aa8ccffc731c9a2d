// Fork-aware beam tree search and tree structure (tree_ops.py:7-89, fc1_builder.py:30-47).
//
// Reference: tree_ops.beam_tree (tree_ops.py:7-53) runs ~20 torch ops per
// step plus a global top-(N-1); tree_ops.tree_struct (tree_ops.py:68-89)
// uses 9 N x N matmuls; Builder.run (fc1_builder.py:38-47) adds tokens /
// nxt / sib.  Here one CTA per request does all of it in shared memory:
//   per step: P = pow2 >= W*M threads score the W x M children (fork-aware
//   PMI closure, half-warp logsumexp and argmax per beam row), bitonic-sort
//   the P keys (descending, ties by flat index) and keep the top W beams;
//   then a warp merges the S sorted per-step key rows into the global
//   top-(N-1) (two warp max-reductions per node over a 64-bit order key
//   instead of a five-round shuffle argmax: score + build 0.457 -> 0.451 ms
//   at batch 64), orders nodes by (step, rank), remaps parents and derives the
//   ancestor masks, depth, conv columns, first child and next sibling.
// Float ops that torch rounds separately are kept separate (__fadd_rn /
// __fmul_rn: no FMA contraction), so trees match the reference except for
// exact or last-ulp score ties.
#include "dft_common.cuh"

using namespace dft;

namespace {

constexpr int kM = 16;
constexpr int kMaxS = 64;

__device__ __forceinline__ bool before(float ka, int ia, float kb, int ib) {
  return ka > kb || (ka == kb && ia < ib);
}

// Order-preserving bits of a key: a > b as floats iff order_bits(a) >
// order_bits(b) as unsigned (-0 is first made +0, so that equal keys give
// equal bits; keys are never NaN).  -inf maps to 0x007fffff, above the 0
// that marks "no key".
__device__ __forceinline__ uint32_t order_bits(float k) {
  const uint32_t u = __float_as_uint(k + 0.0f);
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// torch.logsumexp over the 16 lanes of a half-warp plus one extra value.
__device__ __forceinline__ float half_lse(float x, float extra) {
  float m = x;
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o, 16));
  m = fmaxf(m, extra);
  if (isinf(m)) m = 0.f;  // logsumexp masks an infinite max to 0
  float e = expf(__fsub_rn(x, m));
#pragma unroll
  for (int o = 8; o > 0; o >>= 1) e = __fadd_rn(e, __shfl_xor_sync(0xffffffffu, e, o, 16));
  e = __fadd_rn(e, expf(__fsub_rn(extra, m)));
  return __fadd_rn(logf(e), m);
}

struct SmemLayout {
  size_t lp, rest, sc, key, lv, cand, pc, ppc, al, fl, csc, clv, cfl, sk, si, K, Pb, Cb, Fb, inv, total;
};

__host__ __device__ inline size_t align16(size_t x) { return (x + 15) & ~(size_t)15; }

__host__ __device__ inline SmemLayout smem_layout(int S, int W, int P) {
  SmemLayout L;
  size_t o = 0;
  L.lp = o; o = align16(o + sizeof(float) * S * kM);
  L.rest = o; o = align16(o + sizeof(float) * S);
  L.sc = o; o = align16(o + sizeof(float) * W);
  L.key = o; o = align16(o + sizeof(float) * W);
  L.lv = o; o = align16(o + sizeof(int) * W);
  L.cand = o; o = align16(o + sizeof(int) * W);
  L.pc = o; o = align16(o + sizeof(int) * W);
  L.ppc = o; o = align16(o + sizeof(int) * W);
  L.al = o; o = align16(o + sizeof(int) * W);
  L.fl = o; o = align16(o + sizeof(int) * W);
  L.csc = o; o = align16(o + sizeof(float) * P);
  L.clv = o; o = align16(o + sizeof(int) * P);
  L.cfl = o; o = align16(o + sizeof(int) * P);
  L.sk = o; o = align16(o + sizeof(float) * P);
  L.si = o; o = align16(o + sizeof(int) * P);
  L.K = o; o = align16(o + sizeof(float) * S * W);
  L.Pb = o; o = align16(o + S * W);
  L.Cb = o; o = align16(o + S * W);
  L.Fb = o; o = align16(o + S * W);
  L.inv = o; o = align16(o + S * W);
  L.total = o;
  return L;
}

struct BeamArgs {
  int B, S, N, W, lmax, chain_first, use_ngram, order;
  float lam_a, lam_p;
  const float* lp;
  const int32_t* ids;
  const float* rest;
  const float* T;
  const float* logc;
  const float* c0;
  const int64_t* root;
  dft_tree_out out;
  int32_t* status;
};

template <int P>
__global__ void __launch_bounds__(P) beam_kernel(BeamArgs a) {
  extern __shared__ __align__(16) unsigned char smem[];
  pdl_wait();   // lp / ids / rest / T come from the preceding kernels
  const int b = blockIdx.x;
  const int tid = threadIdx.x, lane = tid & 31;
  const int S = a.S, N = a.N, W = a.W;
  const SmemLayout Ly = smem_layout(S, W, P);
  float* s_lp = (float*)(smem + Ly.lp);
  float* s_rest = (float*)(smem + Ly.rest);
  float* s_sc = (float*)(smem + Ly.sc);
  float* s_key = (float*)(smem + Ly.key);
  int* s_lv = (int*)(smem + Ly.lv);
  int* s_cand = (int*)(smem + Ly.cand);
  int* s_pc = (int*)(smem + Ly.pc);
  int* s_ppc = (int*)(smem + Ly.ppc);
  int* s_al = (int*)(smem + Ly.al);
  int* s_fl = (int*)(smem + Ly.fl);
  float* c_sc = (float*)(smem + Ly.csc);
  int* c_lv = (int*)(smem + Ly.clv);
  int* c_fl = (int*)(smem + Ly.cfl);
  float* sk = (float*)(smem + Ly.sk);
  int* si = (int*)(smem + Ly.si);
  float* K = (float*)(smem + Ly.K);
  uint8_t* Pb = smem + Ly.Pb;
  uint8_t* Cb = smem + Ly.Cb;
  uint8_t* Fb = smem + Ly.Fb;
  uint8_t* inv = smem + Ly.inv;
  __shared__ int n_ss[kMaxNodes], n_bi[kMaxNodes], n_par[kMaxNodes];
  __shared__ int sel_ss[kMaxNodes], sel_bi[kMaxNodes];
  __shared__ unsigned long long n_anc[kMaxNodes];
  __shared__ int n_depth[kMaxNodes];

  const float BIG = a.chain_first ? 10000.0f : 0.0f;
  const float* lpb = a.lp + (int64_t)b * S * kM;
  for (int i = tid; i < S * kM; i += P) s_lp[i] = lpb[i];
  for (int i = tid; i < S; i += P) s_rest[i] = a.rest[(int64_t)b * S + i];
  for (int i = tid; i < S * W; i += P) inv[i] = 0;
  __syncthreads();

  // ---- step 0 beams (tree_ops.py:14-25)
  if (tid < 32) {
    // c0 = lp[0] - logsumexp([lp[0], rest[0]]) unless given (fc1_builder.py:29)
    const int l = lane & 15;
    float c0 = a.c0 ? a.c0[(int64_t)b * kM + l] : __fsub_rn(s_lp[l], half_lse(s_lp[l], s_rest[0]));
    // argmax of c0, first occurrence
    float bv = c0;
    int bi = l;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, bv, o, 16);
      int oi = __shfl_xor_sync(0xffffffffu, bi, o, 16);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    for (int w = lane; w < W; w += 32) {
      float sc;
      int fl, lv, cand, al;
      if (w < kM) {
        sc = c0;  // w == lane < 16 here, and lane l holds c0[l]
        fl = (w == bi);
        lv = !fl;
        cand = w;
        al = (w == 0);
      } else {
        sc = -INFINITY;
        fl = 0;
        lv = a.lmax + 1;
        cand = 0;
        al = 0;
      }
      float key = (lv <= a.lmax && sc > -INFINITY) ? __fadd_rn(sc, fl ? BIG : 0.0f) : -INFINITY;
      s_sc[w] = sc;
      s_fl[w] = fl;
      s_lv[w] = lv;
      s_cand[w] = cand;
      s_al[w] = al;
      s_pc[w] = 0;
      s_ppc[w] = 0;
      s_key[w] = key;
      K[w] = key;
      Pb[w] = 255;
      Cb[w] = (uint8_t)cand;
      Fb[w] = (uint8_t)fl;
    }
  }
  __syncthreads();

  // ---- steps 1 .. S-1 (tree_ops.py:27-43)
  const int WM = W * kM;
  for (int s = 1; s < S; ++s) {
    const int w = tid >> 4, l = tid & 15;
    const bool valid = tid < WM;
    float x = 0.f, lc = -INFINITY;
    const int ww = valid ? w : 0;
    const int cand = s_cand[ww];
    if (a.use_ngram) {
      // the closure's context: cand, pc and ppc are the candidates at
      // positions s-1, s-2 and s-3 of the beam's path (tree_ops.py:28, 40)
      int64_t row = (int64_t)b * (S - 1) + (s - 1);
      if (a.order >= 4) row = row * kM + s_ppc[ww];
      if (a.order >= 3) row = row * kM + s_pc[ww];
      const float t = a.T[(row * kM + cand) * kM + l];
      const float lam = s_al[ww] ? a.lam_a : a.lam_p;
      x = __fadd_rn(s_lp[s * kM + l], __fmul_rn(lam, t));
    } else if (!a.logc) {
      x = s_lp[s * kM + l];
    }
    if (a.logc && !a.use_ngram) {
      lc = a.logc[(((int64_t)b * (S - 1) + (s - 1)) * kM + cand) * kM + l];
    } else {
      lc = __fsub_rn(x, half_lse(x, s_rest[s]));
    }
    // argmax over the beam row (first maximal index)
    float bv = lc;
    int bi = l;
#pragma unroll
    for (int o = 8; o > 0; o >>= 1) {
      float ov = __shfl_xor_sync(0xffffffffu, bv, o, 16);
      int oi = __shfl_xor_sync(0xffffffffu, bi, o, 16);
      if (ov > bv || (ov == bv && oi < bi)) {
        bv = ov;
        bi = oi;
      }
    }
    const int is_top = (l == bi);
    const float sc_c = __fadd_rn(s_sc[ww], lc);
    const int fl_c = s_fl[ww] && is_top;
    const int lv_c = s_lv[ww] + (is_top ? 0 : 1);
    const bool ok = valid && lv_c <= a.lmax && s_key[ww] > -INFINITY;
    float key = ok ? __fadd_rn(sc_c, fl_c ? BIG : 0.0f) : -INFINITY;
    int idx = tid;
    c_sc[tid] = sc_c;
    c_lv[tid] = lv_c;
    c_fl[tid] = fl_c;
    if (W <= 32) {
      // top 32 of the P keys (descending, ties by ascending flat index) without
      // a full sort: every warp sorts its 32 keys (shuffle bitonic), then
      // pairs of sorted lists merge by halves -- max(A[i], B[31 - i]) holds the
      // 32 best of A and B as a bitonic sequence, five shuffle stages sort it
      // -- over log2(P / 32) rounds with one barrier each
#pragma unroll
      for (int size = 2; size <= 32; size <<= 1) {
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
          const float ok_ = __shfl_xor_sync(0xffffffffu, key, stride);
          const int oi_ = __shfl_xor_sync(0xffffffffu, idx, stride);
          const bool lower = (lane & stride) == 0;
          const bool dir = size == 32 || (lane & size) == 0;
          const bool mine_first = before(key, idx, ok_, oi_);
          if ((lower == dir) ? !mine_first : mine_first) {
            key = ok_;
            idx = oi_;
          }
        }
      }
      const int wid = tid >> 5;
#pragma unroll 1
      for (int span = 1; span < P / 32; span <<= 1) {
        sk[tid] = key;
        si[tid] = idx;
        __syncthreads();
        if ((wid & (2 * span - 1)) == 0) {
          const int pj = ((wid + span) << 5) + (31 - lane);
          const float ok_ = sk[pj];
          const int oi_ = si[pj];
          if (!before(key, idx, ok_, oi_)) {
            key = ok_;
            idx = oi_;
          }
#pragma unroll
          for (int stride = 16; stride > 0; stride >>= 1) {
            const float ok2 = __shfl_xor_sync(0xffffffffu, key, stride);
            const int oi2 = __shfl_xor_sync(0xffffffffu, idx, stride);
            const bool lower = (lane & stride) == 0;
            const bool mine_first = before(key, idx, ok2, oi2);
            if (lower ? !mine_first : mine_first) {
              key = ok2;
              idx = oi2;
            }
          }
        }
        __syncthreads();
      }
      if (tid < 32) {
        sk[tid] = key;
        si[tid] = idx;
      }
      __syncthreads();
    } else {
      // bitonic sort, descending by key, ties by ascending flat index
#pragma unroll 1
      for (int size = 2; size <= P; size <<= 1) {
#pragma unroll 1
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
          float ok_;
          int oi_;
          if (stride >= 32) {
            sk[tid] = key;
            si[tid] = idx;
            __syncthreads();
            ok_ = sk[tid ^ stride];
            oi_ = si[tid ^ stride];
            __syncthreads();
          } else {
            ok_ = __shfl_xor_sync(0xffffffffu, key, stride);
            oi_ = __shfl_xor_sync(0xffffffffu, idx, stride);
          }
          const bool lower = (tid & stride) == 0;
          const bool dir = (tid & size) == 0;
          const bool mine_first = before(key, idx, ok_, oi_);
          if ((lower == dir) ? !mine_first : mine_first) {
            key = ok_;
            idx = oi_;
          }
        }
      }
      sk[tid] = key;
      si[tid] = idx;
      __syncthreads();
    }
    // new beams (tree_ops.py:35-43)
    float n_sc = 0.f, n_key = 0.f;
    int n_fl = 0, n_lv = 0, n_pc = 0, n_ppc = 0, n_al = 0, p_ = 0, c_ = 0;
    if (tid < W) {
      const int id = si[tid];
      n_key = sk[tid];
      p_ = id >> 4;
      c_ = id & 15;
      n_sc = c_sc[id];
      n_fl = c_fl[id];
      n_lv = c_lv[id];
      n_pc = s_cand[p_];
      n_ppc = s_pc[p_];
      n_al = s_al[p_] && (c_ == 0);
    }
    __syncthreads();
    if (tid < W) {
      s_sc[tid] = n_sc;
      s_key[tid] = n_key;
      s_fl[tid] = n_fl;
      s_lv[tid] = n_lv;
      s_pc[tid] = n_pc;
      s_ppc[tid] = n_ppc;
      s_al[tid] = n_al;
      s_cand[tid] = c_;
      K[s * W + tid] = n_key;
      Pb[s * W + tid] = (uint8_t)p_;
      Cb[s * W + tid] = (uint8_t)c_;
      Fb[s * W + tid] = (uint8_t)n_fl;
    }
    __syncthreads();
  }

  // ---- global top-(N-1) over the S sorted rows of K (tree_ops.py:44-48)
  // A warp merges the rows: lane r holds the head of rows r and r + 32; each
  // round the best head (descending key, ties by ascending flat index) is
  // found with two warp max-reductions over a 64-bit order key -- the key's
  // order-preserving bits, then the inverted flat index among the lanes
  // holding that key -- and its row advances.
  if (tid < 32) {
    int head0 = 0, head1 = 0;  // rows lane and lane + 32
    for (int r = 0; r < N - 1; ++r) {
      uint32_t hk = 0u, lo = 0u;   // 0 / 0: no head (below every key, -inf included)
      int brow = -1;
      if (lane < S && head0 < W) {
        const int f = lane * W + head0;
        hk = order_bits(K[f]);
        lo = ~(uint32_t)f;
        brow = lane;
      }
      if (lane + 32 < S && head1 < W) {
        const int f2 = (lane + 32) * W + head1;
        const uint32_t h2 = order_bits(K[f2]), l2 = ~(uint32_t)f2;
        if (brow < 0 || h2 > hk || (h2 == hk && l2 > lo)) {
          hk = h2;
          lo = l2;
          brow = lane + 32;
        }
      }
      const uint32_t mh = __reduce_max_sync(0xffffffffu, hk);
      const uint32_t ml = __reduce_max_sync(0xffffffffu, hk == mh ? lo : 0u);
      const int bflat = (int)~ml, wrow = bflat / W;
      if (lane == 0) {
        sel_ss[r] = wrow;
        sel_bi[r] = bflat - wrow * W;
      }
      if (wrow == lane) head0++;
      if (wrow == lane + 32) head1++;
    }
  }
  __syncthreads();
  // order by (step, rank) (tree_ops.py:47-48) and record inv (:49-50)
  if (tid < N - 1) {
    const int my = sel_ss[tid];
    int pos = 0;
    for (int r = 0; r < N - 1; ++r) {
      const int o = sel_ss[r];
      pos += (o < my) || (o == my && r < tid);
    }
    n_ss[pos + 1] = my;
    n_bi[pos + 1] = sel_bi[tid];
    inv[my * W + sel_bi[tid]] = (uint8_t)(pos + 1);
  }
  __syncthreads();
  // parents (tree_ops.py:51-52, fc1_builder.py:38)
  const int64_t* root = a.root;
  if (tid < N) {
    if (tid == 0) {
      n_par[0] = -1;
    } else {
      const int ss = n_ss[tid], bi = n_bi[tid];
      n_par[tid] = ss == 0 ? 0 : inv[(ss - 1) * W + Pb[ss * W + bi]];
    }
  }
  __syncthreads();
  // ancestor masks and depth (tree_ops.py:71-79)
  if (tid < N) {
    unsigned long long m = 0ull;
    int u = tid, d = -1, guard = 0;
    while (u >= 0 && guard <= N) {
      m |= 1ull << u;
      u = n_par[u];
      ++d;
      ++guard;
    }
    n_anc[tid] = m;
    n_depth[tid] = d;
  }
  __syncthreads();
  dft_tree_out& o = a.out;
  const int64_t bN = (int64_t)b * N;
  if (tid < N) {
    const int n = tid;
    const int par = n_par[n];
    const int d = n_depth[n];
    if (o.parent) o.parent[bN + n] = par;
    if (o.depth) o.depth[bN + n] = d;
    if (o.tokens) {
      int64_t tok;
      if (n == 0) {
        tok = root[b];
      } else {
        const int ss = n_ss[n], c = Cb[ss * W + n_bi[n]];
        tok = a.ids[((int64_t)b * S + ss) * kM + c];
      }
      o.tokens[bN + n] = tok;
    }
    if (n > 0) {
      const int ss = n_ss[n], bi = n_bi[n];
      const int64_t j = (int64_t)b * (N - 1) + (n - 1);
      if (o.ss) o.ss[j] = ss;
      if (o.cand) o.cand[j] = Cb[ss * W + bi];
      if (o.flags) o.flags[j] = Fb[ss * W + bi];
    }
    // conv columns: r-th ancestor a_r -> 3 + a_r, else state column 3 - (r - depth)
    if (o.cidx) {
      int u = n;
      for (int r = 0; r < 4; ++r) {
        int col = r <= d ? 3 + u : 3 - (r - d);
        o.cidx[(bN + n) * 4 + (3 - r)] = col;
        if (r <= d) u = n_par[u] >= 0 ? n_par[u] : u;
      }
    }
    // first child and next sibling (fc1_builder.py:41-47)
    int nx = -1, sb = -1;
    for (int v = 1; v < N; ++v) {
      if (nx < 0 && n_par[v] == n) nx = v;
      if (sb < 0 && v > n && n_par[v] == par) sb = v;
    }
    if (o.nxt) o.nxt[bN + n] = nx;
    if (o.sib) o.sib[bN + n] = sb;
  }
  if (o.anc) {
    for (int e = tid; e < N * N; e += P) {
      const int i = e / N, j = e % N;
      o.anc[(int64_t)b * N * N + e] = (n_anc[i] >> j) & 1ull ? 1.0f : 0.0f;
    }
  }
  if (o.keys) {
    for (int e = tid; e < S * W; e += P) o.keys[(int64_t)b * S * W + e] = K[e];
  }
}

template <int P>
int launch_beam(const BeamArgs& a, cudaStream_t st) {
  const size_t sm = smem_layout(a.S, a.W, P).total;
  if (sm > 48 * 1024) {
    if (cudaFuncSetAttribute(beam_kernel<P>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm) != cudaSuccess)
      return DFT_ERR_CUDA;
  }
  // programmatic launch: set up while the PMI (or score) kernel drains
  return launch_pdl(beam_kernel<P>, dim3(a.B), dim3(P), sm, st, a);
}

}  // namespace

int dft_beam_launch(const dft_build_params* p, const float* lp, const int32_t* ids, const float* rest, const float* T,
                    const float* logc, const float* c0, const int64_t* root, const dft_tree_out* out,
                    int32_t* dev_status, cudaStream_t st) {
  BeamArgs a;
  a.B = p->B;
  a.S = p->S;
  a.N = p->N;
  a.W = p->N - 1 > kM ? p->N - 1 : kM;
  a.lmax = p->lmax;
  a.chain_first = p->chain_first;
  a.use_ngram = p->use_ngram;
  a.order = dft::pmi_order_of(p);
  a.lam_a = p->lam_a;
  a.lam_p = p->lam_p;
  a.lp = lp;
  a.ids = ids;
  a.rest = rest;
  a.T = T;
  a.logc = logc;
  a.c0 = c0;
  a.root = root;
  a.out = *out;
  a.status = dev_status;
  const int WM = a.W * kM;
  if (WM <= 256) return launch_beam<256>(a, st);
  if (WM <= 512) return launch_beam<512>(a, st);
  return launch_beam<1024>(a, st);
}

int dft_check_build_params(const dft_build_params* p) {
  if (!p) return DFT_ERR_INVALID;
  if (p->M != kM) return DFT_ERR_UNSUPPORTED;
  if (p->N < 2 || p->N > kMaxNodes) return DFT_ERR_UNSUPPORTED;
  if (p->S < 1 || p->S > kMaxS) return DFT_ERR_UNSUPPORTED;
  if (p->B <= 0 || p->B > 65535 || p->V < kM) return DFT_ERR_INVALID;
  if (p->lmax < 1) return DFT_ERR_INVALID;
  if (p->pmi_order != 0 && (p->pmi_order < 2 || p->pmi_order > 4)) return DFT_ERR_INVALID;
  const int W = p->N - 1 > kM ? p->N - 1 : kM;
  if (W > 64 || (int64_t)p->S * W < p->N - 1) return DFT_ERR_UNSUPPORTED;
  return DFT_OK;
}

extern "C" int dft_beam_build(const dft_build_params* p, const float* lp, const int32_t* ids, const float* rest,
                              const float* T, const float* logc, const float* c0, const int64_t* root,
                              dft_tree_out* out, int32_t* dev_status, void* stream) {
  int rc = dft_check_build_params(p);
  if (rc) return rc;
  if (!lp || !ids || !rest || !root || !out) return DFT_ERR_INVALID;
  if (p->use_ngram && !T) return DFT_ERR_INVALID;
  return dft_beam_launch(p, lp, ids, rest, T, logc, c0, root, out, dev_status, reinterpret_cast<cudaStream_t>(stream));
}

// ------------------------------------------------------------------------
// Standalone tree structure (tree_ops.tree_struct, tree_ops.py:68-89, plus
// nxt / sib of fc1_builder.py:41-47) for caller-given parent arrays.
namespace {

__global__ void tree_struct_kernel(int N, const int64_t* __restrict__ parent, float* anc, int64_t* depth,
                                   int64_t* cidx, int64_t* nxt, int64_t* sib, int32_t* st) {
  const int b = blockIdx.x, tid = threadIdx.x;
  __shared__ int par[kMaxNodes];
  __shared__ unsigned long long am[kMaxNodes];
  __shared__ int dep[kMaxNodes];
  const int64_t bN = (int64_t)b * N;
  if (tid < N) {
    int64_t p = parent[bN + tid];
    // tree_ops.py:72 clamps parents at 0; a parent must precede its child
    if (tid == 0) p = -1;
    if (tid > 0 && (p < 0 || p >= tid)) {
      raise_status(st, DFT_DEV_BAD_INDEX);
      p = p < 0 ? 0 : (p >= tid ? 0 : p);
    }
    par[tid] = (int)p;
  }
  __syncthreads();
  if (tid < N) {
    unsigned long long m = 0ull;
    int u = tid, d = -1;
    while (u >= 0) {
      m |= 1ull << u;
      u = par[u];
      ++d;
    }
    am[tid] = m;
    dep[tid] = d;
  }
  __syncthreads();
  if (tid < N) {
    const int n = tid, d = dep[n];
    if (depth) depth[bN + n] = d;
    if (cidx) {
      int u = n;
      for (int r = 0; r < 4; ++r) {
        cidx[(bN + n) * 4 + (3 - r)] = r <= d ? 3 + u : 3 - (r - d);
        if (r <= d && par[u] >= 0) u = par[u];
      }
    }
    int nx = -1, sb = -1;
    for (int v = 1; v < N; ++v) {
      if (nx < 0 && par[v] == n) nx = v;
      if (sb < 0 && v > n && par[v] == par[n]) sb = v;
    }
    if (nxt) nxt[bN + n] = nx;
    if (sib) sib[bN + n] = sb;
  }
  if (anc)
    for (int e = tid; e < N * N; e += blockDim.x) anc[bN * N + e] = (am[e / N] >> (e % N)) & 1ull ? 1.f : 0.f;
}

// Greedy tree acceptance (SGLang eagle tree verify, called at
// fc1_branch64.py:44): from the root, repeatedly accept the first child
// (nxt / sib order) whose token equals the target model's token at the
// current node; stop when none matches.  path[b] = accepted nodes, root
// first, -1 padded; accept_len[b] = their count; last[b] = the last one;
// bonus[b] = target token at the last node.
__global__ void accept_greedy_kernel(int B, int N, int P, const int64_t* __restrict__ tokens,
                                     const int64_t* __restrict__ nxt, const int64_t* __restrict__ sib,
                                     const int64_t* __restrict__ target, int64_t* path, int64_t* accept_len,
                                     int64_t* last, int64_t* bonus, int32_t* st) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b >= B) return;
  const int64_t bN = (int64_t)b * N;
  int cur = 0, n = 0;
  if (P > 0) path[(int64_t)b * P + n] = 0;
  ++n;
  for (int guard = 0; guard < N; ++guard) {
    const int64_t want = target[bN + cur];
    int64_t c = nxt[bN + cur];
    int found = -1;
    for (int g2 = 0; c >= 0 && g2 < N; ++g2) {
      if (c >= N) {
        raise_status(st, DFT_DEV_BAD_INDEX);
        break;
      }
      if (tokens[bN + c] == want) {
        found = (int)c;
        break;
      }
      c = sib[bN + c];
    }
    if (found < 0) break;
    cur = found;
    if (n < P) path[(int64_t)b * P + n] = cur;
    ++n;
  }
  for (int i = n; i < P; ++i) path[(int64_t)b * P + i] = -1;
  if (accept_len) accept_len[b] = n;
  if (last) last[b] = cur;
  if (bonus) bonus[b] = target[bN + cur];
}

// The same walk for trees of at most kMaxNodes nodes, one warp per request:
// the warp first stages the request's tokens / first children / siblings /
// targets in shared memory with coalesced loads (all in flight at once), so
// the dependent steps of the walk read shared memory instead of making one
// global round trip each.
__global__ void __launch_bounds__(128) accept_greedy_staged(int B, int N, int P, const int64_t* __restrict__ tokens,
                                                            const int64_t* __restrict__ nxt,
                                                            const int64_t* __restrict__ sib,
                                                            const int64_t* __restrict__ target, int64_t* path,
                                                            int64_t* accept_len, int64_t* last, int64_t* bonus,
                                                            int32_t* st) {
  __shared__ long long s_tok[4][kMaxNodes], s_nxt[4][kMaxNodes], s_sib[4][kMaxNodes], s_tgt[4][kMaxNodes];
  const int wl = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int b = blockIdx.x * 4 + wl;
  if (b >= B) return;   // the whole warp
  const int64_t bN = (int64_t)b * N;
  for (int i = lane; i < N; i += 32) {
    s_tok[wl][i] = tokens[bN + i];
    s_nxt[wl][i] = nxt[bN + i];
    s_sib[wl][i] = sib[bN + i];
    s_tgt[wl][i] = target[bN + i];
  }
  __syncwarp();
  if (lane != 0) return;
  int cur = 0, n = 0;
  if (P > 0) path[(int64_t)b * P + n] = 0;
  ++n;
  for (int guard = 0; guard < N; ++guard) {
    const long long want = s_tgt[wl][cur];
    long long c = s_nxt[wl][cur];
    int found = -1;
    for (int g2 = 0; c >= 0 && g2 < N; ++g2) {
      if (c >= N) {
        raise_status(st, DFT_DEV_BAD_INDEX);
        break;
      }
      if (s_tok[wl][c] == want) {
        found = (int)c;
        break;
      }
      c = s_sib[wl][c];
    }
    if (found < 0) break;
    cur = found;
    if (n < P) path[(int64_t)b * P + n] = cur;
    ++n;
  }
  for (int i = n; i < P; ++i) path[(int64_t)b * P + i] = -1;
  if (accept_len) accept_len[b] = n;
  if (last) last[b] = cur;
  if (bonus) bonus[b] = s_tgt[wl][cur];
}

}  // namespace

extern "C" int dft_tree_struct(int32_t B, int32_t N, const int64_t* parent, float* anc, int64_t* depth, int64_t* cidx,
                               int64_t* nxt, int64_t* sib, int32_t* dev_status, void* stream) {
  if (B <= 0 || B > 65535 || N < 1 || N > kMaxNodes || !parent) return B <= 0 || !parent ? DFT_ERR_INVALID
                                                                                         : DFT_ERR_UNSUPPORTED;
  tree_struct_kernel<<<B, 64, 0, reinterpret_cast<cudaStream_t>(stream)>>>(N, parent, anc, depth, cidx, nxt, sib,
                                                                           dev_status);
  DFT_LAUNCH_CHECK();
  return DFT_OK;
}

extern "C" int dft_accept_greedy(int32_t B, int32_t N, int32_t P, const int64_t* tokens, const int64_t* nxt,
                                 const int64_t* sib, const int64_t* target, int64_t* path, int64_t* accept_len,
                                 int64_t* last, int64_t* bonus, int32_t* dev_status, void* stream) {
  if (B <= 0 || N < 1 || P < 1 || !tokens || !nxt || !sib || !target || !path) return DFT_ERR_INVALID;
  if (N <= kMaxNodes)
    accept_greedy_staged<<<(B + 3) / 4, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        B, N, P, tokens, nxt, sib, target, path, accept_len, last, bonus, dev_status);
  else
    accept_greedy_kernel<<<(B + 127) / 128, 128, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        B, N, P, tokens, nxt, sib, target, path, accept_len, last, bonus, dev_status);
  DFT_LAUNCH_CHECK();
  return DFT_OK;
}
