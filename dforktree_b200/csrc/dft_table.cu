// n-gram tables in HBM and the PMI lookup kernels.
//
// Reference: dforktree/ngram_gpu.py -- sorted int64 key arrays searched with
// torch.searchsorted (~log2(8M) = 23 dependent HBM reads per query).  Here the
// arrays become open-addressed, linearly probed hash tables of 16-byte slots
// at load factor <= 0.35, so a query costs one 128-bit load (one 32-byte
// sector) in the common case.  The bigram table and the trigram-context
// table are merged into one "pair" table: both are keyed by u*V+v, and the
// bigram lookups of step t are the context lookups of step t+1.
#include "dft_common.cuh"

#include <cstdio>
#include <cstdlib>
#include <new>

using namespace dft;

struct dft_table {
  TableView view;
  Slot* pair = nullptr;
  Slot* trip = nullptr;
  Slot* quad = nullptr;
  float* prev = nullptr;
  float* pn = nullptr;
  float* n4c = nullptr;
  int64_t pair_slots = 0, trip_slots = 0, quad_slots = 0, bytes = 0;
  int device = -1;
};

namespace {

constexpr int kErrNegative = 1, kErrUnsorted = 2, kErrFull = 4;

__global__ void init_slots(Slot* tab, int64_t n) {
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i < n) {
    Slot s;
    s.key = kEmptyKey;
    s.f0 = 0.f;
    s.u1 = 0u;
    tab[i] = s;
  }
}

// field 0: f0 = value; field 1: u1 = bits(value); field 2: f0 = value, u1 = rank i
__global__ void insert_keys(Slot* tab, unsigned long long mask, const int64_t* __restrict__ keys,
                            const float* __restrict__ vals, int64_t n, int field, int32_t* err) {
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  long long k = keys[i];
  if (k < 0) {
    atomicOr(err, kErrNegative);
    return;
  }
  if (i > 0) {
    long long pk = keys[i - 1];
    if (pk == k) return;  // duplicate: the first occurrence wins (searchsorted 'left')
    if (pk > k) atomicOr(err, kErrUnsorted);
  }
  float v = vals ? vals[i] : 0.f;
  unsigned long long uk = static_cast<unsigned long long>(k);
  unsigned long long h = mix64(uk) & mask;
  for (unsigned long long t = 0; t <= mask; ++t) {
    unsigned long long prev = atomicCAS(&tab[h].key, kEmptyKey, uk);
    if (prev == kEmptyKey || prev == uk) {
      if (field == 0) {
        tab[h].f0 = v;
      } else if (field == 1) {
        tab[h].u1 = __float_as_uint(v);
      } else {
        tab[h].f0 = v;
        tab[h].u1 = static_cast<uint32_t>(i);
      }
      return;
    }
    h = (h + 1) & mask;
  }
  atomicOr(err, kErrFull);
}

int64_t pow2_at_least(double x) {
  int64_t c = 1024;
  while ((double)c < x) c <<= 1;
  return c;
}

int alloc_table(Slot** out, int64_t slots, cudaStream_t st) {
  DFT_CUDA_CHECK(cudaMalloc(out, slots * sizeof(Slot)));
  init_slots<<<(unsigned)((slots + 255) / 256), 256, 0, st>>>(*out, slots);
  DFT_LAUNCH_CHECK();
  return DFT_OK;
}

int insert(Slot* tab, int64_t slots, const int64_t* keys, const float* vals, int64_t n, int field, int32_t* err,
           cudaStream_t st) {
  if (n <= 0) return DFT_OK;
  insert_keys<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(tab, (unsigned long long)(slots - 1), keys, vals, n,
                                                            field, err);
  DFT_LAUNCH_CHECK();
  return DFT_OK;
}

void free_table(dft_table* t) {
  if (!t) return;
  cudaFree(t->pair);
  cudaFree(t->trip);
  cudaFree(t->quad);
  cudaFree(t->prev);
  cudaFree(t->pn);
  cudaFree(t->n4c);
  delete t;
}

}  // namespace

extern "C" int dft_table_create(const dft_table_desc* d, dft_table** out, void* stream) {
  if (!d || !out) return DFT_ERR_INVALID;
  *out = nullptr;
  if (d->V <= 0 || d->V > (int64_t)1 << 30) return DFT_ERR_INVALID;
  if (!d->prev || !d->pn) return DFT_ERR_INVALID;
  if (d->n_bigram < 0 || d->n_trigram < 0 || d->n_ctx3 < 0 || d->n_quad < 0) return DFT_ERR_INVALID;
  if ((d->n_bigram && (!d->keys || !d->cab)) || (d->n_trigram && (!d->keys3 || !d->c3)) ||
      (d->n_ctx3 && (!d->keys3c || !d->n3c)) || (d->n_quad && (!d->keys4 || !d->c4 || !d->n4c)))
    return DFT_ERR_INVALID;
  if (d->n_trigram > 0xFFFFFFFFll) return DFT_ERR_UNSUPPORTED;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  float load = d->max_load > 0.f && d->max_load < 0.95f ? d->max_load : 0.35f;

  dft_table* t = new (std::nothrow) dft_table();
  if (!t) return DFT_ERR_CUDA;
  cudaGetDevice(&t->device);
  int32_t* err = nullptr;
  int rc = DFT_OK;
#define TRY(x)                 \
  do {                         \
    rc = (x);                  \
    if (rc != DFT_OK) goto fail; \
  } while (0)
  TRY(cudaMalloc(&err, sizeof(int32_t)) == cudaSuccess ? DFT_OK : DFT_ERR_CUDA);
  TRY(cudaMemsetAsync(err, 0, sizeof(int32_t), st) == cudaSuccess ? DFT_OK : DFT_ERR_CUDA);

  t->pair_slots = pow2_at_least((double)(d->n_bigram + d->n_ctx3) / load);
  TRY(alloc_table(&t->pair, t->pair_slots, st));
  TRY(insert(t->pair, t->pair_slots, d->keys, d->cab, d->n_bigram, 0, err, st));
  TRY(insert(t->pair, t->pair_slots, d->keys3c, d->n3c, d->n_ctx3, 1, err, st));
  if (d->n_trigram) {
    t->trip_slots = pow2_at_least((double)d->n_trigram / load);
    TRY(alloc_table(&t->trip, t->trip_slots, st));
    TRY(insert(t->trip, t->trip_slots, d->keys3, d->c3, d->n_trigram, 2, err, st));
  }
  if (d->n_quad) {
    t->quad_slots = pow2_at_least((double)d->n_quad / load);
    TRY(alloc_table(&t->quad, t->quad_slots, st));
    TRY(insert(t->quad, t->quad_slots, d->keys4, d->c4, d->n_quad, 0, err, st));
    TRY(cudaMalloc(&t->n4c, d->n_trigram * sizeof(float)) == cudaSuccess ? DFT_OK : DFT_ERR_CUDA);
    TRY(cudaMemcpyAsync(t->n4c, d->n4c, d->n_trigram * sizeof(float), cudaMemcpyDeviceToDevice, st) ==
                cudaSuccess ? DFT_OK : DFT_ERR_CUDA);
  }
  TRY(cudaMalloc(&t->prev, d->V * sizeof(float)) == cudaSuccess ? DFT_OK : DFT_ERR_CUDA);
  TRY(cudaMalloc(&t->pn, d->V * sizeof(float)) == cudaSuccess ? DFT_OK : DFT_ERR_CUDA);
  TRY(cudaMemcpyAsync(t->prev, d->prev, d->V * sizeof(float), cudaMemcpyDeviceToDevice, st) == cudaSuccess
          ? DFT_OK : DFT_ERR_CUDA);
  TRY(cudaMemcpyAsync(t->pn, d->pn, d->V * sizeof(float), cudaMemcpyDeviceToDevice, st) == cudaSuccess
          ? DFT_OK : DFT_ERR_CUDA);
  {
    int32_t herr = 0;
    TRY(cudaMemcpyAsync(&herr, err, sizeof(int32_t), cudaMemcpyDeviceToHost, st) == cudaSuccess ? DFT_OK
                                                                                                 : DFT_ERR_CUDA);
    TRY(cudaStreamSynchronize(st) == cudaSuccess ? DFT_OK : DFT_ERR_CUDA);
    if (herr) {
      rc = DFT_ERR_TABLE;
      goto fail;
    }
  }
  cudaFree(err);
  t->bytes = (t->pair_slots + t->trip_slots + t->quad_slots) * (int64_t)sizeof(Slot) +
             2 * d->V * (int64_t)sizeof(float) + (d->n_quad ? d->n_trigram * (int64_t)sizeof(float) : 0);
  {
    TableView& v = t->view;
    v.V = d->V;
    v.pair = t->pair;
    v.pair_mask = (unsigned long long)(t->pair_slots - 1);
    v.trip = t->trip;
    v.trip_mask = t->trip_slots ? (unsigned long long)(t->trip_slots - 1) : 0ull;
    v.quad = t->quad;
    v.quad_mask = t->quad_slots ? (unsigned long long)(t->quad_slots - 1) : 0ull;
    v.prev = t->prev;
    v.pn = t->pn;
    v.n4c = t->n4c;
    v.has_pair = 1;
    v.has_trip = d->n_trigram > 0;
    v.has_quad = d->n_quad > 0;
    v.has_ctx = d->n_ctx3 > 0;
    v.beta2 = d->beta2;
    v.beta3 = d->beta3;
    v.beta4 = d->beta4;
    v.clip = d->clip;
  }
  *out = t;
  return DFT_OK;
fail:
  cudaFree(err);
  free_table(t);
  return rc;
#undef TRY
}

extern "C" int dft_table_destroy(dft_table* t) {
  if (!t) return DFT_ERR_INVALID;
  free_table(t);
  return DFT_OK;
}

extern "C" int dft_table_info(const dft_table* t, int64_t* V, int64_t* ps, int64_t* ts, int64_t* qs,
                              int64_t* bytes) {
  if (!t) return DFT_ERR_INVALID;
  if (V) *V = t->view.V;
  if (ps) *ps = t->pair_slots;
  if (ts) *ts = t->trip_slots;
  if (qs) *qs = t->quad_slots;
  if (bytes) *bytes = t->bytes;
  return DFT_OK;
}

const TableView* dft_table_view(const dft_table* t) { return t ? &t->view : nullptr; }

// ------------------------------------------------------------ lookups ----

namespace {

__device__ __forceinline__ float prev_at(const TableView& t, long long b, int32_t* st) {
  if (b < 0) return 0.f;  // ngram_gpu.py:41 where(b >= 0, prev[b], 0)
  if (b >= t.V) {
    raise_status(st, DFT_DEV_BAD_TOKEN);
    return 0.f;
  }
  return __ldg(t.prev + b);
}

__device__ float p2_query(const TableView& t, long long b, long long c, int32_t* st) {
  uint4 s = probe(t.pair, t.pair_mask, b * t.V + c, st);
  return p2_from(__uint_as_float(s.z), prev_at(t, b, st), pn_at(t, c, st), t.beta2);
}

__device__ float p3_query(const TableView& t, long long a, long long b, long long c, int32_t* st) {
  bool ok = a >= 0 && b >= 0;
  long long V = t.V;
  float nab = 0.f, nabc = 0.f;
  if (ok) {
    if (t.has_ctx) nab = __uint_as_float(probe(t.pair, t.pair_mask, a * V + b, st).w);
    if (t.has_trip) nabc = __uint_as_float(probe(t.trip, t.trip_mask, (a * V + b) * V + c, st).z);
  }
  return p3_from(nabc, nab, p2_query(t, b, c, st), t.beta3);
}

__device__ float p4_query(const TableView& t, long long z, long long a, long long b, long long c, int32_t* st) {
  bool ok = z >= 0 && a >= 0 && b >= 0;
  long long V = t.V;
  float n4 = 0.f, c4 = 0.f;
  if (ok && t.has_trip) {
    uint4 s = probe(t.trip, t.trip_mask, (z * V + a) * V + b, st);
    if (slot_key(s) == static_cast<unsigned long long>((z * V + a) * V + b)) {
      long long i3 = (long long)s.w;
      if (t.has_quad) {
        n4 = __ldg(t.n4c + i3);
        c4 = __uint_as_float(probe(t.quad, t.quad_mask, i3 * V + c, st).z);
      }
    }
  }
  float p3 = p3_query(t, a, b, c, st);
  return __fdiv_rn(__fadd_rn(c4, __fmul_rn(t.beta4, p3)), __fadd_rn(n4, t.beta4));
}

__global__ void ngram_eval_kernel(TableView t, int order, int what, const int64_t* __restrict__ z,
                                  const int64_t* __restrict__ a, const int64_t* __restrict__ b,
                                  const int64_t* __restrict__ c, int64_t n, float* __restrict__ out, int32_t* st) {
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i >= n) return;
  long long bb = b[i], cc = c[i];
  float p;
  if (order == 2) {
    p = p2_query(t, bb, cc, st);
  } else if (order == 3) {
    p = p3_query(t, a[i], bb, cc, st);
  } else {
    p = p4_query(t, z[i], a[i], bb, cc, st);
  }
  out[i] = what ? pmi_from(p, logf(pn_at(t, cc, st)), t.clip) : p;
}

// Dense PMI tensor for one (request, step t): T[i, j, l] = PMI(a_i, b_j, c_l)
// with a = E[t+1], b = E[t+2] = ids[t], c = ids[t+1] and E = [pre1; root; ids]
// (tree_ops.py:56-62, order 3).  256 threads: phase 1 resolves the 256
// context pairs (a_i, b_j) and 256 bigram pairs (b_j, c_l) in the pair table
// into shared memory; phase 2 issues 16 independent triple probes per thread
// (first-slot loads all in flight) and writes T coalesced.
constexpr int kM = 16;

__global__ void __launch_bounds__(256) pmi_dense_kernel(TableView t, int S, const int32_t* __restrict__ ids,
                                                        const int64_t* __restrict__ root,
                                                        const int64_t* __restrict__ pre1, float* __restrict__ T,
                                                        int32_t* st) {
  const int tstep = blockIdx.x;  // 0 .. S-2
  const int req = blockIdx.y;
  const int tid = threadIdx.x;
  __shared__ long long sa[kM], sb[kM], sc[kM];
  __shared__ float s_nab[kM * kM], s_p2[kM * kM], s_lpn[kM];
  const int32_t* idr = ids + (int64_t)req * S * kM;
  if (tid < kM) {
    sa[tid] = tstep == 0 ? (long long)root[req] : (long long)idr[(tstep - 1) * kM + tid];
    sb[tid] = idr[tstep * kM + tid];
    sc[tid] = idr[(tstep + 1) * kM + tid];
  }
  __syncthreads();
  const long long V = t.V;
  {
    // context pair (a_i, b_j) and bigram pair (b_j, c_l), one each per thread
    int i = tid >> 4, j = tid & 15;
    long long a = sa[i], b = sb[j];
    long long qctx = (a >= 0 && b >= 0 && t.has_ctx) ? a * V + b : -1;
    int jj = tid >> 4, l = tid & 15;
    long long b2 = sb[jj], c2 = sc[l];
    long long qbig = b2 * V + c2;
    uint4 s1 = first_slot(t.pair, t.pair_mask, qctx);
    uint4 s2 = first_slot(t.pair, t.pair_mask, qbig);
    float pnc = pn_at(t, c2, st);
    float prevb = prev_at(t, b2, st);
    s1 = probe_from(t.pair, t.pair_mask, qctx, s1, st);
    s2 = probe_from(t.pair, t.pair_mask, qbig, s2, st);
    s_nab[tid] = __uint_as_float(s1.w);
    s_p2[tid] = p2_from(__uint_as_float(s2.z), prevb, pnc, t.beta2);
    if (jj == 0) s_lpn[l] = logf(pnc);
  }
  __syncthreads();
  float* Tout = T + ((int64_t)req * (S - 1) + tstep) * (kM * kM * kM);
  long long q[16];
  uint4 s[16];
#pragma unroll
  for (int r = 0; r < 16; ++r) {
    int e = tid + 256 * r;
    int i = e >> 8, j = (e >> 4) & 15, l = e & 15;
    long long a = sa[i], b = sb[j];
    q[r] = (a >= 0 && b >= 0 && t.has_trip) ? (a * V + b) * V + sc[l] : -1;
    s[r] = first_slot(t.trip, t.trip_mask, q[r]);
  }
#pragma unroll
  for (int r = 0; r < 16; ++r) {
    int e = tid + 256 * r;
    int i = e >> 8, j = (e >> 4) & 15, l = e & 15;
    uint4 hit = probe_from(t.trip, t.trip_mask, q[r], s[r], st);
    float p3 = p3_from(__uint_as_float(hit.z), s_nab[i * 16 + j], s_p2[j * 16 + l], t.beta3);
    Tout[e] = pmi_from(p3, s_lpn[l], t.clip);
  }
}

}  // namespace

extern "C" int dft_ngram_eval(const dft_table* table, int order, int what, const int64_t* z, const int64_t* a,
                              const int64_t* b, const int64_t* c, int64_t n, float* out, int32_t* dev_status,
                              void* stream) {
  if (!table || !b || !c || !out || n < 0) return DFT_ERR_INVALID;
  if (order < 2 || order > 4 || (what != 0 && what != 1)) return DFT_ERR_INVALID;
  if (order >= 3 && !a) return DFT_ERR_INVALID;
  if (order == 4 && !z) return DFT_ERR_INVALID;
  if (n == 0) return DFT_OK;
  ngram_eval_kernel<<<(unsigned)((n + 255) / 256), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
      table->view, order, what, z, a, b, c, n, out, dev_status);
  DFT_LAUNCH_CHECK();
  return DFT_OK;
}

int dft_pmi_dense_launch(const dft_table* table, const dft_build_params* p, const int32_t* ids, const int64_t* root,
                         const int64_t* pre1, float* T, int32_t* dev_status, cudaStream_t st) {
  (void)pre1;  // order 3 does not read pre1 (E[0] is used by order 4 only)
  dim3 grid(p->S - 1, p->B);
  pmi_dense_kernel<<<grid, 256, 0, st>>>(table->view, p->S, ids, root, pre1, T, dev_status);
  DFT_LAUNCH_CHECK();
  return DFT_OK;
}

extern "C" int dft_pmi_dense(const dft_table* table, const dft_build_params* p, const int32_t* ids,
                             const int64_t* root, const int64_t* pre1, float* T, int32_t* dev_status, void* stream) {
  if (!table || !p || !ids || !root || !T) return DFT_ERR_INVALID;
  if (p->M != kM) return DFT_ERR_UNSUPPORTED;
  if (p->B <= 0 || p->S < 2 || p->B > 65535) return DFT_ERR_INVALID;
  return dft_pmi_dense_launch(table, p, ids, root, pre1, T, dev_status, reinterpret_cast<cudaStream_t>(stream));
}
