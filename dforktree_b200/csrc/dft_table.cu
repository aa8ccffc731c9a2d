// n-gram tables in HBM and the PMI lookup kernels (ngram_gpu.py:8-70).
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
#include <cstring>
#include <new>
#include <string>

using namespace dft;

struct dft_table {
  TableView view;
  Slot* pair = nullptr;
  Slot* trip = nullptr;
  Slot* quad = nullptr;
  uint8_t* pair_fp = nullptr;   // one fingerprint byte per slot (derived: rebuilt on create and load)
  uint8_t* trip_fp = nullptr;
  uint8_t* quad_fp = nullptr;
  float* prev = nullptr;
  float* pn = nullptr;
  float* n4c = nullptr;
  int64_t pair_slots = 0, trip_slots = 0, quad_slots = 0, bytes = 0;
  int64_t n4c_len = 0;  // entries of n4c (the trigram count when a quad table exists)
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

// fingerprint byte of every slot (0 = empty)
__global__ void build_fingerprints(const Slot* tab, uint8_t* fp, int64_t n) {
  int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x;
  if (i < n) {
    const unsigned long long k = tab[i].key;
    fp[i] = k == kEmptyKey ? 0 : (uint8_t)fp_of(mix64(k));
  }
}

int alloc_fingerprints(const Slot* tab, uint8_t** fp, int64_t slots, cudaStream_t st) {
  if (!slots) return DFT_OK;
  DFT_CUDA_CHECK(cudaMalloc(fp, (size_t)slots));
  build_fingerprints<<<(unsigned)((slots + 255) / 256), 256, 0, st>>>(tab, *fp, slots);
  DFT_LAUNCH_CHECK();
  return DFT_OK;
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

// Device view and byte count of a table whose arrays are in place.
void set_view(dft_table* t, int64_t V, bool has_trip, bool has_quad, bool has_ctx, float beta2, float beta3,
              float beta4, float clip) {
  t->bytes = (t->pair_slots + t->trip_slots + t->quad_slots) * (int64_t)(sizeof(Slot) + 1) +
             2 * V * (int64_t)sizeof(float) + t->n4c_len * (int64_t)sizeof(float);
  TableView& v = t->view;
  v.V = V;
  v.pair = t->pair;
  v.pair_mask = (unsigned long long)(t->pair_slots - 1);
  v.trip = t->trip;
  v.trip_mask = t->trip_slots ? (unsigned long long)(t->trip_slots - 1) : 0ull;
  v.quad = t->quad;
  v.quad_mask = t->quad_slots ? (unsigned long long)(t->quad_slots - 1) : 0ull;
  v.pair_fp = t->pair_fp;
  v.trip_fp = t->trip_fp;
  v.quad_fp = t->quad_fp;
  v.prev = t->prev;
  v.pn = t->pn;
  v.n4c = t->n4c;
  v.has_pair = 1;
  v.has_trip = has_trip;
  v.has_quad = has_quad;
  v.has_ctx = has_ctx;
  v.beta2 = beta2;
  v.beta3 = beta3;
  v.beta4 = beta4;
  v.clip = clip;
}

void free_table(dft_table* t) {
  if (!t) return;
  cudaFree(t->pair);
  cudaFree(t->trip);
  cudaFree(t->quad);
  cudaFree(t->pair_fp);
  cudaFree(t->trip_fp);
  cudaFree(t->quad_fp);
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
  err = nullptr;
  TRY(alloc_fingerprints(t->pair, &t->pair_fp, t->pair_slots, st));
  TRY(alloc_fingerprints(t->trip, &t->trip_fp, t->trip_slots, st));
  TRY(alloc_fingerprints(t->quad, &t->quad_fp, t->quad_slots, st));
  TRY(cudaStreamSynchronize(st) == cudaSuccess ? DFT_OK : DFT_ERR_CUDA);
  t->n4c_len = d->n_quad ? d->n_trigram : 0;
  set_view(t, d->V, d->n_trigram > 0, d->n_quad > 0, d->n_ctx3 > 0, d->beta2, d->beta3, d->beta4, d->clip);
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

extern "C" int dft_table_set_params(dft_table* t, float beta2, float beta3, float beta4, float clip) {
  if (!t) return DFT_ERR_INVALID;
  t->view.beta2 = beta2;
  t->view.beta3 = beta3;
  t->view.beta4 = beta4;
  t->view.clip = clip;
  return DFT_OK;
}

extern "C" int dft_table_copy_marginals(const dft_table* t, float* prev, float* pn, void* stream) {
  if (!t) return DFT_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const size_t n = (size_t)t->view.V * sizeof(float);
  if (prev && cudaMemcpyAsync(prev, t->prev, n, cudaMemcpyDefault, st) != cudaSuccess) return DFT_ERR_CUDA;
  if (pn && cudaMemcpyAsync(pn, t->pn, n, cudaMemcpyDefault, st) != cudaSuccess) return DFT_ERR_CUDA;
  return DFT_OK;
}

// ------------------------------------------------------- cached table file --
// The built hash tables as one file: a 128-byte header, then the device images
// of the pair / triple / quad slot arrays, prev[V], pn[V] and n4c, in that
// order, little-endian.  Loading is a sequential read plus host-to-device
// copies (no key sort, no hash insert); the slot images are byte-identical to
// the saved table's, so every lookup answers the same.  A 64-bit checksum over
// the payload guards against truncated or damaged files.
namespace {

constexpr char kMagic[8] = {'D', 'F', 'T', 'T', 'A', 'B', 'L', 'E'};
constexpr uint32_t kFileVersion = 1;
constexpr uint32_t kFlagTrip = 1, kFlagQuad = 2, kFlagCtx = 4;
constexpr size_t kChunk = size_t(32) << 20;  // staging chunk (pinned), multiple of 8

struct FileHeader {
  char magic[8];
  uint32_t version, flags;
  int64_t V, pair_slots, trip_slots, quad_slots, n4c_len;
  float beta2, beta3, beta4, clip;
  uint64_t payload_bytes;
  uint64_t checksum;
  uint64_t reserved[5];
};
static_assert(sizeof(FileHeader) == 128, "table file header is 128 bytes");

// Word-wise FNV-1a (64-bit offset basis and prime); a section's last partial
// word is zero-padded.  Chunks handed in are multiples of 8 bytes except the
// last chunk of a section.
uint64_t fnv_words(const unsigned char* p, size_t n, uint64_t h) {
  size_t w = n / 8;
  for (size_t i = 0; i < w; ++i) {
    uint64_t x;
    memcpy(&x, p + 8 * i, 8);
    h = (h ^ x) * 0x100000001b3ull;
  }
  if (n % 8) {
    uint64_t x = 0;
    memcpy(&x, p + 8 * w, n % 8);
    h = (h ^ x) * 0x100000001b3ull;
  }
  return h;
}
constexpr uint64_t kFnvBasis = 0xcbf29ce484222325ull;

struct Section {
  void* dev;
  size_t bytes;
};

int sections_of(const dft_table* t, Section out[6]) {
  out[0] = {t->pair, (size_t)t->pair_slots * sizeof(Slot)};
  out[1] = {t->trip, (size_t)t->trip_slots * sizeof(Slot)};
  out[2] = {t->quad, (size_t)t->quad_slots * sizeof(Slot)};
  out[3] = {t->prev, (size_t)t->view.V * sizeof(float)};
  out[4] = {t->pn, (size_t)t->view.V * sizeof(float)};
  out[5] = {t->n4c, (size_t)t->n4c_len * sizeof(float)};
  return 6;
}

struct Staging {
  unsigned char* buf[2] = {nullptr, nullptr};
  cudaEvent_t ev[2] = {nullptr, nullptr};
  bool ok() const { return buf[0] && buf[1] && ev[0] && ev[1]; }
  Staging() {
    for (int i = 0; i < 2; ++i) {
      if (cudaMallocHost(&buf[i], kChunk) != cudaSuccess) buf[i] = nullptr;
      if (cudaEventCreateWithFlags(&ev[i], cudaEventDisableTiming) != cudaSuccess) ev[i] = nullptr;
    }
  }
  ~Staging() {
    for (int i = 0; i < 2; ++i) {
      if (buf[i]) cudaFreeHost(buf[i]);
      if (ev[i]) cudaEventDestroy(ev[i]);
    }
  }
};

}  // namespace

extern "C" int dft_table_save(const dft_table* t, const char* path, void* stream) {
  if (!t || !path || !*path) return DFT_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  Staging sg;
  if (!sg.ok()) return DFT_ERR_CUDA;
  Section sec[6];
  sections_of(t, sec);
  FileHeader h;
  memset(&h, 0, sizeof h);
  memcpy(h.magic, kMagic, 8);
  h.version = kFileVersion;
  h.flags = (t->view.has_trip ? kFlagTrip : 0) | (t->view.has_quad ? kFlagQuad : 0) | (t->view.has_ctx ? kFlagCtx : 0);
  h.V = t->view.V;
  h.pair_slots = t->pair_slots;
  h.trip_slots = t->trip_slots;
  h.quad_slots = t->quad_slots;
  h.n4c_len = t->n4c_len;
  h.beta2 = t->view.beta2;
  h.beta3 = t->view.beta3;
  h.beta4 = t->view.beta4;
  h.clip = t->view.clip;
  // written under a temporary name and renamed, so a reader never sees a partial file
  const std::string tmp = std::string(path) + ".partial";
  FILE* f = fopen(tmp.c_str(), "wb");
  if (!f) return DFT_ERR_IO;
  int rc = DFT_OK;
  uint64_t sum = kFnvBasis, total = 0;
  if (fwrite(&h, sizeof h, 1, f) != 1) rc = DFT_ERR_IO;
  // device -> pinned chunk i+1 is in flight while chunk i is hashed and written
  for (int s = 0; s < 6 && rc == DFT_OK; ++s) {
    const unsigned char* src = static_cast<const unsigned char*>(sec[s].dev);
    const size_t n = sec[s].bytes;
    const size_t nchunks = (n + kChunk - 1) / kChunk;
    if (nchunks && (cudaMemcpyAsync(sg.buf[0], src, n < kChunk ? n : kChunk, cudaMemcpyDeviceToHost, st) !=
                        cudaSuccess ||
                    cudaEventRecord(sg.ev[0], st) != cudaSuccess))
      rc = DFT_ERR_CUDA;
    for (size_t c = 0; c < nchunks && rc == DFT_OK; ++c) {
      const size_t off = c * kChunk, len = n - off < kChunk ? n - off : kChunk;
      if (c + 1 < nchunks) {
        const size_t off2 = off + kChunk, len2 = n - off2 < kChunk ? n - off2 : kChunk;
        if (cudaMemcpyAsync(sg.buf[(c + 1) & 1], src + off2, len2, cudaMemcpyDeviceToHost, st) != cudaSuccess ||
            cudaEventRecord(sg.ev[(c + 1) & 1], st) != cudaSuccess) {
          rc = DFT_ERR_CUDA;
          break;
        }
      }
      if (cudaEventSynchronize(sg.ev[c & 1]) != cudaSuccess) {
        rc = DFT_ERR_CUDA;
        break;
      }
      sum = fnv_words(sg.buf[c & 1], len, sum);
      if (fwrite(sg.buf[c & 1], 1, len, f) != len) rc = DFT_ERR_IO;
      total += len;
    }
  }
  if (rc != DFT_OK) cudaStreamSynchronize(st);  // no copy into the staging buffers may outlive them
  h.payload_bytes = total;
  h.checksum = sum;
  if (rc == DFT_OK && (fseek(f, 0, SEEK_SET) != 0 || fwrite(&h, sizeof h, 1, f) != 1)) rc = DFT_ERR_IO;
  if (fclose(f) != 0 && rc == DFT_OK) rc = DFT_ERR_IO;
  if (rc == DFT_OK && rename(tmp.c_str(), path) != 0) rc = DFT_ERR_IO;
  if (rc != DFT_OK) remove(tmp.c_str());
  return rc;
}

extern "C" int dft_table_load(const char* path, dft_table** out, void* stream) {
  if (!path || !out) return DFT_ERR_INVALID;
  *out = nullptr;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  FILE* f = fopen(path, "rb");
  if (!f) return DFT_ERR_IO;
  FileHeader h;
  const auto pow2_or_zero = [](int64_t x, bool required) {
    if (x == 0) return !required;
    return x >= 1024 && x <= ((int64_t)1 << 36) && (x & (x - 1)) == 0;
  };
  if (fread(&h, sizeof h, 1, f) != 1 || memcmp(h.magic, kMagic, 8) != 0 || h.version != kFileVersion ||
      h.V <= 0 || h.V > ((int64_t)1 << 30) || !pow2_or_zero(h.pair_slots, true) ||
      !pow2_or_zero(h.trip_slots, (h.flags & kFlagTrip) != 0) || !pow2_or_zero(h.quad_slots, (h.flags & kFlagQuad) != 0) ||
      ((h.flags & kFlagTrip) == 0) != (h.trip_slots == 0) || ((h.flags & kFlagQuad) == 0) != (h.quad_slots == 0) ||
      h.n4c_len < 0 || h.n4c_len > ((int64_t)1 << 32) || ((h.flags & kFlagQuad) == 0 && h.n4c_len != 0)) {
    fclose(f);
    return DFT_ERR_IO;
  }
  const uint64_t expect = (uint64_t)(h.pair_slots + h.trip_slots + h.quad_slots) * sizeof(Slot) +
                          (uint64_t)(2 * h.V + h.n4c_len) * sizeof(float);
  if (h.payload_bytes != expect) {
    fclose(f);
    return DFT_ERR_IO;
  }
  dft_table* t = new (std::nothrow) dft_table();
  if (!t) {
    fclose(f);
    return DFT_ERR_CUDA;
  }
  cudaGetDevice(&t->device);
  t->pair_slots = h.pair_slots;
  t->trip_slots = h.trip_slots;
  t->quad_slots = h.quad_slots;
  t->n4c_len = h.n4c_len;
  t->view.V = h.V;
  int rc = DFT_OK;
  const auto alloc = [&](void** p, size_t n) {
    if (rc == DFT_OK && n && cudaMalloc(p, n) != cudaSuccess) rc = DFT_ERR_CUDA;
  };
  alloc(reinterpret_cast<void**>(&t->pair), (size_t)h.pair_slots * sizeof(Slot));
  alloc(reinterpret_cast<void**>(&t->trip), (size_t)h.trip_slots * sizeof(Slot));
  alloc(reinterpret_cast<void**>(&t->quad), (size_t)h.quad_slots * sizeof(Slot));
  alloc(reinterpret_cast<void**>(&t->prev), (size_t)h.V * sizeof(float));
  alloc(reinterpret_cast<void**>(&t->pn), (size_t)h.V * sizeof(float));
  alloc(reinterpret_cast<void**>(&t->n4c), (size_t)h.n4c_len * sizeof(float));
  Staging sg;
  if (rc == DFT_OK && !sg.ok()) rc = DFT_ERR_CUDA;
  Section sec[6];
  sections_of(t, sec);
  uint64_t sum = kFnvBasis;
  // file -> pinned buffer c&1 waits only for the copy that last used that buffer
  size_t c = 0;
  bool pending[2] = {false, false};
  for (int s = 0; s < 6 && rc == DFT_OK; ++s) {
    unsigned char* dst = static_cast<unsigned char*>(sec[s].dev);
    for (size_t off = 0; off < sec[s].bytes && rc == DFT_OK; off += kChunk, ++c) {
      const size_t len = sec[s].bytes - off < kChunk ? sec[s].bytes - off : kChunk;
      const int i = (int)(c & 1);
      if (pending[i] && cudaEventSynchronize(sg.ev[i]) != cudaSuccess) {
        rc = DFT_ERR_CUDA;
        break;
      }
      if (fread(sg.buf[i], 1, len, f) != len) {
        rc = DFT_ERR_IO;
        break;
      }
      sum = fnv_words(sg.buf[i], len, sum);
      if (cudaMemcpyAsync(dst + off, sg.buf[i], len, cudaMemcpyHostToDevice, st) != cudaSuccess ||
          cudaEventRecord(sg.ev[i], st) != cudaSuccess) {
        rc = DFT_ERR_CUDA;
        break;
      }
      pending[i] = true;
    }
  }
  unsigned char extra;
  if (rc == DFT_OK && (sum != h.checksum || fread(&extra, 1, 1, f) != 0)) rc = DFT_ERR_IO;
  fclose(f);
  if (cudaStreamSynchronize(st) != cudaSuccess && rc == DFT_OK) rc = DFT_ERR_CUDA;
  if (rc == DFT_OK) rc = alloc_fingerprints(t->pair, &t->pair_fp, t->pair_slots, st);
  if (rc == DFT_OK) rc = alloc_fingerprints(t->trip, &t->trip_fp, t->trip_slots, st);
  if (rc == DFT_OK) rc = alloc_fingerprints(t->quad, &t->quad_fp, t->quad_slots, st);
  if (rc == DFT_OK && cudaStreamSynchronize(st) != cudaSuccess) rc = DFT_ERR_CUDA;
  if (rc != DFT_OK) {
    free_table(t);
    return rc;
  }
  set_view(t, h.V, (h.flags & kFlagTrip) != 0, (h.flags & kFlagQuad) != 0, (h.flags & kFlagCtx) != 0, h.beta2,
           h.beta3, h.beta4, h.clip);
  *out = t;
  return DFT_OK;
}

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
  uint4 s = probe_fp(t.pair, t.pair_fp, t.pair_mask, b * t.V + c, st);
  return p2_from(__uint_as_float(s.z), prev_at(t, b, st), pn_at(t, c, st), t.beta2);
}

__device__ float p3_query(const TableView& t, long long a, long long b, long long c, int32_t* st) {
  bool ok = a >= 0 && b >= 0;
  long long V = t.V;
  float nab = 0.f, nabc = 0.f;
  if (ok) {
    if (t.has_ctx) nab = __uint_as_float(probe_fp(t.pair, t.pair_fp, t.pair_mask, a * V + b, st).w);
    if (t.has_trip) nabc = __uint_as_float(probe_fp(t.trip, t.trip_fp, t.trip_mask, (a * V + b) * V + c, st).z);
  }
  return p3_from(nabc, nab, p2_query(t, b, c, st), t.beta3);
}

__device__ float p4_query(const TableView& t, long long z, long long a, long long b, long long c, int32_t* st) {
  bool ok = z >= 0 && a >= 0 && b >= 0;
  long long V = t.V;
  float n4 = 0.f, c4 = 0.f;
  if (ok && t.has_trip) {
    uint4 s = probe_fp(t.trip, t.trip_fp, t.trip_mask, (z * V + a) * V + b, st);
    if (slot_key(s) == static_cast<unsigned long long>((z * V + a) * V + b)) {
      long long i3 = (long long)s.w;
      if (t.has_quad) {
        n4 = __ldg(t.n4c + i3);
        c4 = __uint_as_float(probe_fp(t.quad, t.quad_fp, t.quad_mask, i3 * V + c, st).z);
      }
    }
  }
  return p4_from(c4, n4, p3_query(t, a, b, c, st), t.beta4);
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

// Fingerprint probing in two rounds for many independent queries: round 1
// loads the 8 fingerprints around each query's bucket (L2-resident), round 2
// scans them -- an empty byte ends a miss, a matching byte names a candidate
// slot, which is then read from HBM and compared.  A false candidate or a
// chain longer than the loaded word continues in probe_fp_from.
__device__ __forceinline__ uint2 fp_round1(const uint8_t* fp, unsigned long long mask, long long q, uint64_t pol) {
  if (q < 0 || fp == nullptr) return make_uint2(0u, 0u);   // scans as an empty bucket: no match
  return ld_fp8(fp + ((mix64(static_cast<unsigned long long>(q)) & mask) & ~7ull), pol);
}

__device__ __forceinline__ uint4 fp_round2(const Slot* tab, const uint8_t* fp, unsigned long long mask, long long q,
                                           uint2 w, int32_t* st) {
  const uint4 z = miss_slot();
  if (q < 0 || tab == nullptr) return z;
  const unsigned long long uq = static_cast<unsigned long long>(q), h = mix64(uq), idx = h & mask;
  const uint32_t f = fp_of(h);
  for (int k = (int)(idx & 7); k < 8; ++k) {
    const uint32_t b = fp_byte(w, k);
    if (b == 0) return z;
    if (b == f) {
      const unsigned long long at = (idx & ~7ull) + k;
      const uint4 s = ldg_slot(tab + at);
      if (slot_key(s) == uq) return s;
      return probe_fp_from(tab, fp, mask, uq, f, (at + 1) & mask, st);
    }
  }
  return probe_fp_from(tab, fp, mask, uq, f, ((idx & ~7ull) + 8) & mask, st);
}

// Dense PMI tensor for one (request, step t): T[i, j, l] = PMI(a_i, b_j, c_l)
// with a = E[t+1], b = E[t+2] = ids[t], c = ids[t+1] and E = [pre1; root; ids]
// (tree_ops.py:56-62, order 3).  256 threads: phase 1 resolves the 256
// context pairs (a_i, b_j) and 256 bigram pairs (b_j, c_l) in the pair table
// into shared memory; phase 2 resolves the 16 x 16 x 16 triples, 16 per
// thread with every first fingerprint load in flight, and writes T coalesced.
// At t = 0 every a_i is the root: one row of triples is probed and written 16
// times.
constexpr int kM = 16;

__global__ void __launch_bounds__(256, 3) pmi_dense_kernel(TableView t, int S, const int32_t* __restrict__ ids,
                                                        const int64_t* __restrict__ root,
                                                        const int64_t* __restrict__ pre1, float* __restrict__ T,
                                                        int32_t* st) {
  pdl_wait();   // ids (and root / pre1) may come from the preceding kernel
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
  const uint64_t pol = l2_evict_last_policy();
  {
    // context pair (a_i, b_j) and bigram pair (b_j, c_l), one each per thread
    int i = tid >> 4, j = tid & 15;
    long long a = sa[i], b = sb[j];
    long long qctx = (a >= 0 && b >= 0 && t.has_ctx) ? a * V + b : -1;
    int jj = tid >> 4, l = tid & 15;
    long long b2 = sb[jj], c2 = sc[l];
    long long qbig = b2 * V + c2;
    const uint2 w1 = fp_round1(t.pair_fp, t.pair_mask, qctx, pol);
    const uint2 w2 = fp_round1(t.pair_fp, t.pair_mask, qbig, pol);
    float pnc = pn_at(t, c2, st);
    float prevb = prev_at(t, b2, st);
    const uint4 s1 = fp_round2(t.pair, t.pair_fp, t.pair_mask, qctx, w1, st);
    const uint4 s2 = fp_round2(t.pair, t.pair_fp, t.pair_mask, qbig, w2, st);
    s_nab[tid] = __uint_as_float(s1.w);
    s_p2[tid] = p2_from(__uint_as_float(s2.z), prevb, pnc, t.beta2);
    if (jj == 0) s_lpn[l] = logf(pnc);
  }
  __syncthreads();
  float* Tout = T + ((int64_t)req * (S - 1) + tstep) * (kM * kM * kM);
  const int rows = tstep == 0 ? 1 : 16;       // row r of this thread's triples is i = r
  // two rounds of 8 probes per thread (every first fingerprint load of a round
  // in flight): 8 rather than 16 keeps the kernel at three CTAs per SM
  float v0 = 0.f;
#pragma unroll
  for (int r0 = 0; r0 < 16; r0 += 8) {
    long long q[8];
    uint2 w[8];
#pragma unroll
    for (int rr = 0; rr < 8; ++rr) {
      const int r = r0 + rr;
      int e = tid + 256 * r;
      int i = e >> 8, j = (e >> 4) & 15, l = e & 15;
      long long a = sa[i], b = sb[j];
      q[rr] = (r < rows && a >= 0 && b >= 0 && t.has_trip) ? (a * V + b) * V + sc[l] : -1;
      w[rr] = fp_round1(t.trip_fp, t.trip_mask, q[rr], pol);
    }
#pragma unroll
    for (int rr = 0; rr < 8; ++rr) {
      const int r = r0 + rr;
      int e = tid + 256 * r;
      int i = e >> 8, j = (e >> 4) & 15, l = e & 15;
      float v;
      if (r < rows) {
        const uint4 hit = fp_round2(t.trip, t.trip_fp, t.trip_mask, q[rr], w[rr], st);
        const float p3 = p3_from(__uint_as_float(hit.z), s_nab[i * 16 + j], s_p2[j * 16 + l], t.beta3);
        v = pmi_from(p3, s_lpn[l], t.clip);
        if (r == 0) v0 = v;
      } else {
        v = v0;   // t = 0: row i equals row 0
      }
      Tout[e] = v;
    }
  }
}

// Order 2: T[j, l] = PMI2(b_j, c_l), b = ids[t], c = ids[t+1]
// (tree_ops.py:59-60); one thread per entry.
__global__ void __launch_bounds__(256) pmi_dense2_kernel(TableView t, int S, const int32_t* __restrict__ ids,
                                                         float* __restrict__ T, int32_t* st) {
  pdl_wait();   // ids may come from the preceding kernel
  const int tstep = blockIdx.x, req = blockIdx.y, tid = threadIdx.x;
  const int32_t* idr = ids + (int64_t)req * S * kM;
  const long long b = idr[tstep * kM + (tid >> 4)], c = idr[(tstep + 1) * kM + (tid & 15)];
  const uint64_t pol = l2_evict_last_policy();
  const long long q = b * t.V + c;
  const uint2 w = fp_round1(t.pair_fp, t.pair_mask, q, pol);
  const float pnc = pn_at(t, c, st), prevb = prev_at(t, b, st);
  const uint4 s = fp_round2(t.pair, t.pair_fp, t.pair_mask, q, w, st);
  const float p2 = p2_from(__uint_as_float(s.z), prevb, pnc, t.beta2);
  T[((int64_t)req * (S - 1) + tstep) * (kM * kM) + tid] = pmi_from(p2, logf(pnc), t.clip);
}

// Order 4: T[h, j, k, l] = PMI4(z_h, a_j, b_k, c_l) with z = E[t], a = E[t+1],
// b = ids[t], c = ids[t+1] and E = [pre1; root; ids] (tree_ops.py:63-64).
// 512 threads per (request, step) in three phases, each with its shared
// inputs resolved once:
//   1. the 256 context pairs (a_j, b_k) and 256 bigrams (b_k, c_l);
//   2. the 16^3 trigrams (a_j, b_k, c_l) -> p3, and the 16^3 context
//      trigrams (z_h, a_j, b_k) -> rank i3 in keys3 (-1: absent) and
//      n4 = n4c[i3] (ngram_gpu.py:57-58);
//   3. the 16^4 quadgrams (i3, c_l), 16 probes in flight per thread, then
//      T written coalesced.
// At t = 0 (z, a constant) and t = 1 (z constant) phase 2 resolves only the
// distinct rows; phase 3 reads them through the collapsed indices.
constexpr int kP4Threads = 512;
struct P4Smem {
  long long sz[kM], sa[kM], sb[kM], sc[kM];
  float nab[kM * kM], p2[kM * kM], lpn[kM];
  float p3[kM * kM * kM];
  float n4[kM * kM * kM];
  int i3[kM * kM * kM];
};

__global__ void __launch_bounds__(kP4Threads, 2) pmi_dense4_kernel(TableView t, int S, const int32_t* __restrict__ ids,
                                                                const int64_t* __restrict__ root,
                                                                const int64_t* __restrict__ pre1,
                                                                float* __restrict__ T, int32_t* st) {
  extern __shared__ __align__(16) unsigned char p4_raw[];
  P4Smem& sm = *reinterpret_cast<P4Smem*>(p4_raw);
  pdl_wait();   // ids (and root / pre1) may come from the preceding kernel
  const int tstep = blockIdx.x, req = blockIdx.y, tid = threadIdx.x;
  const int32_t* idr = ids + (int64_t)req * S * kM;
  if (tid < kM) {
    sm.sz[tid] = tstep == 0 ? (long long)pre1[req]
                            : (tstep == 1 ? (long long)root[req] : (long long)idr[(tstep - 2) * kM + tid]);
    sm.sa[tid] = tstep == 0 ? (long long)root[req] : (long long)idr[(tstep - 1) * kM + tid];
    sm.sb[tid] = idr[tstep * kM + tid];
    sm.sc[tid] = idr[(tstep + 1) * kM + tid];
  }
  __syncthreads();
  const long long V = t.V;
  const uint64_t pol = l2_evict_last_policy();
  // distinct rows: a_j varies from t = 1 on, z_h from t = 2 on
  const int ja = tstep >= 1 ? 16 : 1, hz = tstep >= 2 ? 16 : 1;
  {  // phase 1: threads 0-255 the context pair (a_j, b_k), 256-511 the bigram (b_k, c_l)
    const int x = tid & 255, hi = x >> 4, lo = x & 15;
    long long q;
    float pnc = 0.f, prevb = 0.f;
    if (tid < 256) {
      const long long a = sm.sa[hi], b = sm.sb[lo];
      q = (a >= 0 && b >= 0 && t.has_ctx) ? a * V + b : -1;
    } else {
      const long long b = sm.sb[hi], c = sm.sc[lo];
      q = b * V + c;
      pnc = pn_at(t, c, st);
      prevb = prev_at(t, b, st);
    }
    const uint2 w = fp_round1(t.pair_fp, t.pair_mask, q, pol);
    const uint4 s = fp_round2(t.pair, t.pair_fp, t.pair_mask, q, w, st);
    if (tid < 256) {
      sm.nab[x] = __uint_as_float(s.w);
    } else {
      sm.p2[x] = p2_from(__uint_as_float(s.z), prevb, pnc, t.beta2);
      if (hi == 0) sm.lpn[lo] = logf(pnc);
    }
  }
  __syncthreads();
  {  // phase 2: 8 trigram probes, then 8 context-trigram probes per thread
#pragma unroll 1
    for (int half = 0; half < 2; ++half) {
      long long q[8];
      uint2 w[8];
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const int e = tid + kP4Threads * r;  // 0 .. 4095
        const int hi = e >> 8, mid = (e >> 4) & 15, lo = e & 15;
        if (half == 0) {  // (a_hi, b_mid, c_lo)
          const long long a = sm.sa[hi], b = sm.sb[mid];
          q[r] = (hi < ja && a >= 0 && b >= 0 && t.has_trip) ? (a * V + b) * V + sm.sc[lo] : -1;
        } else {          // (z_hi, a_mid, b_lo)
          const long long z = sm.sz[hi], a = sm.sa[mid], b = sm.sb[lo];
          q[r] = (hi < hz && mid < ja && z >= 0 && a >= 0 && b >= 0 && t.has_trip) ? (z * V + a) * V + b : -1;
        }
        w[r] = fp_round1(t.trip_fp, t.trip_mask, q[r], pol);
      }
#pragma unroll
      for (int r = 0; r < 8; ++r) {
        const int e = tid + kP4Threads * r;
        const int hi = e >> 8, mid = (e >> 4) & 15, lo = e & 15;
        const uint4 s = fp_round2(t.trip, t.trip_fp, t.trip_mask, q[r], w[r], st);
        if (half == 0) {
          if (hi < ja) sm.p3[e] = p3_from(__uint_as_float(s.z), sm.nab[hi * 16 + mid], sm.p2[mid * 16 + lo], t.beta3);
        } else if (hi < hz && mid < ja) {
          const bool hit = q[r] >= 0 && slot_key(s) == static_cast<unsigned long long>(q[r]);
          const int i3 = hit ? (int)s.w : -1;
          sm.i3[e] = i3;
          sm.n4[e] = (hit && t.has_quad) ? __ldg(t.n4c + i3) : 0.f;
        }
      }
    }
  }
  __syncthreads();
  float* Tout = T + ((int64_t)req * (S - 1) + tstep) * (kM * kM * kM * kM);
  const int hmask = hz > 1 ? 15 : 0, jmask = ja > 1 ? 15 : 0;
  // phase 3: 128 quadgrams per thread in batches of 8 (two CTAs per SM)
  for (int r0 = 0; r0 < 128; r0 += 8) {
    long long q[8];
    uint2 w[8];
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int e = tid + kP4Threads * (r0 + r);
      const int h = (e >> 12) & hmask, j = (e >> 8) & jmask, k = (e >> 4) & 15, l = e & 15;
      const int i3 = sm.i3[(h * 16 + j) * 16 + k];
      q[r] = (i3 >= 0 && t.has_quad) ? (long long)i3 * V + sm.sc[l] : -1;
      w[r] = fp_round1(t.quad_fp, t.quad_mask, q[r], pol);
    }
#pragma unroll
    for (int r = 0; r < 8; ++r) {
      const int e = tid + kP4Threads * (r0 + r);
      const int h = (e >> 12) & hmask, j = (e >> 8) & jmask, k = (e >> 4) & 15, l = e & 15;
      const uint4 s = fp_round2(t.quad, t.quad_fp, t.quad_mask, q[r], w[r], st);
      const float p4 = p4_from(__uint_as_float(s.z), sm.n4[(h * 16 + j) * 16 + k], sm.p3[(j * 16 + k) * 16 + l],
                               t.beta4);
      Tout[e] = pmi_from(p4, sm.lpn[l], t.clip);
    }
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
  dim3 grid(p->S - 1, p->B);
  const int order = dft::pmi_order_of(p);
  if (order == 2) {
    // programmatic launches: set up while the score kernel drains
    if (launch_pdl(pmi_dense2_kernel, grid, dim3(256), 0, st, table->view, p->S, ids, T, dev_status) != DFT_OK)
      return DFT_ERR_CUDA;
  } else if (order == 3) {
    if (launch_pdl(pmi_dense_kernel, grid, dim3(256), 0, st, table->view, p->S, ids, root, pre1, T, dev_status) !=
        DFT_OK)
      return DFT_ERR_CUDA;
  } else {
    if (!pre1) return DFT_ERR_INVALID;   // E[0] = pre1 is order 4's first context token
    static_assert(sizeof(P4Smem) <= 227 * 1024, "order-4 PMI shared memory");
    if (cudaFuncSetAttribute(pmi_dense4_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sizeof(P4Smem)) !=
        cudaSuccess)
      return DFT_ERR_CUDA;
    if (launch_pdl(pmi_dense4_kernel, grid, dim3(kP4Threads), sizeof(P4Smem), st, table->view, p->S, ids, root, pre1,
                   T, dev_status) != DFT_OK)
      return DFT_ERR_CUDA;
  }
  DFT_LAUNCH_CHECK();
  return DFT_OK;
}

extern "C" int dft_pmi_dense(const dft_table* table, const dft_build_params* p, const int32_t* ids,
                             const int64_t* root, const int64_t* pre1, float* T, int32_t* dev_status, void* stream) {
  if (!table || !p || !ids || !root || !T) return DFT_ERR_INVALID;
  if (p->M != kM) return DFT_ERR_UNSUPPORTED;
  if (p->B <= 0 || p->S < 2 || p->B > 65535) return DFT_ERR_INVALID;
  if (p->pmi_order != 0 && (p->pmi_order < 2 || p->pmi_order > 4)) return DFT_ERR_INVALID;
  if (dft::pmi_order_of(p) == 4 && !pre1) return DFT_ERR_INVALID;
  return dft_pmi_dense_launch(table, p, ids, root, pre1, T, dev_status, reinterpret_cast<cudaStream_t>(stream));
}
