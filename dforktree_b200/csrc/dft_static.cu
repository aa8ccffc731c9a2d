// dft_score_build_static: score + build without a caller-supplied workspace.
//
// For callers that cannot allocate device memory: a plugin running inside a
// serving engine's decode step, where HBM is owned by the engine's static
// pools and torch's caching allocator (a raw cudaMalloc competes with pools
// sized to fill the device, and cudaFree synchronises it), and C hosts that
// bind only this ABI and have no device allocator of their own.  The scratch
// that dft_score_build takes as `workspace` (drafter lp / ids / rest and the
// dense PMI tensor T) lives here in one file-scope device array of fixed size,
// held by every GPU that loads the library until the process exits.
#include "dft_common.cuh"
#include "dft_ctx.cuh"

#include <cuda.h>

#include <mutex>

int dft_score_launch(const dft_build_params* p, const void* logits, int32_t dtype, int64_t ld_b, int64_t ld_s,
                     float* lp, int32_t* ids, float* rest, cudaStream_t st);
int dft_beam_launch(const dft_build_params* p, const float* lp, const int32_t* ids, const float* rest, const float* T,
                    const float* logc, const float* c0, const int64_t* root, const dft_tree_out* out,
                    int32_t* dev_status, cudaStream_t st);
int dft_pmi_dense_launch(const dft_table* table, const dft_build_params* p, const int32_t* ids, const int64_t* root,
                         const int64_t* pre1, float* T, int32_t* dev_status, cudaStream_t st);
int dft_check_build_params(const dft_build_params* p);

namespace {

// 32 MiB: 64 requests at S = 24 need 24.3 MB (lp, ids, rest and the dense
// order-3 PMI tensor T of 23 x 16^3 floats per request; order 4 needs 16x that).
constexpr int64_t kStaticScratchBytes = 32ll << 20;
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_score_build_scratch[kStaticScratchBytes];

std::mutex g_mu;
void* g_scratch_ptr[kMaxDevices] = {};
CUcontext g_scratch_ctx[kMaxDevices] = {};

// Device address of the scratch array for the current device, resolved with
// that device current the first time the device is used (host code cannot use
// the symbol's name as a device pointer).  The address belongs to the device's
// current context: if that context changed since (cudaDeviceReset, a reset of
// the primary context), it is resolved again in the new one.
int scratch_for_current_device(void** out) {
  int dev = -1;
  CUcontext ctx = nullptr;
  if (!dft::current_device_context(&dev, &ctx)) return dev < 0 ? DFT_ERR_NO_DEVICE : DFT_ERR_CUDA;
  if (dev >= kMaxDevices) return DFT_ERR_UNSUPPORTED;
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[dev] || g_scratch_ctx[dev] != ctx) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_score_build_scratch) != cudaSuccess || !ptr) return DFT_ERR_CUDA;
    g_scratch_ptr[dev] = ptr;
    g_scratch_ctx[dev] = ctx;
  }
  *out = g_scratch_ptr[dev];
  return DFT_OK;
}

}  // namespace

extern "C" int64_t dft_score_build_static_capacity(void) { return kStaticScratchBytes; }

extern "C" int dft_score_build_static(const dft_table* table, const dft_build_params* p, const void* logits,
                                      int32_t logits_dtype, int64_t ld_b, int64_t ld_s, const int64_t* root,
                                      const int64_t* pre1, dft_tree_out* out, int32_t* dev_status, void* stream) {
  int rc = dft_check_build_params(p);
  if (rc) return rc;
  if (!logits || !root || !out) return DFT_ERR_INVALID;
  if (p->use_ngram && !table) return DFT_ERR_INVALID;
  if (p->use_ngram && dft::pmi_order_of(p) == 4 && !pre1) return DFT_ERR_INVALID;
  if (!dft::valid_dtype(logits_dtype)) return DFT_ERR_INVALID;
  if (ld_s < p->V || ld_b < (int64_t)p->S * ld_s - (ld_s - p->V)) return DFT_ERR_INVALID;
  // the same scratch layout as dft_score_build's workspace
  const dft::BuildScratch w = dft::build_scratch_layout(p);
  if (w.total > kStaticScratchBytes) return DFT_ERR_CAPACITY;
  void* base = nullptr;
  rc = scratch_for_current_device(&base);
  if (rc) return rc;
  char* ws = reinterpret_cast<char*>(base);
  float* lp = reinterpret_cast<float*>(ws + w.lp);
  int32_t* ids = reinterpret_cast<int32_t*>(ws + w.ids);
  float* rest = reinterpret_cast<float*>(ws + w.rest);
  float* T = p->use_ngram ? reinterpret_cast<float*>(ws + w.T) : nullptr;
  // every scratch byte read below is written earlier in the same call (score
  // writes all lp / ids / rest rows, the PMI kernel all of T): nothing needs
  // clearing between calls
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  rc = dft_score_launch(p, logits, logits_dtype, ld_b, ld_s, lp, ids, rest, st);
  if (rc) return rc;
  if (p->use_ngram && p->S > 1) {
    rc = dft_pmi_dense_launch(table, p, ids, root, pre1, T, dev_status, st);
    if (rc) return rc;
  }
  return dft_beam_launch(p, lp, ids, rest, T, nullptr, nullptr, root, out, dev_status, st);
}
