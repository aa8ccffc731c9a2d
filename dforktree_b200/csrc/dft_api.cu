// C-ABI glue: status strings, version, and the composite score+build call
// (Builder.run, fc1_builder.py:26-47) = score -> dense PMI -> beam/tree.
#include "dft_common.cuh"

int dft_score_launch(const dft_build_params* p, const void* logits, int32_t dtype, int64_t ld_b, int64_t ld_s,
                     float* lp, int32_t* ids, float* rest, cudaStream_t st);
int dft_beam_launch(const dft_build_params* p, const float* lp, const int32_t* ids, const float* rest, const float* T,
                    const float* logc, const float* c0, const int64_t* root, const dft_tree_out* out,
                    int32_t* dev_status, cudaStream_t st);
int dft_check_build_params(const dft_build_params* p);

extern "C" const char* dft_status_string(int s) {
  switch (s) {
    case DFT_OK: return "ok";
    case DFT_ERR_INVALID: return "invalid argument";
    case DFT_ERR_UNSUPPORTED: return "unsupported shape";
    case DFT_ERR_CUDA: return "CUDA runtime error";
    case DFT_ERR_TABLE: return "n-gram table keys unsorted, negative or table full";
    case DFT_ERR_NO_DEVICE: return "no sm_100 device";
    case DFT_ERR_CAPACITY: return "shape exceeds the static scratch of dft_score_build_static (32 MiB)";
    case DFT_ERR_IO: return "table file missing, unwritable, truncated or damaged";
    default: return "unknown status";
  }
}

extern "C" int dft_version(void) { return 10000; }

extern "C" int64_t dft_score_build_workspace_bytes(const dft_build_params* p) {
  if (dft_check_build_params(p)) return -1;
  return dft::build_scratch_layout(p).total;
}

int dft_pmi_dense_launch(const dft_table* table, const dft_build_params* p, const int32_t* ids, const int64_t* root,
                         const int64_t* pre1, float* T, int32_t* dev_status, cudaStream_t st);

extern "C" int dft_score_build(const dft_table* table, const dft_build_params* p, const void* logits,
                               int32_t logits_dtype, int64_t ld_b, int64_t ld_s, const int64_t* root,
                               const int64_t* pre1, void* workspace, dft_tree_out* out, int32_t* dev_status,
                               void* stream) {
  int rc = dft_check_build_params(p);
  if (rc) return rc;
  if (!logits || !root || !workspace || !out) return DFT_ERR_INVALID;
  if (p->use_ngram && !table) return DFT_ERR_INVALID;
  if (p->use_ngram && dft::pmi_order_of(p) == 4 && !pre1) return DFT_ERR_INVALID;
  if (!dft::valid_dtype(logits_dtype)) return DFT_ERR_INVALID;
  if (ld_s < p->V || ld_b < (int64_t)p->S * ld_s - (ld_s - p->V)) return DFT_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const dft::BuildScratch w = dft::build_scratch_layout(p);
  char* ws = reinterpret_cast<char*>(workspace);
  float* lp = reinterpret_cast<float*>(ws + w.lp);
  int32_t* ids = reinterpret_cast<int32_t*>(ws + w.ids);
  float* rest = reinterpret_cast<float*>(ws + w.rest);
  float* T = p->use_ngram ? reinterpret_cast<float*>(ws + w.T) : nullptr;
  rc = dft_score_launch(p, logits, logits_dtype, ld_b, ld_s, lp, ids, rest, st);
  if (rc) return rc;
  if (p->use_ngram && p->S > 1) {
    rc = dft_pmi_dense_launch(table, p, ids, root, pre1, T, dev_status, st);
    if (rc) return rc;
  }
  return dft_beam_launch(p, lp, ids, rest, T, nullptr, nullptr, root, out, dev_status, st);
}
