// Tree-aware causal depthwise conv (fc1_conv.py:8-27, tree_kernels.py:17-33).
// Reference: fc1_conv.conv (fc1_conv.py:8-27) and tree_kernels._tree_conv_kernel
// (tree_kernels.py:17-33): y[n, c] = SiLU(sum_j w[c, j] * x_j + bias[c]) where
// tap j reads conv column cidx[n, j] -- columns 0..2 are the conv state, 3+m
// is new token m -- and taps 1..3 are written as the node's conv window.
// Batched over requests; one thread per (request, node, channel), channels
// fastest so every load and store is coalesced.
#include "dft_common.cuh"

using namespace dft;

namespace {

__global__ void tree_conv_kernel(dft_conv_args a, int32_t* st) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int n = blockIdx.y;
  const int b = blockIdx.z;
  if (c >= a.C) return;
  const int64_t slot = a.state_slots ? a.state_slots[b] : b;
  const int64_t dst = a.iw_slots ? a.iw_slots[b] : b;
  float acc = 0.f;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    int64_t col = a.cidx[((int64_t)b * a.N + n) * 4 + j];
    float v = 0.f;
    if (col < 0 || col >= 3 + a.N) {
      raise_status(st, DFT_DEV_BAD_INDEX);
    } else if (col < 3) {
      v = load_any(a.conv_state, a.cs_dtype, slot * a.cs_ss + (int64_t)c * a.cs_sc + col * a.cs_st);
    } else {
      v = load_any(a.x, a.x_dtype, (int64_t)b * a.x_sb + (col - 3) * a.x_sn + (int64_t)c * a.x_sc);
    }
    const float w = load_any(a.weight, a.w_dtype, (int64_t)c * 4 + j);
    acc = __fadd_rn(acc, __fmul_rn(v, w));  // fc1_conv.py:20 rounds the product and the sum
    if (j > 0 && a.iw)
      store_any(a.iw, a.iw_dtype, dst * a.iw_sd + (int64_t)n * a.iw_sn + (int64_t)c * a.iw_sc + (j - 1) * a.iw_sj, v);
  }
  if (a.bias) acc = __fadd_rn(acc, load_any(a.bias, a.w_dtype, c));
  // SiLU with the hardware exp2 / reciprocal (same arithmetic as the conv fused
  // into the tcgen05 verifier, so both produce identical y)
  const float y = silu_hw(acc);
  store_any(a.y, a.y_dtype, (int64_t)b * a.y_sb + (int64_t)n * a.y_sn + c, y);
}

}  // namespace

extern "C" int dft_tree_conv(const dft_conv_args* a, int32_t* dev_status, void* stream) {
  if (!a || !a->x || !a->conv_state || !a->weight || !a->cidx || !a->y) return DFT_ERR_INVALID;
  if (a->B <= 0 || a->N <= 0 || a->C <= 0 || a->B > 65535 || a->N > 65535) return DFT_ERR_INVALID;
  if (!valid_dtype(a->x_dtype) || !valid_dtype(a->cs_dtype) || !valid_dtype(a->w_dtype) ||
      !valid_dtype(a->y_dtype) || (a->iw && !valid_dtype(a->iw_dtype)))
    return DFT_ERR_INVALID;
  dim3 grid((a->C + 255) / 256, a->N, a->B);
  tree_conv_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(*a, dev_status);
  DFT_LAUNCH_CHECK();
  return DFT_OK;
}

// ------------------------------------------------------ conv-window commit --
// conv_state[l, slot(b), c, j] <- input at column cidx[b, u, j + 1], u = last[b]:
// the window of the last accepted node (fc1_conv.py:22-27 writes the same taps
// into intermediate_conv_window; SGLang's commit copies them into the state).
// One thread per (channel, request, layer); the three values are read before
// any is written, so the update is in place.
namespace {

__global__ void conv_commit_kernel(dft_conv_commit_args a, int32_t* st) {
  const int c = blockIdx.x * blockDim.x + threadIdx.x;
  const int b = blockIdx.y, l = blockIdx.z;
  if (c >= a.C) return;
  const int64_t u = a.last[b];
  if (u < 0) return;
  if (u >= a.N) {
    if (c == 0) raise_status(st, DFT_DEV_BAD_INDEX);
    return;
  }
  const int64_t slot = a.slots ? a.slots[b] : b;
  const int64_t sbase = (int64_t)l * a.cs_sl + slot * a.cs_ss + (int64_t)c * a.cs_sc;
  float v[3];
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int64_t col = a.cidx[((int64_t)b * a.N + u) * 4 + j + 1];
    if (col < 0 || col >= 3 + a.N) {
      raise_status(st, DFT_DEV_BAD_INDEX);
      return;
    }
    v[j] = col < 3 ? load_any(a.conv_state, a.cs_dtype, sbase + col * a.cs_st)
                   : load_any(a.x, a.x_dtype, (int64_t)l * a.x_sl + (int64_t)b * a.x_sb + (col - 3) * a.x_sn + c);
  }
#pragma unroll
  for (int j = 0; j < 3; ++j) store_any(a.conv_state, a.cs_dtype, sbase + j * a.cs_st, v[j]);
}

}  // namespace

extern "C" int dft_conv_commit(const dft_conv_commit_args* a, int32_t* dev_status, void* stream) {
  if (!a || !a->x || !a->conv_state || !a->cidx || !a->last) return DFT_ERR_INVALID;
  if (a->L <= 0 || a->B <= 0 || a->N <= 0 || a->C <= 0 || a->B > 65535 || a->L > 65535) return DFT_ERR_INVALID;
  if (!valid_dtype(a->x_dtype) || !valid_dtype(a->cs_dtype)) return DFT_ERR_INVALID;
  dim3 grid((a->C + 255) / 256, a->B, a->L);
  conv_commit_kernel<<<grid, 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(*a, dev_status);
  DFT_LAUNCH_CHECK();
  return DFT_OK;
}
