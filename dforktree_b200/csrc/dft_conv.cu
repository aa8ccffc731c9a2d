// Tree-aware causal depthwise conv (fc1_conv.py:8-27, tree_kernels.py:17-33).
// Reference: fc1_conv.conv (fc1_conv.py:8-27) and tree_kernels._tree_conv_kernel
// (tree_kernels.py:17-33): y[n, c] = SiLU(sum_j w[c, j] * x_j + bias[c]) where
// tap j reads conv column cidx[n, j] -- columns 0..2 are the conv state, 3+m
// is new token m -- and taps 1..3 are written as the node's conv window.
// Batched over requests; one thread per (request, node, channel), channels
// fastest so every load and store is coalesced.
#include "dft_common.cuh"

#include <cstring>

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

// Packed form for bf16 states in the [.., C, 3] layout and bf16 inputs: one
// thread per 8 channels reads their 48-byte state block and the 16-byte input
// rows its taps name, and writes the 48-byte block back (all accesses 16-byte).
__global__ void conv_commit_packed_kernel(dft_conv_commit_args a, int32_t* st) {
  const int c0 = (blockIdx.x * blockDim.x + threadIdx.x) * 8;
  const int b = blockIdx.y, l = blockIdx.z;
  if (c0 >= a.C) return;
  const int64_t u = a.last[b];
  if (u < 0) return;
  if (u >= a.N) {
    if (c0 == 0) raise_status(st, DFT_DEV_BAD_INDEX);
    return;
  }
  const int64_t slot = a.slots ? a.slots[b] : b;
  uint4* sp = reinterpret_cast<uint4*>(static_cast<uint16_t*>(a.conv_state) + (int64_t)l * a.cs_sl + slot * a.cs_ss +
                                       (int64_t)c0 * 3);
  const uint4 o0 = sp[0], o1 = sp[1], o2 = sp[2];
  uint16_t old[24], out[24];
  memcpy(old, &o0, 16);
  memcpy(old + 8, &o1, 16);
  memcpy(old + 16, &o2, 16);
#pragma unroll
  for (int j = 0; j < 3; ++j) {
    const int64_t col = a.cidx[((int64_t)b * a.N + u) * 4 + j + 1];
    if (col < 0 || col >= 3 + a.N) {
      raise_status(st, DFT_DEV_BAD_INDEX);
      return;
    }
    if (col < 3) {
#pragma unroll
      for (int e = 0; e < 8; ++e)  // register selects, no indexing by a runtime column
        out[3 * e + j] = col == 0 ? old[3 * e] : (col == 1 ? old[3 * e + 1] : old[3 * e + 2]);
    } else {
      const uint4 xv = *reinterpret_cast<const uint4*>(static_cast<const uint16_t*>(a.x) + (int64_t)l * a.x_sl +
                                                       (int64_t)b * a.x_sb + (col - 3) * a.x_sn + c0);
      uint16_t xr[8];
      memcpy(xr, &xv, 16);
#pragma unroll
      for (int e = 0; e < 8; ++e) out[3 * e + j] = xr[e];
    }
  }
  uint4 n0, n1, n2;
  memcpy(&n0, out, 16);
  memcpy(&n1, out + 8, 16);
  memcpy(&n2, out + 16, 16);
  sp[0] = n0;
  sp[1] = n1;
  sp[2] = n2;
}

}  // namespace

extern "C" int dft_conv_commit(const dft_conv_commit_args* a, int32_t* dev_status, void* stream) {
  if (!a || !a->x || !a->conv_state || !a->cidx || !a->last) return DFT_ERR_INVALID;
  if (a->L <= 0 || a->B <= 0 || a->N <= 0 || a->C <= 0 || a->B > 65535 || a->L > 65535) return DFT_ERR_INVALID;
  if (!valid_dtype(a->x_dtype) || !valid_dtype(a->cs_dtype)) return DFT_ERR_INVALID;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  const bool packed = a->cs_dtype == DFT_BF16 && a->x_dtype == DFT_BF16 && a->cs_st == 1 && a->cs_sc == 3 &&
                      a->C % 8 == 0 && ((uintptr_t)a->conv_state & 15) == 0 && ((uintptr_t)a->x & 15) == 0 &&
                      a->cs_sl % 8 == 0 && a->cs_ss % 8 == 0 && a->x_sl % 8 == 0 && a->x_sb % 8 == 0 &&
                      a->x_sn % 8 == 0;
  if (packed) {
    dim3 grid((a->C / 8 + 255) / 256, a->B, a->L);
    conv_commit_packed_kernel<<<grid, 256, 0, st>>>(*a, dev_status);
  } else {
    dim3 grid((a->C + 255) / 256, a->B, a->L);
    conv_commit_kernel<<<grid, 256, 0, st>>>(*a, dev_status);
  }
  DFT_LAUNCH_CHECK();
  return DFT_OK;
}
