// DLRM pairwise dot interaction for sm_100a (CUDA cores).
//
// No counterpart in the reference: its DLRM bundle feeds the pooled
// embeddings to a DCN-v2 tower (examples/dlrm/model_jce.py:141-164). This
// kernel computes the dot interaction that replaces it:
//   Z_b = [dense_b; pooled_b,0; ...; pooled_b,T-1]   ((T+1) x D)
//   out_b = [dense_b, Z_b[i] . Z_b[j] for 0 <= i < j <= T, row-major]
//
// Design: one warp per sample. Lane l holds columns [l*CPL, l*CPL+CPL) of
// every row of Z_b in registers (D = 32*CPL), loaded with coalesced 16-byte
// loads straight from HBM, so Z is read exactly once and shared memory is
// not needed. The pair loop is fully unrolled: each lane forms partial dots
// of 32 pairs, then a 31-shuffle reduce-scatter leaves the complete dot of
// pair (batch*32 + l) in lane l, which stores it (coalesced). HBM traffic per
// sample: (T+1)*D*4 bytes read, (D + P)*4 bytes written.

#include <cuda_runtime.h>
#include <stdint.h>

#include "xse_internal.h"

namespace xse {
namespace {

constexpr int kInteractionThreads = 128;

// Sums v[k] across the warp so that lane l ends with the total of v[l].
__device__ __forceinline__ float ReduceScatter32(float (&v)[32]) {
  const int lane = threadIdx.x & 31;
#pragma unroll
  for (int s = 16; s >= 1; s >>= 1) {
    const bool upper = (lane & s) != 0;
#pragma unroll
    for (int k = 0; k < s; ++k) {
      const float send = upper ? v[k] : v[k + s];
      const float keep = upper ? v[k + s] : v[k];
      v[k] = keep + __shfl_xor_sync(0xffffffffu, send, s);
    }
  }
  return v[0];
}

template <int R, int CPL>
__global__ void __launch_bounds__(kInteractionThreads)
    DotInteractionKernel(const float* __restrict__ dense,
                         int64_t dense_stride,
                         const float* __restrict__ pooled,
                         int64_t pooled_stride, int64_t batch,
                         float* __restrict__ out, int64_t out_stride) {
  constexpr int D = 32 * CPL;
  constexpr int P = R * (R - 1) / 2;
  constexpr int W = D + P;
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) *
                        (kInteractionThreads / 32);
  for (int64_t b = static_cast<int64_t>(blockIdx.x) *
                       (kInteractionThreads / 32) +
                   threadIdx.x / 32;
       b < batch; b += warps) {
    float z[R][CPL];
    const float* dense_row = dense + b * dense_stride + lane * CPL;
    const float* pooled_rows = pooled + b * pooled_stride + lane * CPL;
#pragma unroll
    for (int i = 0; i < R; ++i) {
      const float* src = i == 0 ? dense_row : pooled_rows + (i - 1) * D;
      if constexpr (CPL % 4 == 0) {
#pragma unroll
        for (int c = 0; c < CPL; c += 4) {
          const float4 x = __ldg(reinterpret_cast<const float4*>(src + c));
          z[i][c] = x.x;
          z[i][c + 1] = x.y;
          z[i][c + 2] = x.z;
          z[i][c + 3] = x.w;
        }
      } else {
#pragma unroll
        for (int c = 0; c < CPL; ++c) z[i][c] = __ldg(src + c);
      }
    }
    float* o = out + b * out_stride;
#pragma unroll
    for (int c = 0; c < CPL; ++c) o[lane * CPL + c] = z[0][c];
    for (int64_t c = W + lane; c < out_stride; c += 32) o[c] = 0.0f;

    float v[32];
    int q = 0;
#pragma unroll
    for (int i = 0; i < R; ++i) {
#pragma unroll
      for (int j = i + 1; j < R; ++j) {
        float s = 0.0f;
#pragma unroll
        for (int c = 0; c < CPL; ++c) s = fmaf(z[i][c], z[j][c], s);
        v[q & 31] = s;
        if ((q & 31) == 31 || q == P - 1) {
#pragma unroll
          for (int k = (q & 31) + 1; k < 32; ++k) v[k] = 0.0f;
          const float total = ReduceScatter32(v);
          const int pair = (q & ~31) + lane;
          if (pair < P) o[D + pair] = total;
        }
        ++q;
      }
    }
  }
}

// Any shape: one thread per output element of a sample, row order as above.
__global__ void DotInteractionGenericKernel(
    const float* __restrict__ dense, int64_t dense_stride,
    const float* __restrict__ pooled, int64_t pooled_stride, int64_t batch,
    int num_tables, int dim, float* __restrict__ out, int64_t out_stride) {
  const int rows = num_tables + 1;
  const int64_t pairs = static_cast<int64_t>(rows) * (rows - 1) / 2;
  const int64_t width = dim + pairs;
  const int64_t total = batch * out_stride;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       e < total; e += stride) {
    const int64_t b = e / out_stride;
    const int64_t k = e % out_stride;
    if (k >= width) {
      out[e] = 0.0f;
      continue;
    }
    if (k < dim) {
      out[e] = dense[b * dense_stride + k];
      continue;
    }
    // Decode pair index k - dim into (i, j), i < j, row-major.
    int64_t rem = k - dim;
    int i = 0;
    while (rem >= rows - 1 - i) {
      rem -= rows - 1 - i;
      ++i;
    }
    const int j = i + 1 + static_cast<int>(rem);
    const float* zi = i == 0 ? dense + b * dense_stride
                             : pooled + b * pooled_stride + (i - 1) * dim;
    const float* zj = pooled + b * pooled_stride + (j - 1) * dim;
    float s = 0.0f;
    for (int c = 0; c < dim; ++c) s = fmaf(zi[c], zj[c], s);
    out[e] = s;
  }
}

}  // namespace

cudaError_t LaunchDotInteraction(const float* dense, int64_t dense_stride,
                                 const float* pooled, int64_t pooled_stride,
                                 int64_t batch, int num_tables, int dim,
                                 float* out, int64_t out_stride,
                                 cudaStream_t stream) {
  if (batch <= 0) return cudaSuccess;
  const bool aligned =
      ((reinterpret_cast<uintptr_t>(dense) |
        reinterpret_cast<uintptr_t>(pooled)) & 15u) == 0 &&
      dense_stride % 4 == 0 && pooled_stride % 4 == 0;
  if (aligned && num_tables == 26 && dim == 128) {
    const int64_t warps_per_block = kInteractionThreads / 32;
    int64_t blocks = (batch + warps_per_block - 1) / warps_per_block;
    if (blocks > 148 * 64) blocks = 148 * 64;
    DotInteractionKernel<27, 4><<<static_cast<int>(blocks),
                                  kInteractionThreads, 0, stream>>>(
        dense, dense_stride, pooled, pooled_stride, batch, out, out_stride);
    return cudaGetLastError();
  }
  const int64_t total = batch * out_stride;
  int64_t blocks = (total + 255) / 256;
  if (blocks > 148 * 32) blocks = 148 * 32;
  DotInteractionGenericKernel<<<static_cast<int>(blocks), 256, 0, stream>>>(
      dense, dense_stride, pooled, pooled_stride, batch, num_tables, dim, out,
      out_stride);
  return cudaGetLastError();
}

}  // namespace xse
