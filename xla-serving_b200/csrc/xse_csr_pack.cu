// Packing of CSR slices for the table-wise ids all-to-all
// (include/xse_shard.h): per segment, the id range [offsets[0],
// offsets[num_bags]) (and its weights) is copied to the destination chunk
// and the offsets are rebased into it. HBM-bound copies: each element is
// read and written once, with consecutive threads on consecutive elements.

#include <cuda_runtime.h>
#include <stdint.h>

#include "xse_internal.h"
#include "../../include/xse_emb.h"
#include "../../include/xse_shard.h"

namespace xse {
namespace {

constexpr int kPackThreads = 256;
constexpr int kMaxSegments = 128;  // per launch (parameter space)
constexpr int kChunksPerSegment = 32;  // blocks per segment (grid x)

struct PackParams {
  int32_t n;
  int32_t reserved;
  xse_csr_segment s[kMaxSegments];
};

__device__ __forceinline__ int64_t Idx(const void* base, int32_t type,
                                       int64_t i) {
  return type == XSE_INDEX_I64
             ? static_cast<const long long*>(base)[i]
             : static_cast<int64_t>(static_cast<const int*>(base)[i]);
}

// The segment's id range, or false when it is not within [0, num_ids).
__device__ __forceinline__ bool Range(const xse_csr_segment& g, int64_t* lo,
                                      int64_t* hi) {
  *lo = Idx(g.offsets, g.offsets_type, 0);
  *hi = Idx(g.offsets, g.offsets_type, g.num_bags);
  return *lo >= 0 && *hi >= *lo && *hi <= g.num_ids;
}

__global__ void ExtentsKernel(const __grid_constant__ PackParams p,
                              int64_t* __restrict__ extents) {
  const int k = blockIdx.x * blockDim.x + threadIdx.x;
  if (k >= p.n) return;
  int64_t lo, hi;
  extents[k] = Range(p.s[k], &lo, &hi) ? hi - lo : -1;
}

__global__ void __launch_bounds__(kPackThreads)
    PackKernel(const __grid_constant__ PackParams p) {
  const xse_csr_segment& g = p.s[blockIdx.y];
  int64_t lo, hi;
  if (!Range(g, &lo, &hi)) return;
  const int64_t step = static_cast<int64_t>(gridDim.x) * kPackThreads;
  const int64_t first =
      static_cast<int64_t>(blockIdx.x) * kPackThreads + threadIdx.x;
  for (int64_t i = first; i <= g.num_bags; i += step) {
    g.dst_offsets[i] = Idx(g.offsets, g.offsets_type, i) - lo + g.dst_base;
  }
  const int64_t count = hi - lo;
  if (count > 0 && g.dst_ids == nullptr) return;  // nowhere to put the ids
  if (g.ids_type == XSE_INDEX_I64) {
    const long long* src = static_cast<const long long*>(g.ids) + lo;
    long long* dst = static_cast<long long*>(g.dst_ids);
    for (int64_t i = first; i < count; i += step) dst[i] = src[i];
  } else {
    const int* src = static_cast<const int*>(g.ids) + lo;
    int* dst = static_cast<int*>(g.dst_ids);
    for (int64_t i = first; i < count; i += step) dst[i] = src[i];
  }
  if (g.weights != nullptr && g.dst_weights != nullptr) {
    for (int64_t i = first; i < count; i += step) {
      g.dst_weights[i] = g.weights[lo + i];
    }
  }
}

}  // namespace
}  // namespace xse

extern "C" {

int xse_csr_extents(const xse_csr_segment* segs, int32_t n, int64_t* extents,
                    void* stream) {
  if (n < 0 || (n > 0 && (segs == nullptr || extents == nullptr))) {
    xse::SetLastErrorMessage("segments and extents must be non-null");
    return XSE_INVALID_ARGUMENT;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int32_t base = 0; base < n; base += xse::kMaxSegments) {
    xse::PackParams p{};
    p.n = n - base < xse::kMaxSegments ? n - base : xse::kMaxSegments;
    for (int k = 0; k < p.n; ++k) p.s[k] = segs[base + k];
    xse::ExtentsKernel<<<1, xse::kMaxSegments, 0, s>>>(p, extents + base);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
      xse::SetLastErrorMessage(cudaGetErrorString(e));
      return XSE_INTERNAL;
    }
  }
  xse::SetLastErrorMessage("");
  return XSE_OK;
}

int xse_csr_pack(const xse_csr_segment* segs, int32_t n, void* stream) {
  if (n < 0 || (n > 0 && segs == nullptr)) {
    xse::SetLastErrorMessage("segments must be non-null");
    return XSE_INVALID_ARGUMENT;
  }
  for (int32_t k = 0; k < n; ++k) {
    if (segs[k].num_bags < 0 || segs[k].offsets == nullptr ||
        segs[k].dst_offsets == nullptr ||
        (segs[k].num_ids > 0 && segs[k].ids == nullptr) ||
        (segs[k].ids_type != XSE_INDEX_I32 &&
         segs[k].ids_type != XSE_INDEX_I64) ||
        (segs[k].offsets_type != XSE_INDEX_I32 &&
         segs[k].offsets_type != XSE_INDEX_I64)) {
      xse::SetLastErrorMessage("bad CSR segment");
      return XSE_INVALID_ARGUMENT;
    }
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int32_t base = 0; base < n; base += xse::kMaxSegments) {
    xse::PackParams p{};
    p.n = n - base < xse::kMaxSegments ? n - base : xse::kMaxSegments;
    for (int k = 0; k < p.n; ++k) p.s[k] = segs[base + k];
    xse::PackKernel<<<dim3(xse::kChunksPerSegment, p.n),
                      xse::kPackThreads, 0, s>>>(p);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
      xse::SetLastErrorMessage(cudaGetErrorString(e));
      return XSE_INTERNAL;
    }
  }
  xse::SetLastErrorMessage("");
  return XSE_OK;
}

}  // extern "C"
