// Pooled embedding-bag kernels for sm_100a.
//
// Replaces the reference's CPU hot loop ReducePortable / BagScale
// (data/cpu_embedding/cc/embedding_bag.cc:146-194) and its group validation
// (embedding_bag.cc:89-144).
//
// Design: a group of G lanes owns one bag (G = 4..32, so a warp pools 32/G
// bags at once). Each lane owns V 16-byte column vectors of a row, so a row
// gather is G*V independent 16-byte loads. The ids (and weights) of a bag are
// loaded G at a time, one per lane, and broadcast through the group with
// shuffles; U rows are loaded before any of them is added, which keeps
// U*V loads in flight per lane while the adds still run in CSR order. Every
// element is accumulated in fp32 in exactly the reference's order
// (out = 0; out += row or out += w*row, one separately rounded multiply and
// add), so fp32 results are bit-identical to the reference semantics; mean and
// sqrt-n scales are applied as one multiply by a correctly rounded reciprocal.
//
// HBM traffic per id: one row (dim * elem bytes) + the id (4/8 B) + the weight
// if any; per bag: one offset and the fp32 output row.

#include <cuda_runtime.h>
#include <stdint.h>

#include "xse_internal.h"

namespace xse {
namespace {

constexpr int kThreads = 256;

template <int DT>
struct ElemsPerVec;
template <>
struct ElemsPerVec<0> {
  static constexpr int value = 4;  // fp32
};
template <>
struct ElemsPerVec<1> {
  static constexpr int value = 8;  // bf16
};
template <>
struct ElemsPerVec<2> {
  static constexpr int value = 16;  // int8
};

__device__ __forceinline__ int64_t LoadIndex(const void* base, int is64,
                                             int64_t i) {
  return is64 ? __ldg(static_cast<const long long*>(base) + i)
              : static_cast<int64_t>(__ldg(static_cast<const int*>(base) + i));
}

// Read-only 16-byte row load that does not allocate in L1 (rows are touched
// once per id; reuse of hot rows comes from L2).
__device__ __forceinline__ uint4 LoadRowVec(const uint4* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ float Bf16Lo(uint32_t w) {
  return __uint_as_float(w << 16);
}
__device__ __forceinline__ float Bf16Hi(uint32_t w) {
  return __uint_as_float(w & 0xffff0000u);
}
__device__ __forceinline__ float I8At(uint32_t w, int k) {
  // Sign-extend byte k of w.
  return __int2float_rn(static_cast<int>(w << (24 - 8 * k)) >> 24);
}

// Unpacks one 16-byte vector into EPV fp32 values (int8 rows dequantized as
// float(q)*scale + bias, each step rounded separately).
template <int DT>
__device__ __forceinline__ void Unpack(const uint4& r, float2 sb,
                                       float (&x)[ElemsPerVec<DT>::value]) {
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
  if constexpr (DT == 0) {
#pragma unroll
    for (int k = 0; k < 4; ++k) x[k] = __uint_as_float(w[k]);
  } else if constexpr (DT == 1) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      x[2 * k] = Bf16Lo(w[k]);
      x[2 * k + 1] = Bf16Hi(w[k]);
    }
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
#pragma unroll
      for (int b = 0; b < 4; ++b) {
        x[4 * k + b] = __fadd_rn(__fmul_rn(I8At(w[k], b), sb.x), sb.y);
      }
    }
  }
}

__device__ __forceinline__ void RecordError(DevStatus* st, int slot,
                                            unsigned int flag) {
  atomicOr(&st->req[slot].flags, flag);
  atomicOr(&st->group_error, 1u);
}

__device__ __forceinline__ void RecordBadId(DevStatus* st, int slot,
                                            int64_t index) {
  atomicMax(&st->req[slot].inv_min_bad_index,
            ~static_cast<unsigned long long>(index));
  RecordError(st, slot, kErrBadId);
}

// Bag scale (embedding_bag.cc:146-167), computed once per bag.
__device__ __forceinline__ float BagScale(int combine, bool weighted,
                                          int64_t n, float wsum) {
  const float denom = weighted ? wsum : __ll2float_rn(n);
  return combine == 2 ? __fdiv_rn(1.0f, denom)
                      : __fdiv_rn(1.0f, __fsqrt_rn(denom));
}

// Locates the descriptor of `task`; descriptors are ordered by task_begin and
// every group walks its tasks in increasing order, so the search only moves
// forward.
__device__ __forceinline__ int AdvanceDesc(const PoolParams& p, int t,
                                           int64_t task) {
  while (t + 1 < p.n && task >= p.d[t + 1].task_begin) ++t;
  return t;
}

// Offsets of bag `bag`, checked. Returns false when the bag must be skipped.
__device__ __forceinline__ bool BagRange(const PoolParams& p,
                                         const BagDesc& d, int64_t bag,
                                         int64_t* begin, int64_t* end) {
  *begin = LoadIndex(d.offsets, d.offs64, bag);
  *end = LoadIndex(d.offsets, d.offs64, bag + 1);
  const bool weights_short = d.weights != nullptr && *end > d.num_weights;
  const bool bad = *begin < 0 || *end < *begin || *end > d.num_ids ||
                   weights_short;
  if (bad && p.fused_checks) {
    unsigned int f = 0;
    if (*begin < 0 || *end < *begin) f |= kErrBadOffsets;
    if (*end > d.num_ids) f |= kErrLastExceedsIds;
    if (weights_short) f |= kErrLastExceedsWeights;
    RecordError(p.status, d.slot, f);
  }
  return !bad;
}

template <int DT, int G, int V>
__global__ void __launch_bounds__(kThreads)
    PoolVecKernel(const __grid_constant__ PoolParams p) {
  constexpr int EPV = ElemsPerVec<DT>::value;
  constexpr int U = V >= 8 ? 1 : 8 / V;
  constexpr int kGroupsPerBlock = kThreads / G;
  if (!p.fused_checks && p.status->group_error != 0) return;

  const int lane = threadIdx.x & 31;
  const int gl = lane % G;
  const unsigned gmask =
      G == 32 ? 0xffffffffu : (((1u << G) - 1u) << (lane - gl));
  const int64_t stride = static_cast<int64_t>(gridDim.x) * kGroupsPerBlock;
  int t = 0;
  for (int64_t task = static_cast<int64_t>(blockIdx.x) * kGroupsPerBlock +
                      threadIdx.x / G;
       task < p.total_tasks; task += stride) {
    t = AdvanceDesc(p, t, task);
    const BagDesc& d = p.d[t];
    const int64_t bag = task - d.task_begin;
    int64_t begin, end;
    if (!BagRange(p, d, bag, &begin, &end)) continue;

    const int row_vecs = d.dim / EPV;  // 16-byte vectors per row
    const bool weighted = d.weights != nullptr;
    const uint4* rows = static_cast<const uint4*>(d.rows);
    float acc[V][EPV];
#pragma unroll
    for (int v = 0; v < V; ++v)
#pragma unroll
      for (int e = 0; e < EPV; ++e) acc[v][e] = 0.0f;
    float wsum = 0.0f;

    for (int64_t base = begin; base < end; base += G) {
      const int cnt = static_cast<int>(end - base < G ? end - base : G);
      // Stage G ids (and weights) of the bag, one per lane. -1 marks an id
      // that contributes nothing (invalid, or outside this shard's window).
      int64_t my_row = -1;
      float my_w = 1.0f;
      if (gl < cnt) {
        const int64_t id = LoadIndex(d.ids, d.ids64, base + gl);
        if (weighted) my_w = __ldg(d.weights + base + gl);
        if (id < 0 || id >= d.vocab) {
          if (p.fused_checks) RecordBadId(p.status, d.slot, base + gl);
        } else if (id >= d.row_begin && id < d.row_end) {
          my_row = id - d.row_begin;
        }
      }
      for (int j0 = 0; j0 < cnt; j0 += U) {
        uint4 raw[U][V];
        float2 sb[U];
        int64_t row[U];
        float w[U];
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int j = j0 + u < cnt ? j0 + u : cnt - 1;
          row[u] = __shfl_sync(gmask, my_row, j, G);
          w[u] = __shfl_sync(gmask, my_w, j, G);
          if (j0 + u >= cnt) row[u] = -1;
          sb[u] = make_float2(0.0f, 0.0f);
          if constexpr (DT == 2) {
            if (row[u] >= 0) sb[u] = __ldg(d.scale_bias + row[u]);
          }
#pragma unroll
          for (int v = 0; v < V; ++v) {
            const int k = gl + v * G;
            if (row[u] >= 0 && k < row_vecs) {
              raw[u][v] = LoadRowVec(rows + row[u] * row_vecs + k);
            } else {
              raw[u][v] = make_uint4(0, 0, 0, 0);
            }
          }
        }
#pragma unroll
        for (int u = 0; u < U; ++u) {
          if (j0 + u < cnt) {
            if (weighted) {
              wsum = __fadd_rn(wsum, d.combine == 3 ? __fmul_rn(w[u], w[u])
                                                    : w[u]);
            }
            if (row[u] >= 0) {
#pragma unroll
              for (int v = 0; v < V; ++v) {
                float x[EPV];
                Unpack<DT>(raw[u][v], sb[u], x);
#pragma unroll
                for (int e = 0; e < EPV; ++e) {
                  acc[v][e] = weighted
                                  ? __fadd_rn(acc[v][e], __fmul_rn(w[u], x[e]))
                                  : __fadd_rn(acc[v][e], x[e]);
                }
              }
            }
          }
        }
      }
    }

    const int64_t n = end - begin;
    if (n > 0 && d.combine != 1) {
      const float s = BagScale(d.combine, weighted, n, wsum);
#pragma unroll
      for (int v = 0; v < V; ++v)
#pragma unroll
        for (int e = 0; e < EPV; ++e) acc[v][e] = __fmul_rn(acc[v][e], s);
    }
    float* out = d.out + bag * d.out_stride;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int k = gl + v * G;
      if (k < row_vecs) {
        float* o = out + k * EPV;
        if (d.vec_out) {
#pragma unroll
          for (int e = 0; e < EPV; e += 4) {
            *reinterpret_cast<float4*>(o + e) =
                make_float4(acc[v][e], acc[v][e + 1], acc[v][e + 2],
                            acc[v][e + 3]);
          }
        } else {
#pragma unroll
          for (int e = 0; e < EPV; ++e) o[e] = acc[v][e];
        }
      }
    }
  }
}

// Element-wise variant for rows that are not whole 16-byte vectors (odd
// dims or unaligned tables). A warp owns a bag; lanes own columns
// c = lane + 32*k, in column chunks of 32*kCols.
template <int DT>
__global__ void __launch_bounds__(kThreads)
    PoolScalarKernel(const __grid_constant__ PoolParams p) {
  constexpr int kCols = 4;
  if (!p.fused_checks && p.status->group_error != 0) return;
  const int lane = threadIdx.x & 31;
  const int64_t warps_per_block = kThreads / 32;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * warps_per_block;
  int t = 0;
  for (int64_t task = blockIdx.x * warps_per_block + threadIdx.x / 32;
       task < p.total_tasks; task += stride) {
    t = AdvanceDesc(p, t, task);
    const BagDesc& d = p.d[t];
    const int64_t bag = task - d.task_begin;
    int64_t begin, end;
    if (!BagRange(p, d, bag, &begin, &end)) continue;
    const bool weighted = d.weights != nullptr;
    const int64_t n = end - begin;
    for (int c0 = 0; c0 < d.dim; c0 += 32 * kCols) {
      float acc[kCols];
#pragma unroll
      for (int k = 0; k < kCols; ++k) acc[k] = 0.0f;
      float wsum = 0.0f;
      for (int64_t pidx = begin; pidx < end; ++pidx) {
        const int64_t id = LoadIndex(d.ids, d.ids64, pidx);
        const float w = weighted ? __ldg(d.weights + pidx) : 1.0f;
        if (weighted) {
          wsum = __fadd_rn(wsum, d.combine == 3 ? __fmul_rn(w, w) : w);
        }
        if (id < 0 || id >= d.vocab) {
          if (p.fused_checks && lane == 0 && c0 == 0) {
            RecordBadId(p.status, d.slot, pidx);
          }
          continue;
        }
        if (id < d.row_begin || id >= d.row_end) continue;
        const int64_t r = id - d.row_begin;
#pragma unroll
        for (int k = 0; k < kCols; ++k) {
          const int c = c0 + lane + 32 * k;
          if (c < d.dim) {
            float x;
            const int64_t at = r * d.dim + c;
            if constexpr (DT == 0) {
              x = __ldg(static_cast<const float*>(d.rows) + at);
            } else if constexpr (DT == 1) {
              const unsigned short b =
                  __ldg(static_cast<const unsigned short*>(d.rows) + at);
              x = __uint_as_float(static_cast<uint32_t>(b) << 16);
            } else {
              const float2 sb = __ldg(d.scale_bias + r);
              const float q = __int2float_rn(
                  __ldg(static_cast<const signed char*>(d.rows) + at));
              x = __fadd_rn(__fmul_rn(q, sb.x), sb.y);
            }
            acc[k] = weighted ? __fadd_rn(acc[k], __fmul_rn(w, x))
                              : __fadd_rn(acc[k], x);
          }
        }
      }
      float s = 1.0f;
      if (n > 0 && d.combine != 1) s = BagScale(d.combine, weighted, n, wsum);
#pragma unroll
      for (int k = 0; k < kCols; ++k) {
        const int c = c0 + lane + 32 * k;
        if (c < d.dim) {
          d.out[bag * d.out_stride + c] =
              (n > 0 && d.combine != 1) ? __fmul_rn(acc[k], s) : acc[k];
        }
      }
    }
  }
}

// Group validation (ValidateEmbeddingBagInput, embedding_bag.cc:99-133):
// one work item per offset and per id position. Offsets must start >= 0 and
// never decrease; the final offset must not exceed the ids (or weights);
// every id in [first, last) must be in [0, vocab).
__global__ void __launch_bounds__(kThreads)
    ValidateKernel(const __grid_constant__ PoolParams p, int64_t total_work) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  int t = 0;
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       w < total_work; w += stride) {
    while (t + 1 < p.n && w >= p.d[t + 1].work_begin) ++t;
    const BagDesc& d = p.d[t];
    const int64_t i = w - d.work_begin;
    const int64_t num_offsets = d.num_bags + 1;
    if (i < num_offsets) {
      const int64_t cur = LoadIndex(d.offsets, d.offs64, i);
      if (i == 0) {
        if (cur < 0) RecordError(p.status, d.slot, kErrBadOffsets);
      } else if (LoadIndex(d.offsets, d.offs64, i - 1) > cur) {
        RecordError(p.status, d.slot, kErrBadOffsets);
      }
      if (i == num_offsets - 1) {
        if (cur > d.num_ids) RecordError(p.status, d.slot, kErrLastExceedsIds);
        if (d.weights != nullptr && cur > d.num_weights) {
          RecordError(p.status, d.slot, kErrLastExceedsWeights);
        }
      }
    } else if (d.ids != nullptr) {
      const int64_t pos = i - num_offsets;
      const int64_t first = LoadIndex(d.offsets, d.offs64, 0);
      const int64_t last = LoadIndex(d.offsets, d.offs64, d.num_bags);
      if (pos >= first && pos < last) {
        const int64_t id = LoadIndex(d.ids, d.ids64, pos);
        if (id < 0 || id >= d.vocab) RecordBadId(p.status, d.slot, pos);
      }
    }
  }
}

__global__ void InterleaveKernel(const float* scale, const float* bias,
                                 float2* out, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < n; i += stride) {
    out[i] = make_float2(scale[i], bias[i]);
  }
}

int SmCount() {
  static int sms = [] {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
  }();
  return sms;
}

template <typename Kernel>
int GridFor(Kernel kernel, int64_t groups_needed, int groups_per_block) {
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, 0);
  if (per_sm <= 0) per_sm = 1;
  const int64_t max_grid = static_cast<int64_t>(SmCount()) * per_sm;
  const int64_t want = (groups_needed + groups_per_block - 1) / groups_per_block;
  return static_cast<int>(want < 1 ? 1 : (want < max_grid ? want : max_grid));
}

template <int DT, int G, int V>
cudaError_t LaunchVec(const PoolParams& p, cudaStream_t stream) {
  auto kernel = PoolVecKernel<DT, G, V>;
  const int grid = GridFor(kernel, p.total_tasks, kThreads / G);
  kernel<<<grid, kThreads, 0, stream>>>(p);
  return cudaGetLastError();
}

template <int DT>
cudaError_t LaunchForDtype(const Layout& l, const PoolParams& p,
                           cudaStream_t stream) {
  if (l.v == 0) {
    auto kernel = PoolScalarKernel<DT>;
    const int grid = GridFor(kernel, p.total_tasks, kThreads / 32);
    kernel<<<grid, kThreads, 0, stream>>>(p);
    return cudaGetLastError();
  }
  if (l.v == 1) {
    switch (l.g) {
      case 4: return LaunchVec<DT, 4, 1>(p, stream);
      case 8: return LaunchVec<DT, 8, 1>(p, stream);
      case 16: return LaunchVec<DT, 16, 1>(p, stream);
      default: return LaunchVec<DT, 32, 1>(p, stream);
    }
  }
  if (l.v == 2) return LaunchVec<DT, 32, 2>(p, stream);
  if constexpr (DT == 2) {
    return LaunchVec<DT, 32, 4>(p, stream);
  } else {
    if (l.v == 4) return LaunchVec<DT, 32, 4>(p, stream);
    return LaunchVec<DT, 32, 8>(p, stream);
  }
}

}  // namespace

Layout ChooseLayout(int dtype, int dim, const void* rows) {
  const int elem = dtype == 0 ? 4 : dtype == 1 ? 2 : 1;
  const int64_t row_bytes = static_cast<int64_t>(dim) * elem;
  const bool aligned = (reinterpret_cast<uintptr_t>(rows) & 15u) == 0;
  if (!aligned || row_bytes % 16 != 0) return {dtype, 32, 0};
  const int64_t vecs = row_bytes / 16;
  if (vecs <= 32) {
    int g = 4;
    while (g < vecs) g *= 2;
    return {dtype, g, 1};
  }
  const int64_t per_lane = (vecs + 31) / 32;
  if (per_lane <= 2) return {dtype, 32, 2};
  if (per_lane <= 4) return {dtype, 32, 4};
  if (per_lane <= 8 && dtype != 2) return {dtype, 32, 8};
  return {dtype, 32, 0};
}

cudaError_t LaunchPool(const Layout& layout, const PoolParams& p,
                       cudaStream_t stream, int* launches) {
  if (p.total_tasks <= 0) return cudaSuccess;
  ++*launches;
  switch (layout.dtype) {
    case 0: return LaunchForDtype<0>(layout, p, stream);
    case 1: return LaunchForDtype<1>(layout, p, stream);
    default: return LaunchForDtype<2>(layout, p, stream);
  }
}

cudaError_t LaunchValidate(const PoolParams& p, int64_t total_work,
                           cudaStream_t stream) {
  if (total_work <= 0) return cudaSuccess;
  const int grid = GridFor(ValidateKernel, total_work, kThreads);
  ValidateKernel<<<grid, kThreads, 0, stream>>>(p, total_work);
  return cudaGetLastError();
}

cudaError_t LaunchInterleaveScaleBias(const float* scale, const float* bias,
                                      float2* out, int64_t n,
                                      cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  const int64_t blocks = (n + kThreads - 1) / kThreads;
  const int grid = static_cast<int>(blocks < 4096 ? blocks : 4096);
  InterleaveKernel<<<grid, kThreads, 0, stream>>>(scale, bias, out, n);
  return cudaGetLastError();
}

}  // namespace xse
