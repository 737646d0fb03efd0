// The engine's legacy per-feature path on the device (xse_engine_execute_legacy
// in include/xse_emb.h).
//
// CpuEmbeddingEngine::Execute (data/cpu_embedding/cc/cpu_embedding_engine.cc:
// 91-166) takes validated FeatureBatchCsrInput batches
// (feature_batch_csr_input.cc:33-57) and, per feature, either pools in the
// table's own type -- AssembleCombinedEmbeddings<T>
// (compute_activations.cc:36-154), where a bf16 table accumulates in bf16 --
// or, for a sequence feature, gathers the first max_sequence_length rows of
// each sample into [samples, max_sequence_length, dim] with zero padding
// (AssembleSequenceEmbeddings, compute_activations.cc:187-224).
//
// One warp per (request, sample), lanes over columns: this path is kept for
// compatibility, not throughput. Every bf16 operation computes in fp32 and
// rounds to bf16 to nearest even, as Eigen's bfloat16 does; fp32 products and
// sums round separately (no FMA), as the reference's order requires.

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "xse_internal.h"

namespace xse {
namespace {

constexpr int kLegacyThreads = 256;

__device__ __forceinline__ int64_t Index(const void* base, int is64,
                                         int64_t i) {
  return is64 ? static_cast<const long long*>(base)[i]
              : static_cast<int64_t>(static_cast<const int*>(base)[i]);
}

__device__ __forceinline__ float Bf(uint16_t bits) {
  return __uint_as_float(static_cast<uint32_t>(bits) << 16);
}

__device__ __forceinline__ uint16_t ToBf(float v) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(v));
}

__device__ __forceinline__ void Flag(DevStatus* st, int slot,
                                     unsigned int f) {
  atomicOr(&st->req[slot].flags, f);
  atomicOr(&st->group_error, 1u);
}

// Locates the descriptor of flattened sample `task`.
__device__ __forceinline__ int Advance(const LegacyParams& p, int t,
                                       int64_t task) {
  while (t + 1 < p.n && task >= p.d[t + 1].task_begin) ++t;
  return t;
}

// FeatureBatchCsrInput's checks (row pointers start at 0, end at the id
// count, never decrease; weights empty or one per id) and the id bounds of
// the positions the feature reads (all of a pooled sample, the first
// max_sequence_length of a sequence sample).
__global__ void __launch_bounds__(kLegacyThreads)
    LegacyValidateKernel(const __grid_constant__ LegacyParams p) {
  const int lane = threadIdx.x & 31;
  const int64_t warps =
      static_cast<int64_t>(gridDim.x) * (kLegacyThreads / 32);
  int t = 0;
  for (int64_t task = static_cast<int64_t>(blockIdx.x) * (kLegacyThreads / 32) +
                      threadIdx.x / 32;
       task < p.total_tasks; task += warps) {
    t = Advance(p, t, task);
    const LegacyDesc& d = p.d[t];
    const int64_t b = task - d.task_begin;
    const int64_t begin = Index(d.offsets, d.offs64, b);
    const int64_t end = Index(d.offsets, d.offs64, b + 1);
    if (lane == 0) {
      unsigned int f = 0;
      if (end < begin) f |= kLegacyNotSorted;
      if (b == 0 && begin != 0) f |= kLegacySizeMismatch;
      if (b == d.num_bags - 1) {
        if (end != d.num_ids) f |= kLegacySizeMismatch;
        if (d.num_weights > 0 && d.num_weights != end) f |= kLegacyWeights;
      }
      if (f) Flag(p.status, d.slot, f);
    }
    if (end < begin || begin < 0 || end > d.num_ids) continue;
    int64_t last = end;
    if (d.max_seq > 0 && end - begin > d.max_seq) last = begin + d.max_seq;
    int64_t bad = -1;
    for (int64_t pos = begin + lane; pos < last; pos += 32) {
      const int64_t id = Index(d.ids, d.ids64, pos);
      if (id < 0 || id >= d.vocab) {
        bad = pos;
        break;
      }
    }
    if (bad >= 0) {
      atomicMax(&p.status->req[d.slot].inv_min_bad_index,
                ~static_cast<unsigned long long>(bad));
      Flag(p.status, d.slot, kLegacyBadId);
    }
  }
}

// Pooled sample in the table's type: fp32, or bf16 accumulated in bf16.
// Descriptors of other kinds are skipped.
template <int DT>
__global__ void __launch_bounds__(kLegacyThreads)
    LegacyPoolKernel(const __grid_constant__ LegacyParams p) {
  if (p.status->group_error != 0) return;
  constexpr int kKind = DT == 0 ? kLegacyPoolF32 : kLegacyPoolBf16;
  const int lane = threadIdx.x & 31;
  const int64_t warps =
      static_cast<int64_t>(gridDim.x) * (kLegacyThreads / 32);
  int t = 0;
  for (int64_t task = static_cast<int64_t>(blockIdx.x) * (kLegacyThreads / 32) +
                      threadIdx.x / 32;
       task < p.total_tasks; task += warps) {
    t = Advance(p, t, task);
    const LegacyDesc& d = p.d[t];
    if (d.kind != kKind) continue;
    const int64_t b = task - d.task_begin;
    const int64_t begin = Index(d.offsets, d.offs64, b);
    const int64_t n = Index(d.offsets, d.offs64, b + 1) - begin;
    // The weight total (CSR order) and the bag's scale, as in the reference.
    float scale = 1.0f;
    if (n > 0 && d.combine != 1) {
      if (d.weights == nullptr) {
        const float fn = static_cast<float>(n);
        scale = d.combine == 2 ? __fdiv_rn(1.0f, fn)
                               : __fdiv_rn(1.0f, __fsqrt_rn(fn));
      } else {
        float sw = 0.0f;
        for (int64_t k = 0; k < n; ++k) {
          const float w = d.weights[begin + k];
          sw = __fadd_rn(sw, d.combine == 2 ? w : __fmul_rn(w, w));
        }
        scale = d.combine == 2 ? __fdiv_rn(1.0f, sw)
                               : __fdiv_rn(1.0f, __fsqrt_rn(sw));
      }
    }
    for (int c = lane; c < d.dim; c += 32) {
      if constexpr (DT == 0) {
        const float* rows = static_cast<const float*>(d.rows);
        float acc = 0.0f;
        for (int64_t k = 0; k < n; ++k) {
          const int64_t id = Index(d.ids, d.ids64, begin + k);
          const float x = rows[id * d.dim + c];
          acc = d.weights == nullptr
                    ? __fadd_rn(acc, x)
                    : __fadd_rn(acc, __fmul_rn(d.weights[begin + k], x));
        }
        if (scale != 1.0f) acc = __fmul_rn(acc, scale);
        static_cast<float*>(d.out)[b * d.dim + c] = acc;
      } else {
        const uint16_t* rows = static_cast<const uint16_t*>(d.rows);
        uint16_t acc = 0;
        for (int64_t k = 0; k < n; ++k) {
          const int64_t id = Index(d.ids, d.ids64, begin + k);
          float x = Bf(rows[id * d.dim + c]);
          if (d.weights != nullptr) {
            x = Bf(ToBf(__fmul_rn(Bf(ToBf(d.weights[begin + k])), x)));
          }
          acc = ToBf(__fadd_rn(Bf(acc), x));
        }
        if (scale != 1.0f) acc = ToBf(__fmul_rn(Bf(acc), Bf(ToBf(scale))));
        static_cast<uint16_t*>(d.out)[b * d.dim + c] = acc;
      }
    }
  }
}

// Sequence sample: rows of its first min(len, max_seq) ids, then zeros.
__global__ void __launch_bounds__(kLegacyThreads)
    LegacySequenceKernel(const __grid_constant__ LegacyParams p) {
  if (p.status->group_error != 0) return;
  const int lane = threadIdx.x & 31;
  const int64_t warps =
      static_cast<int64_t>(gridDim.x) * (kLegacyThreads / 32);
  int t = 0;
  for (int64_t task = static_cast<int64_t>(blockIdx.x) * (kLegacyThreads / 32) +
                      threadIdx.x / 32;
       task < p.total_tasks; task += warps) {
    t = Advance(p, t, task);
    const LegacyDesc& d = p.d[t];
    if (d.kind != kLegacySequence) continue;
    const int64_t b = task - d.task_begin;
    const int64_t begin = Index(d.offsets, d.offs64, b);
    int64_t n = Index(d.offsets, d.offs64, b + 1) - begin;
    if (n > d.max_seq) n = d.max_seq;
    const size_t elem = d.dtype == 0 ? 4 : 2;
    char* out = static_cast<char*>(d.out) + b * d.max_seq * d.dim * elem;
    for (int64_t s = 0; s < d.max_seq; ++s) {
      const int64_t id = s < n ? Index(d.ids, d.ids64, begin + s) : -1;
      for (int c = lane; c < d.dim; c += 32) {
        if (d.dtype == 0) {
          reinterpret_cast<float*>(out)[s * d.dim + c] =
              id >= 0 ? static_cast<const float*>(d.rows)[id * d.dim + c]
                      : 0.0f;
        } else {
          reinterpret_cast<uint16_t*>(out)[s * d.dim + c] =
              id >= 0 ? static_cast<const uint16_t*>(d.rows)[id * d.dim + c]
                      : static_cast<uint16_t>(0);
        }
      }
    }
  }
}

int GridFor(int64_t tasks) {
  int64_t g = (tasks + kLegacyThreads / 32 - 1) / (kLegacyThreads / 32);
  if (g > 148 * 16) g = 148 * 16;
  return static_cast<int>(g < 1 ? 1 : g);
}

}  // namespace

cudaError_t LaunchLegacy(const LegacyParams& p, cudaStream_t stream) {
  if (p.total_tasks <= 0) return cudaSuccess;
  const int grid = GridFor(p.total_tasks);
  // Every request is checked before any output is written.
  LegacyValidateKernel<<<grid, kLegacyThreads, 0, stream>>>(p);
  cudaError_t e = cudaGetLastError();
  bool kinds[3] = {false, false, false};
  for (int k = 0; k < p.n; ++k) kinds[p.d[k].kind] = true;
  if (e == cudaSuccess && kinds[kLegacyPoolF32]) {
    LegacyPoolKernel<0><<<grid, kLegacyThreads, 0, stream>>>(p);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess && kinds[kLegacyPoolBf16]) {
    LegacyPoolKernel<1><<<grid, kLegacyThreads, 0, stream>>>(p);
    e = cudaGetLastError();
  }
  if (e == cudaSuccess && kinds[kLegacySequence]) {
    LegacySequenceKernel<<<grid, kLegacyThreads, 0, stream>>>(p);
    e = cudaGetLastError();
  }
  return e;
}

}  // namespace xse
