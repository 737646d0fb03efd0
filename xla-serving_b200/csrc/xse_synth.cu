// Seeded synthetic inputs generated on the device.
//
// Counter-based: every value is a pure function of (seed, stream, index), so
// tables of any size (the 327 GB sharded set included) are generated in
// place, and any row can be regenerated on the host to check it.
//   bits(seed, stream, i) = mix(mix(seed*A + stream*B) + i*A)   (splitmix64)
//   u24 = bits >> 40, u = u24 / 2^24 (exact in fp32)
// Streams: table*16 + {0 values, 1 lengths, 2 ids, 3 weights, 5 scale,
// 6 bias}.
// Zipf ids use rejection-inversion (Hormann & Derflinger, ACM TOMACS 1996).

#include <cuda_runtime.h>
#include <stdint.h>

#include "xse_internal.h"

namespace xse {
namespace {

constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;
constexpr uint64_t kStreamMul = 0xD1B54A32D192ED03ull;

__host__ __device__ __forceinline__ uint64_t Mix64(uint64_t z) {
  z += kGolden;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

__device__ __forceinline__ uint64_t Bits64(uint64_t key, uint64_t index) {
  return Mix64(key + index * kGolden);
}

__host__ __device__ __forceinline__ uint64_t StreamKey(uint64_t seed,
                                                       uint64_t stream) {
  return Mix64(seed * kGolden + stream * kStreamMul);
}

__device__ __forceinline__ float U24(uint64_t bits) {
  return __uint2float_rn(static_cast<uint32_t>(bits >> 40)) *
         (1.0f / 16777216.0f);
}

__device__ __forceinline__ unsigned short F32ToBf16(float f) {
  const uint32_t w = __float_as_uint(f);
  if ((w & 0x7fffffffu) > 0x7f800000u) {
    return static_cast<unsigned short>((w >> 16) | 0x0040u);
  }
  return static_cast<unsigned short>((w + 0x7fffu + ((w >> 16) & 1u)) >> 16);
}

__global__ void SynthValuesKernel(void* rows, int dtype, uint64_t key,
                                  int64_t row0, int64_t nrows, int dim) {
  const int64_t total = nrows * dim;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       e < total; e += stride) {
    const uint64_t index = static_cast<uint64_t>(row0 * dim + e);
    const uint64_t bits = Bits64(key, index);
    if (dtype == 2) {
      const uint64_t u24 = bits >> 40;
      static_cast<signed char*>(rows)[e] =
          static_cast<signed char>(-127 + static_cast<int>((u24 * 255) >> 24));
    } else {
      const float v = __fadd_rn(-0.05f, __fmul_rn(0.1f, U24(bits)));
      if (dtype == 0) {
        static_cast<float*>(rows)[e] = v;
      } else {
        static_cast<unsigned short*>(rows)[e] = F32ToBf16(v);
      }
    }
  }
}

__global__ void SynthScaleBiasKernel(float* scale, float* bias,
                                     uint64_t scale_key, uint64_t bias_key,
                                     int64_t row0, int64_t nrows) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       r < nrows; r += stride) {
    const uint64_t row = static_cast<uint64_t>(row0 + r);
    scale[r] = __fadd_rn(1e-3f, __fmul_rn(9e-3f, U24(Bits64(scale_key, row))));
    bias[r] = __fadd_rn(-0.1f, __fmul_rn(0.2f, U24(Bits64(bias_key, row))));
  }
}

__global__ void SynthLengthsKernel(int64_t* lengths, int64_t n, int lo,
                                   int hi, uint64_t key) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const uint64_t span = static_cast<uint64_t>(hi - lo + 1);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < n; i += stride) {
    const uint64_t u24 = Bits64(key, static_cast<uint64_t>(i)) >> 40;
    lengths[i] = lo + static_cast<int64_t>((u24 * span) >> 24);
  }
}

__global__ void SynthWeightsKernel(float* weights, int64_t n, uint64_t key,
                                   int64_t index0) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < n; i += stride) {
    weights[i] = U24(Bits64(key, static_cast<uint64_t>(index0 + i)));
  }
}

struct ZipfDev {
  double alpha, n, h_lo, h_hi, squeeze;

  __device__ static double Log1pOverX(double x) {
    return fabs(x) > 1e-8 ? log1p(x) / x
                          : 1.0 - x * (0.5 - x * (1.0 / 3.0 - 0.25 * x));
  }
  __device__ static double Expm1OverX(double x) {
    return fabs(x) > 1e-8
               ? expm1(x) / x
               : 1.0 + x * 0.5 * (1.0 + x * (1.0 / 3.0) * (1.0 + 0.25 * x));
  }
  __device__ double Hat(double x) const { return exp(-alpha * log(x)); }
  __device__ double H(double x) const {
    const double lx = log(x);
    return Expm1OverX((1.0 - alpha) * lx) * lx;
  }
  __device__ double HInverse(double y) const {
    double t = y * (1.0 - alpha);
    if (t < -1.0) t = -1.0;
    return exp(Log1pOverX(t) * y);
  }
  __device__ void Init(int64_t count, double a) {
    alpha = a;
    n = static_cast<double>(count);
    h_lo = H(1.5) - 1.0;
    h_hi = H(n + 0.5);
    squeeze = 2.0 - HInverse(H(2.5) - Hat(2.0));
  }
  __device__ int64_t Try(double u) const {
    const double y = h_hi + u * (h_lo - h_hi);
    const double x = HInverse(y);
    double k = floor(x + 0.5);
    if (k < 1.0) k = 1.0;
    if (k > n) k = n;
    if (k - x <= squeeze || y >= H(k + 0.5) - Hat(k)) {
      return static_cast<int64_t>(k);
    }
    return 0;
  }
};

__global__ void SynthIdsKernel(int64_t* ids, int64_t n, int64_t vocab,
                               double alpha, uint64_t perm_mul,
                               uint64_t perm_add, uint64_t key,
                               int64_t index0) {
  __shared__ ZipfDev zipf;
  if (alpha > 0.0 && threadIdx.x == 0) zipf.Init(vocab, alpha);
  __syncthreads();
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  const uint64_t uv = static_cast<uint64_t>(vocab);
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < n; i += stride) {
    const uint64_t index = static_cast<uint64_t>(index0 + i);
    if (alpha <= 0.0) {
      ids[i] = static_cast<int64_t>(__umul64hi(Bits64(key, index), uv));
      continue;
    }
    int64_t k = 0;
    for (uint64_t attempt = 0; attempt < 64 && k == 0; ++attempt) {
      const uint64_t bits = Bits64(key, index * 64 + attempt);
      const double u = static_cast<double>(bits >> 11) *
                       (1.0 / 9007199254740992.0);
      k = zipf.Try(u);
    }
    if (k == 0) k = 1;
    // rank -> row: ((k-1)*perm_mul + perm_add) mod vocab. The caller keeps
    // vocab < 2^31 and perm_mul, perm_add < 2^32, so this cannot overflow.
    ids[i] = static_cast<int64_t>(
        (static_cast<uint64_t>(k - 1) * perm_mul + perm_add) % uv);
  }
}

int Blocks(int64_t n) {
  const int64_t b = (n + 255) / 256;
  return static_cast<int>(b < 1 ? 1 : (b > 148 * 16 ? 148 * 16 : b));
}

}  // namespace
}  // namespace xse

// C ABI (declared in include/xse_emb.h).
extern "C" int xse_synth_table_impl(void* rows, float* scale, float* bias,
                                    int32_t dtype, uint64_t seed,
                                    uint64_t table, int64_t row0,
                                    int64_t nrows, int32_t dim,
                                    cudaStream_t stream) {
  using namespace xse;
  if (nrows <= 0) return 0;
  SynthValuesKernel<<<Blocks(nrows * dim), 256, 0, stream>>>(
      rows, dtype, StreamKey(seed, table * 16 + 0), row0, nrows, dim);
  if (dtype == 2) {
    SynthScaleBiasKernel<<<Blocks(nrows), 256, 0, stream>>>(
        scale, bias, StreamKey(seed, table * 16 + 5),
        StreamKey(seed, table * 16 + 6), row0, nrows);
  }
  return cudaGetLastError() == cudaSuccess ? 0 : 13;
}

extern "C" int xse_synth_lengths_impl(int64_t* lengths, int64_t n, int32_t lo,
                                      int32_t hi, uint64_t seed,
                                      uint64_t table, cudaStream_t stream) {
  using namespace xse;
  if (n <= 0) return 0;
  SynthLengthsKernel<<<Blocks(n), 256, 0, stream>>>(
      lengths, n, lo, hi, StreamKey(seed, table * 16 + 1));
  return cudaGetLastError() == cudaSuccess ? 0 : 13;
}

extern "C" int xse_synth_ids_impl(int64_t* ids, int64_t n, int64_t vocab,
                                  double alpha, uint64_t perm_mul,
                                  uint64_t perm_add, uint64_t seed,
                                  uint64_t table, int64_t index0,
                                  cudaStream_t stream) {
  using namespace xse;
  if (n <= 0) return 0;
  SynthIdsKernel<<<Blocks(n), 256, 0, stream>>>(
      ids, n, vocab, alpha, perm_mul, perm_add,
      StreamKey(seed, table * 16 + 2), index0);
  return cudaGetLastError() == cudaSuccess ? 0 : 13;
}

extern "C" int xse_synth_weights_impl(float* weights, int64_t n,
                                      uint64_t seed, uint64_t table,
                                      int64_t index0, cudaStream_t stream) {
  using namespace xse;
  if (n <= 0) return 0;
  SynthWeightsKernel<<<Blocks(n), 256, 0, stream>>>(
      weights, n, StreamKey(seed, table * 16 + 3), index0);
  return cudaGetLastError() == cudaSuccess ? 0 : 13;
}
