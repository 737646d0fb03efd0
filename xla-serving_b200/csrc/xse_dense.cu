// Dense layers of the DLRM tower (declared in include/xse_dlrm.h).
//
// A Dense layer y = act(x K + b) (flax.linen.Dense in the reference's model,
// examples/dlrm/model_jce.py:107-138) is a plain GEMM. It runs on cuBLASLt
// with fp32 inputs and outputs (arithmetic per XSE_MATH_*: fp32 FMA, fp32
// emulated with bf16x9 on the tensor cores, or TF32) with the bias and the
// ReLU in the GEMM epilogue. The first call of each layer shape times
// cuBLASLt's heuristic candidates on the caller's buffers and keeps the
// fastest. The 1-wide sigmoid head (256 -> 1) is a dot product per row and
// runs as one kernel: a warp per row, coalesced reads of x, a shuffle
// reduction, the bias and the sigmoid.
//
// Layout: row-major x [rows, in] (row stride xs) and kernel [in, out] are, to
// column-major cuBLAS, x^T [in, rows] (ld xs) and K^T [out, in] (ld out), so
// y^T [out, rows] (ld ys) = K^T x^T with no transposes, and the epilogue's
// bias vector (length m = out) is added per output feature.

#include <cublasLt.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <map>
#include <mutex>
#include <tuple>

#include "../../include/xse_dlrm.h"
#include "../../include/xse_emb.h"
#include "xse_internal.h"

namespace xse {
namespace {

int Fail(int code, const char* fmt, ...) __attribute__((format(printf, 2, 3)));
int Fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list args;
  va_start(args, fmt);
  vsnprintf(buf, sizeof(buf), fmt, args);
  va_end(args);
  SetLastErrorMessage(buf);
  return code;
}

// Largest power of two (<= 256) dividing the address: the alignment cuBLASLt
// may assume when it picks a kernel.
uint32_t AlignmentOf(const void* p) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(p);
  uint32_t align = 256;
  while (align > 1 && (a & (align - 1)) != 0) align >>= 1;
  return align;
}

using PlanKey = std::tuple<int64_t, int32_t, int32_t, int64_t, int64_t,
                           int32_t, bool, uint32_t, uint32_t, uint32_t,
                           int32_t>;

cublasComputeType_t ComputeTypeOf(int32_t math) {
  switch (math) {
    case XSE_MATH_BF16X9:
      return CUBLAS_COMPUTE_32F_EMULATED_16BFX9;
    case XSE_MATH_TF32:
      return CUBLAS_COMPUTE_32F_FAST_TF32;
    default:
      return CUBLAS_COMPUTE_32F;
  }
}

constexpr int kMaxCandidates = 8;

struct Plan {
  cublasLtMatmulDesc_t op = nullptr;
  cublasLtMatrixLayout_t a = nullptr, b = nullptr, c = nullptr;
  cublasLtMatmulAlgo_t algo;
  cublasLtMatmulAlgo_t candidates[kMaxCandidates];
  int num_candidates = 0;
  bool tuned = false;
};

// One cuBLASLt handle and a plan cache per device. Plans are keyed by every
// shape, stride, epilogue and alignment that the algorithm choice depends
// on; the bias pointer is set on the plan's descriptor under the mutex just
// before the (asynchronous) launch, so concurrent callers do not race on it.
struct LtDevice {
  std::mutex mu;
  cublasLtHandle_t handle = nullptr;
  std::map<PlanKey, Plan> plans;
};

LtDevice* GetLtDevice(int device) {
  static std::mutex mu;
  static std::map<int, LtDevice*> devices;
  std::lock_guard<std::mutex> lock(mu);
  auto it = devices.find(device);
  if (it != devices.end()) return it->second;
  LtDevice* d = new LtDevice();  // kept until exit: handles are per device
  if (cublasLtCreate(&d->handle) != CUBLAS_STATUS_SUCCESS) {
    delete d;
    return nullptr;
  }
  devices[device] = d;
  return d;
}

int LtFail(cublasStatus_t s, const char* what) {
  return Fail(XSE_INTERNAL, "cuBLASLt %s failed (status %d)", what,
              static_cast<int>(s));
}

int MakePlan(LtDevice* dev, const PlanKey& key, Plan* plan) {
  const int64_t rows = std::get<0>(key);
  const int32_t in = std::get<1>(key), out = std::get<2>(key);
  const int64_t xs = std::get<3>(key), ys = std::get<4>(key);
  const int32_t act = std::get<5>(key);
  const bool has_bias = std::get<6>(key);
  const int32_t math = std::get<10>(key);
  cublasStatus_t s =
      cublasLtMatmulDescCreate(&plan->op, ComputeTypeOf(math), CUDA_R_32F);
  if (s != CUBLAS_STATUS_SUCCESS) {
    if (math != XSE_MATH_FP32) {
      return Fail(XSE_UNIMPLEMENTED,
                  "GEMM math mode %d is not offered by the loaded cuBLASLt "
                  "(status %d)", math, static_cast<int>(s));
    }
    return LtFail(s, "descriptor");
  }
  const cublasOperation_t n = CUBLAS_OP_N;
  cublasLtMatmulDescSetAttribute(plan->op, CUBLASLT_MATMUL_DESC_TRANSA, &n,
                                 sizeof(n));
  cublasLtMatmulDescSetAttribute(plan->op, CUBLASLT_MATMUL_DESC_TRANSB, &n,
                                 sizeof(n));
  const bool relu = act == XSE_ACT_RELU;
  cublasLtEpilogue_t epi =
      has_bias ? (relu ? CUBLASLT_EPILOGUE_RELU_BIAS : CUBLASLT_EPILOGUE_BIAS)
               : (relu ? CUBLASLT_EPILOGUE_RELU : CUBLASLT_EPILOGUE_DEFAULT);
  cublasLtMatmulDescSetAttribute(plan->op, CUBLASLT_MATMUL_DESC_EPILOGUE, &epi,
                                 sizeof(epi));
  s = cublasLtMatrixLayoutCreate(&plan->a, CUDA_R_32F, out, in, out);
  if (s == CUBLAS_STATUS_SUCCESS) {
    s = cublasLtMatrixLayoutCreate(&plan->b, CUDA_R_32F, in, rows, xs);
  }
  if (s == CUBLAS_STATUS_SUCCESS) {
    s = cublasLtMatrixLayoutCreate(&plan->c, CUDA_R_32F, out, rows, ys);
  }
  if (s != CUBLAS_STATUS_SUCCESS) return LtFail(s, "layout");
  cublasLtMatmulPreference_t pref = nullptr;
  s = cublasLtMatmulPreferenceCreate(&pref);
  if (s != CUBLAS_STATUS_SUCCESS) return LtFail(s, "preference");
  // No workspace: a workspace shared between streams would race, and the
  // fp32 kernels of these shapes need none.
  const size_t ws = 0;
  cublasLtMatmulPreferenceSetAttribute(
      pref, CUBLASLT_MATMUL_PREF_MAX_WORKSPACE_BYTES, &ws, sizeof(ws));
  const uint32_t align_a = std::get<7>(key), align_b = std::get<8>(key),
                 align_c = std::get<9>(key);
  cublasLtMatmulPreferenceSetAttribute(
      pref, CUBLASLT_MATMUL_PREF_MIN_ALIGNMENT_A_BYTES, &align_a,
      sizeof(align_a));
  cublasLtMatmulPreferenceSetAttribute(
      pref, CUBLASLT_MATMUL_PREF_MIN_ALIGNMENT_B_BYTES, &align_b,
      sizeof(align_b));
  cublasLtMatmulPreferenceSetAttribute(
      pref, CUBLASLT_MATMUL_PREF_MIN_ALIGNMENT_C_BYTES, &align_c,
      sizeof(align_c));
  cublasLtMatmulPreferenceSetAttribute(
      pref, CUBLASLT_MATMUL_PREF_MIN_ALIGNMENT_D_BYTES, &align_c,
      sizeof(align_c));
  cublasLtMatmulHeuristicResult_t results[kMaxCandidates] = {};
  int found = 0;
  s = cublasLtMatmulAlgoGetHeuristic(dev->handle, plan->op, plan->a, plan->b,
                                     plan->c, plan->c, pref, kMaxCandidates,
                                     results, &found);
  cublasLtMatmulPreferenceDestroy(pref);
  if ((s != CUBLAS_STATUS_SUCCESS || found == 0) && math != XSE_MATH_FP32) {
    return Fail(XSE_UNIMPLEMENTED,
                "GEMM math mode %d has no kernel in the loaded cuBLASLt for a "
                "%lld x %d x %d layer (status %d)", math,
                static_cast<long long>(rows), in, out, static_cast<int>(s));
  }
  if (s != CUBLAS_STATUS_SUCCESS || found == 0) {
    return Fail(XSE_INTERNAL,
                "cuBLASLt has no fp32 kernel for a %lld x %d x %d layer "
                "(status %d)", static_cast<long long>(rows), in, out,
                static_cast<int>(s));
  }
  plan->num_candidates = 0;
  for (int i = 0; i < found; ++i) {
    if (results[i].state == CUBLAS_STATUS_SUCCESS) {
      plan->candidates[plan->num_candidates++] = results[i].algo;
    }
  }
  if (plan->num_candidates == 0) {
    return Fail(XSE_INTERNAL, "cuBLASLt returned no usable algorithm");
  }
  plan->algo = plan->candidates[0];
  plan->tuned = plan->num_candidates == 1;
  return XSE_OK;
}

// Times every heuristic candidate of a new plan on the caller's own buffers
// (each run computes the same y) and keeps the fastest. Runs once per plan,
// outside stream capture; a capturing caller keeps the first candidate.
void TunePlan(LtDevice* dev, Plan* plan, const float* x, const float* kernel,
              int64_t y_floats, cudaStream_t s) {
  plan->tuned = true;
  cudaStreamCaptureStatus cap = cudaStreamCaptureStatusNone;
  if (cudaStreamIsCapturing(s, &cap) != cudaSuccess ||
      cap != cudaStreamCaptureStatusNone || plan->num_candidates < 2) {
    return;
  }
  // The candidates write a scratch output, so the caller's y (which a
  // following GEMM may accumulate into) is left alone.
  float* y = nullptr;
  if (cudaStreamSynchronize(s) != cudaSuccess ||
      cudaMalloc(&y, y_floats * sizeof(float)) != cudaSuccess) {
    cudaGetLastError();
    return;
  }
  cudaEvent_t e0, e1;
  if (cudaEventCreate(&e0) != cudaSuccess) {
    cudaFree(y);
    return;
  }
  if (cudaEventCreate(&e1) != cudaSuccess) {
    cudaEventDestroy(e0);
    cudaFree(y);
    return;
  }
  const float alpha = 1.0f, beta = 0.0f;
  float best_ms = 0.0f;
  int best = -1;
  for (int i = 0; i < plan->num_candidates; ++i) {
    bool ok = true;
    for (int rep = 0; rep < 4 && ok; ++rep) {  // first run warms up
      if (rep == 1) cudaEventRecord(e0, s);
      ok = cublasLtMatmul(dev->handle, plan->op, &alpha, kernel, plan->a, x,
                          plan->b, &beta, y, plan->c, y, plan->c,
                          &plan->candidates[i], nullptr, 0,
                          s) == CUBLAS_STATUS_SUCCESS;
    }
    cudaEventRecord(e1, s);
    float ms = 0.0f;
    if (!ok || cudaEventSynchronize(e1) != cudaSuccess ||
        cudaEventElapsedTime(&ms, e0, e1) != cudaSuccess) {
      cudaGetLastError();
      continue;
    }
    if (best < 0 || ms < best_ms) {
      best = i;
      best_ms = ms;
    }
  }
  cudaEventDestroy(e0);
  cudaEventDestroy(e1);
  cudaStreamSynchronize(s);
  cudaFree(y);
  if (best >= 0) plan->algo = plan->candidates[best];
}

void DestroyPlan(Plan* p) {
  if (p->a) cublasLtMatrixLayoutDestroy(p->a);
  if (p->b) cublasLtMatrixLayoutDestroy(p->b);
  if (p->c) cublasLtMatrixLayoutDestroy(p->c);
  if (p->op) cublasLtMatmulDescDestroy(p->op);
}

__device__ __forceinline__ float Sigmoid(float v) {
  return 1.0f / (1.0f + expf(-v));
}

// y[r] = sigmoid(x[r, :] . k + b): one warp per row.
__global__ void __launch_bounds__(256)
    SigmoidHeadKernel(const float* __restrict__ x, int64_t rows, int in_dim,
                      int64_t x_stride, const float* __restrict__ k,
                      const float* __restrict__ bias,
                      float* __restrict__ y, int64_t y_stride) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  for (int64_t r = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) +
                   threadIdx.x / 32;
       r < rows; r += warps) {
    const float* xr = x + r * x_stride;
    float s = 0.0f;
    for (int c = lane; c < in_dim; c += 32) s = fmaf(xr[c], __ldg(k + c), s);
#pragma unroll
    for (int o = 16; o >= 1; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) y[r * y_stride] = Sigmoid(s + (bias ? bias[0] : 0.0f));
  }
}

// In-place sigmoid of a [rows, cols] block with row stride `stride`.
__global__ void SigmoidKernel(float* __restrict__ y, int64_t rows, int cols,
                              int64_t stride) {
  const int64_t total = rows * cols;
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       e < total; e += step) {
    float* p = y + (e / cols) * stride + e % cols;
    *p = Sigmoid(*p);
  }
}

int BlocksFor(int64_t work, int per_block, int cap) {
  int64_t b = (work + per_block - 1) / per_block;
  if (b > cap) b = cap;
  return static_cast<int>(b < 1 ? 1 : b);
}

// y = act(beta*y + x K + bias) on cuBLASLt with the plan of this shape.
int RunGemm(const float* x, int64_t rows, int32_t in_dim, int64_t x_stride,
            const float* kernel, const float* bias, int32_t out_dim,
            int32_t act, int32_t math, float beta, float* y, int64_t y_stride,
            cudaStream_t s) {
  int device = 0;
  cudaGetDevice(&device);
  LtDevice* dev = GetLtDevice(device);
  if (dev == nullptr) return Fail(XSE_INTERNAL, "cuBLASLt handle creation failed");
  const PlanKey key(rows, in_dim, out_dim, x_stride, y_stride, act,
                    bias != nullptr, AlignmentOf(kernel), AlignmentOf(x),
                    AlignmentOf(y), math);
  std::lock_guard<std::mutex> lock(dev->mu);
  auto it = dev->plans.find(key);
  if (it == dev->plans.end()) {
    Plan plan;
    const int rc = MakePlan(dev, key, &plan);
    if (rc != XSE_OK) {
      DestroyPlan(&plan);
      return rc;
    }
    it = dev->plans.emplace(key, plan).first;
  }
  Plan& plan = it->second;
  if (bias != nullptr) {
    cublasLtMatmulDescSetAttribute(plan.op, CUBLASLT_MATMUL_DESC_BIAS_POINTER,
                                   &bias, sizeof(bias));
  }
  if (!plan.tuned) TunePlan(dev, &plan, x, kernel, rows * y_stride, s);
  const float alpha = 1.0f;
  const cublasStatus_t st = cublasLtMatmul(
      dev->handle, plan.op, &alpha, kernel, plan.a, x, plan.b, &beta, y,
      plan.c, y, plan.c, &plan.algo, nullptr, 0, s);
  if (st != CUBLAS_STATUS_SUCCESS) return LtFail(st, "matmul");
  return XSE_OK;
}

// hi = src rounded to TF32 (nearest, ties away from zero), lo = src - hi
// (exact: hi agrees with src in sign, exponent and the top 10 fraction bits).
__global__ void Tf32SplitKernel(const float* __restrict__ src, int64_t rows,
                                int cols, int64_t stride,
                                float* __restrict__ hi,
                                float* __restrict__ lo) {
  const int64_t total = rows * cols;
  const int64_t step = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t e = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       e < total; e += step) {
    const int64_t at = (e / cols) * stride + e % cols;
    const float v = src[at];
    uint32_t h;
    asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(v));
    const float vh = __uint_as_float(h);
    hi[at] = vh;
    lo[at] = __fsub_rn(v, vh);
  }
}

}  // namespace
}  // namespace xse

extern "C" int xse_linear_forward(const float* x, int64_t rows,
                                  int32_t in_dim, int64_t x_stride,
                                  const float* kernel, const float* bias,
                                  int32_t out_dim, int32_t activation,
                                  int32_t math, float* y, int64_t y_stride,
                                  void* stream) {
  using namespace xse;
  SetLastLaunchCount(0);
  if (rows < 0 || in_dim < 1 || out_dim < 1 || x_stride < in_dim ||
      y_stride < out_dim) {
    return Fail(XSE_INVALID_ARGUMENT,
                "Dense layer needs rows >= 0, positive dimensions and row "
                "strides x >= in_dim, y >= out_dim.");
  }
  if (activation < XSE_ACT_NONE || activation > XSE_ACT_SIGMOID) {
    return Fail(XSE_INVALID_ARGUMENT, "Unknown activation: %d", activation);
  }
  if (math < XSE_MATH_FP32 || math > XSE_MATH_TF32) {
    return Fail(XSE_INVALID_ARGUMENT, "Unknown GEMM math mode: %d", math);
  }
  if (rows == 0) return XSE_OK;
  if (x == nullptr || kernel == nullptr || y == nullptr) {
    return Fail(XSE_INVALID_ARGUMENT, "Dense layer buffers must be non-null.");
  }
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (activation == XSE_ACT_SIGMOID && out_dim == 1) {
    SigmoidHeadKernel<<<BlocksFor(rows, 8, 148 * 16), 256, 0, s>>>(
        x, rows, in_dim, x_stride, kernel, bias, y, y_stride);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
      return Fail(XSE_INTERNAL, "sigmoid head launch: %s",
                  cudaGetErrorString(e));
    }
    SetLastLaunchCount(1);
    return XSE_OK;
  }
  const int32_t gemm_act = activation == XSE_ACT_RELU ? XSE_ACT_RELU
                                                      : XSE_ACT_NONE;
  const int rc = RunGemm(x, rows, in_dim, x_stride, kernel, bias, out_dim,
                         gemm_act, math, 0.0f, y, y_stride, s);
  if (rc != XSE_OK) return rc;
  int launches = 1;
  if (activation == XSE_ACT_SIGMOID) {
    SigmoidKernel<<<BlocksFor(rows * out_dim, 256, 148 * 16), 256, 0, s>>>(
        y, rows, out_dim, y_stride);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
      return Fail(XSE_INTERNAL, "sigmoid launch: %s", cudaGetErrorString(e));
    }
    ++launches;
  }
  SetLastLaunchCount(launches);
  return XSE_OK;
}

extern "C" int xse_tf32_split(const float* src, int64_t rows, int32_t cols,
                              int64_t stride, float* hi, float* lo,
                              void* stream) {
  using namespace xse;
  SetLastLaunchCount(0);
  if (rows < 0 || cols < 1 || stride < cols) {
    return Fail(XSE_INVALID_ARGUMENT,
                "TF32 split needs rows >= 0, cols >= 1 and stride >= cols.");
  }
  if (rows == 0) return XSE_OK;
  if (src == nullptr || hi == nullptr || lo == nullptr) {
    return Fail(XSE_INVALID_ARGUMENT, "TF32 split buffers must be non-null.");
  }
  Tf32SplitKernel<<<BlocksFor(rows * cols, 256, 148 * 16), 256, 0,
                    static_cast<cudaStream_t>(stream)>>>(src, rows, cols,
                                                         stride, hi, lo);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return Fail(XSE_INTERNAL, "TF32 split launch: %s", cudaGetErrorString(e));
  }
  SetLastLaunchCount(1);
  return XSE_OK;
}

extern "C" int xse_linear_forward_tf32x3(
    const float* x_hi, const float* x_lo, int64_t rows, int32_t in_dim,
    int64_t x_stride, const float* k_hi, const float* k_lo, const float* bias,
    int32_t out_dim, int32_t activation, float* y, int64_t y_stride,
    void* stream) {
  using namespace xse;
  SetLastLaunchCount(0);
  if (rows < 0 || in_dim < 1 || out_dim < 1 || x_stride < in_dim ||
      y_stride < out_dim) {
    return Fail(XSE_INVALID_ARGUMENT,
                "Dense layer needs rows >= 0, positive dimensions and row "
                "strides x >= in_dim, y >= out_dim.");
  }
  if (activation != XSE_ACT_NONE && activation != XSE_ACT_RELU) {
    return Fail(XSE_INVALID_ARGUMENT,
                "The split-TF32 layer takes no activation or ReLU, got %d",
                activation);
  }
  if (rows == 0) return XSE_OK;
  if (x_hi == nullptr || x_lo == nullptr || k_hi == nullptr ||
      k_lo == nullptr || y == nullptr) {
    return Fail(XSE_INVALID_ARGUMENT, "Dense layer buffers must be non-null.");
  }
  const cudaStream_t s = static_cast<cudaStream_t>(stream);
  // Small terms first, then the leading term with the bias and activation.
  int rc = RunGemm(x_lo, rows, in_dim, x_stride, k_hi, nullptr, out_dim,
                   XSE_ACT_NONE, XSE_MATH_TF32, 0.0f, y, y_stride, s);
  if (rc == XSE_OK) {
    rc = RunGemm(x_hi, rows, in_dim, x_stride, k_lo, nullptr, out_dim,
                 XSE_ACT_NONE, XSE_MATH_TF32, 1.0f, y, y_stride, s);
  }
  if (rc == XSE_OK) {
    rc = RunGemm(x_hi, rows, in_dim, x_stride, k_hi, bias, out_dim,
                 activation, XSE_MATH_TF32, 1.0f, y, y_stride, s);
  }
  if (rc != XSE_OK) return rc;
  SetLastLaunchCount(3);
  return XSE_OK;
}
