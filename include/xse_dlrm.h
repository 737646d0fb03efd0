/* DLRM dense tower on the B200: dense layers and the strided dot
 * interaction.
 *
 * The reference's DLRM bundle pools its 26 sparse features through
 * CpuEmbeddingLookupTransform and runs the dense tower (bottom MLP
 * 13-512-256-128 with ReLU, feature interaction, top MLP with a sigmoid head)
 * under XLA (examples/dlrm/model_jce.py:98-189). These entry points run that
 * tower on the device next to the pooled embeddings, so a forward pass never
 * leaves HBM. All tensors are fp32 device memory; `stream` is a
 * cudaStream_t (NULL: the legacy default stream). Status codes and
 * xse_last_error() as in xse_emb.h.
 */
#ifndef XSE_DLRM_H_
#define XSE_DLRM_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  XSE_ACT_NONE = 0,
  XSE_ACT_RELU = 1,
  XSE_ACT_SIGMOID = 2,
};

/* GEMM arithmetic of a Dense layer. */
enum {
  XSE_MATH_FP32 = 0,     /* fp32 FMA (CUDA cores) */
  XSE_MATH_BF16X9 = 1,   /* fp32 emulated on the tensor cores with three
                            bf16 terms per operand (fp32-level accuracy);
                            needs a cuBLASLt that offers it */
  XSE_MATH_TF32 = 2,     /* operands rounded to TF32 on the tensor cores:
                            reduced precision */
};

/* y = act(x K + bias), one flax.linen.Dense layer with its activation
 * (model_jce.py:107-138).
 *   x: [rows, in_dim], row stride x_stride floats (>= in_dim)
 *   kernel: [in_dim, out_dim] row-major, the Dense layer's kernel layout
 *   bias: [out_dim] or NULL
 *   y: [rows, out_dim], row stride y_stride floats (>= out_dim)
 * `math` is an XSE_MATH_* mode for the GEMM; XSE_MATH_BF16X9 returns
 * UNIMPLEMENTED where the loaded cuBLASLt lacks it. Bias and ReLU are fused
 * into the GEMM (cuBLASLt epilogue); a sigmoid head with out_dim == 1 runs as
 * one fp32 kernel (dot, bias, sigmoid) in every mode. */
int xse_linear_forward(const float* x, int64_t rows, int32_t in_dim,
                       int64_t x_stride, const float* kernel, const float* bias,
                       int32_t out_dim, int32_t activation, int32_t math,
                       float* y, int64_t y_stride, void* stream);

/* hi = src rounded to TF32 (round to nearest, ties away from zero) and
 * lo = src - hi (exact), for a [rows, cols] block with row stride `stride`
 * (the same stride in hi and lo). */
int xse_tf32_split(const float* src, int64_t rows, int32_t cols,
                   int64_t stride, float* hi, float* lo, void* stream);

/* y = act(x K + bias) from split operands (x = x_hi + x_lo, K = k_hi + k_lo
 * as made by xse_tf32_split) as three TF32 tensor-core GEMMs accumulated in
 * fp32: y = x_lo k_hi + x_hi k_lo + x_hi k_hi (+ bias, then act). The hi
 * parts are exact in TF32 and the dropped x_lo k_lo term is below 2^-22 of
 * |x||K|, so the result has fp32-level accuracy. act: XSE_ACT_NONE or
 * XSE_ACT_RELU. Layouts as xse_linear_forward; x_hi and x_lo share
 * x_stride, k_hi and k_lo are [in_dim, out_dim]. */
int xse_linear_forward_tf32x3(const float* x_hi, const float* x_lo,
                              int64_t rows, int32_t in_dim, int64_t x_stride,
                              const float* k_hi, const float* k_lo,
                              const float* bias, int32_t out_dim,
                              int32_t activation, float* y, int64_t y_stride,
                              void* stream);

/* The dot interaction of xse_emb.h's xse_dot_interaction with strides:
 * dense rows every dense_stride floats, pooled samples every pooled_stride
 * floats ([T, dim] each, contiguous), output rows every out_stride floats
 * (>= dim + (T+1)T/2). Columns past the interaction width up to out_stride
 * are written with zeros, so a padded row feeds a Dense layer whose kernel
 * has zero rows there. No counterpart in the reference (it uses a
 * DCN-v2 cross network, model_jce.py:140-161). */
int xse_dot_interaction_strided(const float* dense, int64_t dense_stride,
                                const float* pooled, int64_t pooled_stride,
                                int64_t batch, int32_t num_tables,
                                int32_t dim, float* out, int64_t out_stride,
                                void* stream);

#ifdef __cplusplus
}
#endif

#endif /* XSE_DLRM_H_ */
