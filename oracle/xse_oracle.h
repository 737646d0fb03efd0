/* CPU oracle for the embedding-bag / DLRM interaction path.
 *
 * TEST INFRASTRUCTURE ONLY. This library is a plain C++17 restatement of the
 * reference CPU embedding engine (openxla/xla-serving, directory
 * data/cpu_embedding/cc and data/kernels/cpu_embedding). It is the
 * reference result that the CUDA path is compared against in the tests, and
 * the timed CPU baseline. Only the test suite, the smoke check and the
 * benchmark's CPU-baseline leg may load it; the product never links or
 * calls it.
 *
 * Parity pins: the reference cannot be compiled here (it needs Bazel, abseil
 * and Eigen, none of which are present), so the restatement is pinned against
 * the reference's own known-answer tests (transcribed as golden vectors) and
 * against the reference's numpy lookup (examples/dlrm_benchmark/common.py),
 * executed on seeded inputs by tests/golden/make_golden.py.
 *
 * Status codes follow absl::StatusCode numbering.
 */
#ifndef XSE_ORACLE_H_
#define XSE_ORACLE_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

enum {
  ORACLE_OK = 0,
  ORACLE_INVALID_ARGUMENT = 3,
  ORACLE_NOT_FOUND = 5,
  ORACLE_FAILED_PRECONDITION = 9,
};

/* Table storage. F32 follows the reference; BF16 rows are widened to fp32 and
 * pooled in fp32; I8_ROWWISE rows are dequantized as float(q)*scale+bias and
 * then pooled in fp32. */
enum { ORACLE_F32 = 0, ORACLE_BF16 = 1, ORACLE_I8_ROWWISE = 2 };
/* Combine modes, numbered as in the reference manifest proto
 * (data/kernels/cpu_embedding/cpu_embedding.proto:21-26). */
enum { ORACLE_SUM = 1, ORACLE_MEAN = 2, ORACLE_SQRTN = 3 };

typedef struct {
  int32_t dtype;
  int32_t combine;
  const void* table;   /* [vocab, dim] row-major */
  const float* scale;  /* [vocab], I8_ROWWISE only */
  const float* bias;   /* [vocab], I8_ROWWISE only */
  int64_t vocab;
  int64_t dim;
  const int64_t* ids;
  int64_t num_ids;
  const void* offsets; /* absolute CSR offsets, num_offsets entries */
  int32_t offsets_i64; /* 1: int64 offsets, 0: int32 */
  int64_t num_offsets;
  const float* weights; /* NULL or num_weights entries */
  int64_t num_weights;
  float* out;          /* (num_offsets-1) x dim */
} oracle_request;

/* ExecuteEmbeddingBagBatch restatement (embedding_bag.cc:477-535): validates
 * the whole group, checks output isolation, then pools. num_threads <= 1 runs
 * inline; otherwise bag-range tasks (4 per thread, never splitting a bag) are
 * taken by a persistent pool of num_threads workers, unless the total output
 * is at most inline_threshold floats. */
int oracle_embedding_bag_batch(const oracle_request* reqs, int32_t n,
                               int32_t num_threads, int64_t inline_threshold,
                               char* err, int32_t errlen);

/* AssembleCombinedEmbeddings<bfloat16> restatement (compute_activations.cc:
 * 36-154): bf16 table, bf16 accumulator, bf16 scale; int32 row pointers. The
 * output is bf16 bits. */
int oracle_assemble_bf16_accumulate(const uint16_t* table, int64_t vocab,
                                    int64_t dim, int32_t combine,
                                    const int64_t* ids, int64_t num_ids,
                                    const int32_t* row_pointers,
                                    int64_t num_row_pointers,
                                    const float* weights, uint16_t* out,
                                    char* err, int32_t errlen);

/* AssembleSequenceEmbeddings (compute_activations.cc:187-224): out is
 * [samples, max_seq, dim] of the table's type (ORACLE_F32 or ORACLE_BF16
 * bits), zeroed by the caller; each sample's first min(len, max_seq) ids are
 * bounds-checked (index = position within the sample) and their rows copied. */
int oracle_sequence_gather(const void* table, int32_t dtype, int64_t vocab,
                           int64_t dim, const int64_t* ids,
                           const int32_t* row_pointers,
                           int64_t num_row_pointers, int64_t max_seq,
                           void* out, char* err, int32_t errlen);

/* DenseCpuEmbeddingLookupTransform CSR build (dense_cpu_embedding_lookup_
 * transform.cc:186-225). dense is [batch, seq] int32 or int64. Writes ids
 * (capacity >= batch*seq + batch) and batch+1 int32 row pointers; returns the
 * number of ids through *num_ids. */
int oracle_dense_to_csr(const void* dense, int32_t dense_i64, int64_t batch,
                        int64_t seq, int64_t pad_value, int64_t* ids,
                        int32_t* row_pointers, int64_t* num_ids, char* err,
                        int32_t errlen);

/* Dense row-pointer generation for dense_lookup (cpu_embedding_lookup_
 * transform.cc:297-316), including its int32 overflow guards. */
int oracle_dense_lookup_row_pointers(int64_t batch, int64_t valency,
                                     int32_t* row_pointers, char* err,
                                     int32_t errlen);

/* DLRM pairwise dot interaction. Z_b = [dense_b; pooled_b,0..T-1] (T+1 rows
 * of dim D). out_b = [dense_b (D values), Z_b[i].Z_b[j] for i<j row-major].
 * Accumulates in double. pooled is [batch, T, D]. */
void oracle_dot_interaction(const float* dense, const float* pooled,
                            int64_t batch, int32_t num_tables, int32_t dim,
                            float* out);

/* Counter-based synthetic data, restated independently of the device
 * generator so the device tables can be checked bit for bit. */
double oracle_uniform(uint64_t seed, uint64_t stream, uint64_t index);
void oracle_synth_rows_f32(uint64_t seed, uint64_t table, int64_t row0,
                           int64_t nrows, int64_t dim, float* out);
void oracle_synth_rows_bf16(uint64_t seed, uint64_t table, int64_t row0,
                            int64_t nrows, int64_t dim, uint16_t* out);
void oracle_synth_rows_i8(uint64_t seed, uint64_t table, int64_t row0,
                          int64_t nrows, int64_t dim, int8_t* q, float* scale,
                          float* bias);
/* Rows rows[0..n) of a synthetic table (any order, repeats allowed): out is
 * [n, dim] in the table's storage type; int8 tables also fill scale[n] and
 * bias[n]. */
void oracle_synth_rows_at(int32_t dtype, uint64_t seed, uint64_t table,
                          const int64_t* rows, int64_t n, int64_t dim,
                          void* out, float* scale, float* bias);
/* Bag lengths uniform in [lo, hi], per-id weights U(0,1) and ids (uniform
 * when alpha <= 0, else bounded Zipf(alpha) ranks mapped to rows by
 * ((rank - 1) * perm_mul + perm_add) mod vocab), as the device generates
 * them for the same (seed, table) stream. */
void oracle_synth_lengths(int64_t n, int32_t lo, int32_t hi, uint64_t seed,
                          uint64_t table, int64_t* out);
void oracle_synth_weights(int64_t n, uint64_t seed, uint64_t table,
                          int64_t index0, float* out);
void oracle_synth_ids(int64_t n, int64_t vocab, double alpha,
                      uint64_t perm_mul, uint64_t perm_add, uint64_t seed,
                      uint64_t table, int64_t index0, int64_t* out);
/* Bounded Zipf(alpha) rank in [1, n] by rejection-inversion. */
int64_t oracle_zipf_rank(uint64_t seed, uint64_t stream, uint64_t index,
                         int64_t n, double alpha);

/* Host cores usable by this process (sched_getaffinity). */
int32_t oracle_host_cores(void);

#ifdef __cplusplus
}
#endif

#endif /* XSE_ORACLE_H_ */
