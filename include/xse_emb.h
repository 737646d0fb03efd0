/* xse_emb.h: C ABI of the B200 embedding-bag and DLRM interaction engine.
 *
 * This is the drop-in boundary for the CPU embedding path of
 * openxla/xla-serving. Each entry point names the reference interface it
 * replaces (paths are relative to the reference project). Plain pointers and
 * sizes only: no C++ or torch types cross this boundary, and no C++ exception
 * escapes it. Functions return 0 on success or an absl::StatusCode number;
 * xse_last_error() returns the message of the calling thread's last failure.
 *
 * Device pointers are CUDA global-memory pointers of the engine's device.
 * Streams are cudaStream_t values passed as void* (NULL = legacy default).
 */
#ifndef XSE_EMB_H_
#define XSE_EMB_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define XSE_ABI_VERSION 1

/* absl::StatusCode numbering (the reference returns absl::Status). */
enum {
  XSE_OK = 0,
  XSE_CANCELLED = 1,
  XSE_UNKNOWN = 2,
  XSE_INVALID_ARGUMENT = 3,
  XSE_DEADLINE_EXCEEDED = 4,
  XSE_NOT_FOUND = 5,
  XSE_ALREADY_EXISTS = 6,
  XSE_RESOURCE_EXHAUSTED = 8,
  XSE_FAILED_PRECONDITION = 9,
  XSE_UNIMPLEMENTED = 12,
  XSE_INTERNAL = 13,
};

/* Table storage types. F32 is the reference's only batched type
 * (data/cpu_embedding/cc/embedding_bag.cc:74-87); BF16 and I8_ROWWISE
 * (int8 row + per-row fp32 scale and bias) extend it. Every type pools in
 * fp32. */
enum { XSE_DT_F32 = 0, XSE_DT_BF16 = 1, XSE_DT_I8_ROWWISE = 2 };

/* Combine modes, numbered as CpuEmbeddingManifest.EmbeddingTable.CombineMode
 * (data/kernels/cpu_embedding/cpu_embedding.proto:21-26). */
enum { XSE_COMBINE_SUM = 1, XSE_COMBINE_MEAN = 2, XSE_COMBINE_SQRTN = 3 };

/* Index element types for ids and CSR offsets. */
enum { XSE_INDEX_I32 = 0, XSE_INDEX_I64 = 1 };

/* Table placement for xse_engine_add_table. */
enum {
  XSE_PLACE_COPY_FROM_HOST = 0,   /* rows are host memory; copied to HBM */
  XSE_PLACE_COPY_FROM_DEVICE = 1, /* rows are device memory; copied */
  XSE_PLACE_ADOPT_DEVICE = 2,     /* rows are device memory; borrowed, must
                                     outlive the engine */
};

/* Execution flags for xse_engine_execute_batch. */
enum {
  /* Default: a validation pass runs first and nothing is written unless the
   * whole group is valid (embedding_bag.cc:477-497). The call synchronizes
   * the stream and returns the group's status. */
  XSE_EXEC_STRICT = 0,
  /* Ids and offsets are checked inside the pooling kernel instead of in a
   * separate pass. Errors are still reported, but outputs of a failing group
   * are unspecified. */
  XSE_EXEC_FUSED = 1,
  /* Do not synchronize: the result is read later with xse_status_wait. */
  XSE_EXEC_ASYNC = 2,
};

/* Message of this thread's last failing call ("" if none). */
const char* xse_last_error(void);
int32_t xse_abi_version(void);

/* ---------------------------------------------------------------------------
 * Engine: tables and feature specs resident in HBM.
 * Replaces CpuEmbeddingEngine (data/cpu_embedding/cc/cpu_embedding_engine.h:
 * 41-103) and the table type EmbeddingTable (embedding_table.h:39-96).
 * ------------------------------------------------------------------------- */
typedef struct xse_engine xse_engine;

typedef struct {
  int32_t device; /* CUDA device ordinal the engine's tables live on */
  int32_t reserved;
} xse_engine_options;

/* Replaces CpuEmbeddingEngine::CpuEmbeddingEngine(Options)
 * (cpu_embedding_engine.cc:51-56). */
int xse_engine_create(const xse_engine_options* options, xse_engine** out);
void xse_engine_destroy(xse_engine* engine);

typedef struct {
  const char* name;
  int32_t dtype;     /* XSE_DT_* */
  int32_t combine;   /* XSE_COMBINE_* */
  int64_t vocab;     /* global row count; ids are validated against it */
  int32_t dim;       /* embedding dimension */
  int32_t placement; /* XSE_PLACE_* */
  const void* rows;  /* [row_end-row_begin, dim] row-major, dtype elements */
  const float* scale; /* I8_ROWWISE: [row_end-row_begin] per-row scale */
  const float* bias;  /* I8_ROWWISE: [row_end-row_begin] per-row bias */
  /* Row-wise shard window: this engine holds global rows [row_begin,
   * row_end). Ids outside the window are skipped (they belong to another
   * shard). row_begin = row_end = 0 means the whole table. */
  int64_t row_begin;
  int64_t row_end;
} xse_table_desc;

/* Replaces EmbeddingTable::Create (embedding_table.cc:56-70) followed by
 * CpuEmbeddingEngine::AddLocalTable (cpu_embedding_engine.cc:71-81):
 * XSE_ALREADY_EXISTS on a duplicate name. */
int xse_engine_add_table(xse_engine* engine, const xse_table_desc* table);

/* Replaces CpuEmbeddingEngine::RegisterFeatureSpec (cpu_embedding_engine.cc:
 * 60-69) with FeatureSpec{name, table_name, max_sequence_length}
 * (feature_spec.h:25-29). */
int xse_engine_register_feature(xse_engine* engine, const char* feature,
                                const char* table,
                                int32_t max_sequence_length);

/* Replaces CpuEmbeddingEngine::Clear (cpu_embedding_engine.cc:83-89). */
int xse_engine_clear(xse_engine* engine);

typedef struct {
  int32_t dtype, combine, dim, reserved;
  int64_t vocab, row_begin, row_end;
  const void* rows; /* device */
} xse_table_info;

/* Replaces CpuEmbeddingEngine::GetLocalTable (cpu_embedding_engine.cc:
 * 347-356). */
int xse_engine_table_info(xse_engine* engine, const char* table,
                          xse_table_info* out);
/* Replaces CpuEmbeddingEngine::GetFeatureSpec (cpu_embedding_engine.cc:
 * 336-345), returning the feature's table name into buf. */
int xse_engine_feature_table(xse_engine* engine, const char* feature,
                             char* buf, int32_t buflen,
                             int32_t* max_sequence_length);

/* ---------------------------------------------------------------------------
 * Pooled lookup.
 * Replaces CpuEmbeddingEngine::ExecuteBatch(Span<FeatureBatchInput<float>>)
 * (cpu_embedding_engine.h:55-62,79, cpu_embedding_engine.cc:168-217) and
 * internal::ExecuteEmbeddingBagBatch (embedding_bag.h:87-90). Inputs and
 * outputs are device memory owned by the caller.
 * ------------------------------------------------------------------------- */
typedef struct {
  const char* feature_name;
  const void* ids;      /* device, num_ids elements of ids_type */
  int32_t ids_type;     /* XSE_INDEX_* */
  int32_t offsets_type; /* XSE_INDEX_*; the reference uses int32 */
  int64_t num_ids;
  const void* offsets;  /* device, absolute CSR offsets, num_offsets entries */
  int64_t num_offsets;  /* number of bags + 1 */
  const float* weights; /* device per-id weights, or NULL */
  int64_t num_weights;
  float* output;        /* device, bag b at output + b*output_stride */
  int64_t output_stride; /* floats between bags; 0 means dim */
} xse_bag_request;

/* Device-side status block of one execution (scratch owned by the caller).
 * It holds up to max_requests request slots. */
typedef struct xse_status xse_status;
int xse_status_create(int32_t max_requests, xse_status** out);
void xse_status_destroy(xse_status* status);

/* Runs one group of requests. status may be NULL unless XSE_EXEC_ASYNC is
 * set; a NULL status uses an engine-owned block and serializes such calls.
 * Errors use the reference's messages and request prefix
 * ("FP32 embedding-bag request %d: ...", embedding_bag.cc:229-233).
 * The engine chooses its pooling kernel per launch signature (tables,
 * layout, request count, batch size class): for large launches the first
 * four executions of a signature alternate two kernels with CUDA events
 * around each launch, and the faster is kept. Results are bit-identical
 * whichever kernel runs. */
int xse_engine_execute_batch(xse_engine* engine, const xse_bag_request* reqs,
                             int32_t n, void* stream, int32_t flags,
                             xse_status* status);

/* Waits for the stream and returns the status of the last group executed
 * with this block (and its message through xse_last_error). */
int xse_status_wait(xse_status* status, void* stream);

/* Replaces CpuEmbeddingEngine::Execute(Span<const FeatureBatchCsrInput>)
 * (cpu_embedding_engine.cc:91-166), the per-feature path. For each request,
 * a feature whose spec has max_sequence_length == 0 is pooled in its table's
 * type (AssembleCombinedEmbeddings, compute_activations.cc:36-154): fp32 as
 * xse_engine_execute_batch, bf16 accumulating in bf16 (every operation
 * rounded to bf16), into output = [num_bags, dim]; a sequence feature
 * gathers the rows of each sample's first max_sequence_length ids, zero
 * padded, into output = [num_bags, max_sequence_length, dim] in the table's
 * type (LookupEmbeddingSequence, compute_activations.cc:187-224, 321-346).
 * `output` points to that array (bf16 as raw 16-bit values); output_stride
 * is ignored. Requests follow FeatureBatchCsrInput (feature_batch_csr_
 * input.cc:33-57): offsets start at 0 and end at num_ids, never decrease;
 * weights empty or one per id (none for a sequence feature). Tables fp32 or
 * bf16, whole (no shard window). At most 64 requests; synchronous; checked
 * before any output is written; messages as the reference's. */
int xse_engine_execute_legacy(xse_engine* engine, const xse_bag_request* reqs,
                              int32_t n, void* stream);

/* Allocation-free variant of xse_engine_execute_batch (strict mode,
 * synchronous). No counterpart in the reference, which pools on the host.
 *
 * For callers that must not allocate GPU memory while serving a request:
 * code running inside a host framework that owns every device buffer (an
 * XLA custom call or a serving runtime with its own pre-sized arena), or a
 * latency-critical thread where a cudaMalloc would synchronize the device.
 * The caller passes inputs and outputs as for xse_engine_execute_batch; the
 * per-call validation status that the regular call keeps in a status block
 * lives instead in one fixed array in device memory, sized for at most
 * XSE_NOALLOC_MAX_REQUESTS requests (larger groups are rejected with
 * XSE_INVALID_ARGUMENT). Every device that loads this library holds that
 * array (about 1 KB) until the process exits. The call allocates no device
 * or pinned memory and calls no allocating library routine.
 *
 * The first call on a device looks up the array's device address
 * (cudaGetSymbolAddress); make that first call outside any CUDA stream
 * capture. All calls share the one array and clear it at their start, so
 * calls that overlap on the GPU (from several host threads or streams at
 * once) race on it: serialize them. Errors are resolved in the order of
 * xse_engine_execute_batch (request by request: early argument errors,
 * offsets, null ids or weights, out-of-range ids; output isolation last),
 * with the same codes and messages. */
#define XSE_NOALLOC_MAX_REQUESTS 64
int xse_engine_execute_batch_noalloc(xse_engine* engine,
                                     const xse_bag_request* reqs, int32_t n,
                                     void* stream);

/* Number of CUDA kernels the last xse_engine_execute_batch on this thread
 * launched. */
int32_t xse_last_launch_count(void);

/* Kernel timing (tracing aid; the reference traces with tsl TraceMe spans,
 * data/processor/cc/core/graph/graph_executor.cc:62,111). With period n > 0,
 * every n-th xse_engine_execute_batch from now on (the first, the (n+1)-th,
 * ...) records CUDA events on its stream around its pooling kernels; 0 turns
 * timing off. An event pair costs a few microseconds of stream time and
 * serialises the kernels it separates, so a period above 1 keeps the timed
 * executions representative of untimed ones. xse_engine_profile_read waits
 * for the recorded events and returns the summed pooling time, the number of
 * timed executions and (when `calls` is non-null) the number of executions,
 * timed or not, since profiling was set or last read; the read restarts the
 * sampling. */
int xse_engine_set_profiling(xse_engine* engine, int32_t period);
int xse_engine_profile_read(xse_engine* engine, double* pool_ms,
                            int64_t* executions, int64_t* calls);
/* As xse_engine_profile_read, and also the validation kernels' summed time
 * (from an event recorded before them to the one before the pooling
 * kernels) and the number of timed executions that ran them
 * (validate_ms / validated may be NULL). The events serialise the
 * validation kernels with the pooling kernels that would otherwise overlap
 * them (programmatic dependent launch), so this is each kernel's own
 * duration, not its share of an untimed execution. Same tracing role as
 * xse_engine_profile_read (graph_executor.cc:62,111). */
int xse_engine_profile_read_stages(xse_engine* engine, double* validate_ms,
                                   int64_t* validated, double* pool_ms,
                                   int64_t* executions, int64_t* calls);

/* ---------------------------------------------------------------------------
 * DLRM dot interaction. No counterpart in the reference: its DLRM bundle uses
 * DCN-v2 (examples/dlrm/model_jce.py:141-164); this computes the pairwise dot
 * interaction that replaces it. Z_b = [dense_b; pooled_b,0 .. pooled_b,T-1],
 * out_b = [dense_b, Z_b[i].Z_b[j] for i < j in row-major order].
 * dense is [batch, dim], pooled is [batch, T, dim], out is
 * [batch, dim + (T+1)T/2], all fp32 device memory.
 * ------------------------------------------------------------------------- */
int xse_dot_interaction(const float* dense, const float* pooled,
                        int64_t batch, int32_t num_tables, int32_t dim,
                        float* out, void* stream);

/* Pooled lookup fused with the dot interaction: request t (t = 0..n-1, each
 * with `batch` bags over a whole table, all tables of one dimension) pools
 * feature t of every sample, and out row b (every out_stride floats, at least
 * dim + (n+1)n/2) receives [dense_b, Z_b[i].Z_b[j] for i < j] with the pooled
 * rows in Z_b as xse_dot_interaction has them, zeros up to out_stride. The
 * requests' output fields are not used: where one kernel serves the tables'
 * layout (fp32 or bf16 rows of 32 16-byte vectors -- dim 128 fp32 or 256
 * bf16 --, one weighting mode for all requests, n <= 31, 16-byte aligned
 * dense rows) the pooled rows of a sample are gathered into shared memory
 * and its interaction computed there, so the pooled [batch, n, dim] tensor
 * never reaches HBM; otherwise the bags are pooled into scratch and the
 * interaction kernel runs after. The pooled
 * values equal xse_engine_execute_batch's bit for bit. Flags, status,
 * validation and errors as xse_engine_execute_batch (XSE_EXEC_STRICT
 * validates every request before the kernel runs); when the call reports an
 * error the contents of out are unspecified. No counterpart in the reference
 * (its DLRM feeds the pooled rows to a DCN-v2 cross network,
 * examples/dlrm/model_jce.py:141-164). */
int xse_engine_execute_interaction(xse_engine* engine,
                                   const xse_bag_request* reqs, int32_t n,
                                   const float* dense, int64_t dense_stride,
                                   int64_t batch, float* out,
                                   int64_t out_stride, void* stream,
                                   int32_t flags, xse_status* status);

/* xse_engine_execute_interaction writing the split operands of the next
 * layer's three-pass TF32 GEMM (xse_linear_forward_tf32x3) instead of the
 * values: out_hi receives each value rounded to TF32 (as xse_tf32_split) and
 * out_lo the exact remainder (out_hi + out_lo == the value), both rows of
 * out_stride floats. The fused kernel writes them directly, so the top MLP's
 * first layer needs no separate split pass over the interaction rows. */
int xse_engine_execute_interaction_tf32(
    xse_engine* engine, const xse_bag_request* reqs, int32_t n,
    const float* dense, int64_t dense_stride, int64_t batch, float* out_hi,
    float* out_lo, int64_t out_stride, void* stream, int32_t flags,
    xse_status* status);

/* ---------------------------------------------------------------------------
 * Seeded synthetic inputs on the device (counter-based, reproducible on the
 * host). Used by tests and benchmarks; no reference counterpart (the
 * reference generates with numpy, examples/dlrm/export_jce.py:73-118).
 * ------------------------------------------------------------------------- */
/* Rows [row0, row0+nrows) of table `table`: value = -0.05 + 0.1*u. For
 * I8_ROWWISE: q uniform in [-127,127], scale U(1e-3,1e-2), bias
 * U(-0.1,0.1). */
int xse_synth_table(void* rows, float* scale, float* bias, int32_t dtype,
                    uint64_t seed, uint64_t table, int64_t row0,
                    int64_t nrows, int32_t dim, void* stream);
/* n bag lengths uniform in [lo, hi]. */
int xse_synth_lengths(int64_t* lengths, int64_t n, int32_t lo, int32_t hi,
                      uint64_t seed, uint64_t table, void* stream);
/* n ids over [0, vocab): uniform when zipf_alpha <= 0, else bounded
 * Zipf(alpha) ranks mapped to rows by (rank-1)*perm_mul + perm_add mod
 * vocab (perm_mul coprime to vocab). Element i uses counter index0 + i. */
int xse_synth_ids(int64_t* ids, int64_t n, int64_t vocab, double zipf_alpha,
                  uint64_t perm_mul, uint64_t perm_add, uint64_t seed,
                  uint64_t table, int64_t index0, void* stream);
/* n weights uniform in [0, 1). */
int xse_synth_weights(float* weights, int64_t n, uint64_t seed,
                      uint64_t table, int64_t index0, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* XSE_EMB_H_ */
