/* Input side of table-wise sharding: data-parallel ids -> table owners.
 *
 * No counterpart in the reference (its engine runs in one host process,
 * data/cpu_embedding/cc/cpu_embedding_engine.h:41-103). In a data-parallel
 * input layout every rank holds the CSR ids of all tables for its own sample
 * block; table-wise pooling needs, on the owner of table t, table t's ids
 * for every sample block. Each rank packs, per destination rank, the id
 * ranges of the destination's tables into one contiguous chunk with offsets
 * rebased into that chunk (one launch), and an all-to-all (NCCL) delivers
 * the chunks; the owner then pools block s of table t straight from source
 * s's chunk (absolute offsets, no further copy). The kernels below are the
 * packing step; the exchange is the caller's (torch.distributed in the
 * Python package).
 *
 * Status codes and xse_last_error() as in xse_emb.h.
 */
#ifndef XSE_SHARD_H_
#define XSE_SHARD_H_

#include <stdint.h>

#include "xse_emb.h"

#ifdef __cplusplus
extern "C" {
#endif

/* One CSR slice: bags [0, num_bags) of (ids, offsets[, weights]), all device
 * memory. offsets holds num_bags + 1 absolute entries of offsets_type;
 * the ids read are [offsets[0], offsets[num_bags]), which must lie within
 * [0, num_ids). The pack writes that id range (and the weights of the same
 * positions, when both weights and dst_weights are set) to dst_ids
 * (dst_weights) and offsets[i] - offsets[0] + dst_base (int64) to
 * dst_offsets[i], i = 0..num_bags. dst ids have the source's id type. */
typedef struct {
  const void* ids;
  const void* offsets;
  const float* weights;
  int64_t num_ids;
  int64_t num_bags;
  int32_t ids_type;     /* XSE_INDEX_* */
  int32_t offsets_type; /* XSE_INDEX_* */
  void* dst_ids;
  int64_t* dst_offsets;
  float* dst_weights;
  int64_t dst_base;
} xse_csr_segment;

/* extents[k] (device int64, n entries) = offsets[num_bags] - offsets[0] of
 * segment k, or -1 when that range is not within [0, num_ids) (negative
 * first offset, decreasing ends, or past the ids). Reads two offsets per
 * segment; one launch. */
int xse_csr_extents(const xse_csr_segment* segs, int32_t n, int64_t* extents,
                    void* stream);

/* Packs every segment as described above; one launch (grid over segments
 * and their elements). Segments whose range is invalid (extent -1), or
 * with ids to copy and a NULL dst_ids, are skipped. */
int xse_csr_pack(const xse_csr_segment* segs, int32_t n, void* stream);

/* ---------------------------------------------------------------------------
 * Sharded execution, driven from C or C++.
 *
 * Replaces CpuEmbeddingEngine::ExecuteBatch (data/cpu_embedding/cc/
 * cpu_embedding_engine.h:79, cpu_embedding_engine.cc:168-217) when the
 * tables of one job are sharded over the GPUs of a node, one process (or
 * host thread) per GPU; the reference keeps every table in one host
 * process and has no counterpart. Each rank owns an xse_engine holding its
 * shard of the tables, one NCCL communicator over the job's ranks
 * (xse_shard_comm) and one exchange (xse_shard_exchange) that runs a step:
 * it pools this rank's tables and returns every sample block's pooled rows
 * to the rank that owns the sample.
 *
 *   table-wise (XSE_SHARD_TABLE_*): global table t lives on rank t mod W.
 *     Each rank passes its tables' requests over the whole batch; rank r
 *     ends with samples [r B/W, (r+1) B/W) of every table.
 *       PEER: the pooling kernel stores every block straight into its
 *         owner's output slot over NVLink (CUDA IPC mappings set up through
 *         the communicator), then a stream-ordered flag barrier; no copy.
 *       A2A: pooling into a send buffer, then one NCCL all-to-all (grouped
 *         send/recv) and a reorder into the output layout.
 *       PIPELINED: one pooling group per destination block, each block's
 *         send/recv on a communication stream while the next is pooled.
 *   row-wise (XSE_SHARD_ROW): every table's rows are split over the ranks
 *     (engine tables added with their row window); every rank passes the
 *     requests of all tables over the whole batch, pools partial sums and
 *     NCCL reduce-scatters them (chunked, overlapped with the pooling).
 *
 * NCCL is loaded at run time (libnccl.so.2; the copy already loaded in the
 * process when there is one). Every rank must issue the same calls in the
 * same order. Status codes and xse_last_error() as in xse_emb.h.
 * ------------------------------------------------------------------------- */
#define XSE_SHARD_ID_BYTES 128
#define XSE_SHARD_MAX_RANKS 8

typedef struct xse_shard_comm xse_shard_comm;

/* A new communicator's NCCL unique id (ncclGetUniqueId): one rank creates
 * it and hands the bytes to every rank over any host channel. */
int xse_shard_unique_id(unsigned char id[XSE_SHARD_ID_BYTES]);
/* This rank's communicator on `device` (ncclCommInitRank); every rank of
 * the job calls it with the same id. world <= XSE_SHARD_MAX_RANKS. */
int xse_shard_comm_create(int32_t device, int32_t world, int32_t rank,
                          const unsigned char id[XSE_SHARD_ID_BYTES],
                          xse_shard_comm** out);
/* Wraps a communicator the caller created (an ncclComm_t passed as a
 * pointer) for `device`; the caller keeps ownership. */
int xse_shard_comm_adopt(void* nccl_comm, int32_t device, int32_t world,
                         int32_t rank, xse_shard_comm** out);
/* ncclCommAbort: collectives in flight or issued later end with an error
 * (failure handling when another rank is gone); the communicator cannot be
 * used again. */
int xse_shard_comm_abort(xse_shard_comm* comm);
void xse_shard_comm_destroy(xse_shard_comm* comm);

enum {
  XSE_SHARD_TABLE_PEER = 0,
  XSE_SHARD_TABLE_A2A = 1,
  XSE_SHARD_TABLE_PIPELINED = 2,
  XSE_SHARD_ROW = 3,
};

typedef struct {
  int32_t mode;       /* XSE_SHARD_* */
  int32_t num_tables; /* table-wise: tables of the whole job; row-wise: the
                         tables every rank holds a window of */
  int32_t dim;        /* embedding dimension of every table */
  int32_t chunks;     /* row-wise: pieces pooled and reduce-scattered in
                         turn (0 or 1: one) */
  int64_t batch;      /* samples of the whole batch, divisible by the world
                         size (row-wise: by world * chunks) */
  int64_t spin_limit; /* PEER: polls (~1 us each) before a barrier wait gives
                         up; 0: about 2 s */
} xse_shard_plan;

typedef struct xse_shard_exchange xse_shard_exchange;

/* Sets up one exchange for `engine` (which holds this rank's tables) over
 * `comm`: output slots (PEER: mapped into every rank; a collective call),
 * send buffers, a status block and streams. */
int xse_shard_exchange_create(xse_engine* engine, xse_shard_comm* comm,
                              const xse_shard_plan* plan,
                              xse_shard_exchange** out);

/* Flags of xse_shard_exchange_run. */
#define XSE_SHARD_DEFER_WAIT 1

/* One step on `stream`. features[k] is the whole-batch request of this
 * rank's k-th table: table-wise, global table rank + k * world (n = the
 * number of tables this rank holds); row-wise, table k (n = num_tables).
 * Their output and output_stride are ignored. Inputs are read by work
 * queued on `stream`; they must stay valid until it has run.
 *
 * *out (if out is not NULL) receives this rank's pooled rows:
 * [batch / world][num_tables][dim] fp32, sample-major, global table order.
 * Without XSE_SHARD_DEFER_WAIT they are ready for work queued on `stream`
 * after the call. With it (PEER), `stream` is not ordered after the
 * step's barrier, so the next step's pooling can overlap it; call
 * xse_shard_exchange_ready before reading the rows. Readers of a step's
 * rows must be queued before the next call of run (the slot is then
 * reused). Execution is asynchronous: validation errors, a barrier that
 * gave up and NCCL errors are reported by xse_shard_exchange_check. */
int xse_shard_exchange_run(xse_shard_exchange* ex,
                           const xse_bag_request* features, int32_t n,
                           int32_t flags, void* stream, float** out);
/* Orders `stream` after the last step's exchange (PEER with
 * XSE_SHARD_DEFER_WAIT; a no-op otherwise). */
int xse_shard_exchange_ready(xse_shard_exchange* ex, void* stream);
/* Waits for `stream` and the exchange's own streams and reports the first
 * error of the steps so far: a request error (the messages of
 * xse_engine_execute_batch), DEADLINE_EXCEEDED when a peer barrier gave up
 * waiting for a rank, INTERNAL for an NCCL error. */
int xse_shard_exchange_check(xse_shard_exchange* ex, void* stream);
/* Frees the exchange (PEER: every rank must be done with the others'
 * slots first, e.g. after a host barrier). */
void xse_shard_exchange_destroy(xse_shard_exchange* ex);

#ifdef __cplusplus
}
#endif

#endif  /* XSE_SHARD_H_ */
