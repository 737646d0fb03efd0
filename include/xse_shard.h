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

#ifdef __cplusplus
}
#endif

#endif  /* XSE_SHARD_H_ */
