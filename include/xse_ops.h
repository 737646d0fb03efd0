/* xse_ops.h: C ABI of the operator layer -- the host-buffer operators and
 * the table resource that XSE's processor graph calls.
 *
 * These mirror, with the same names, argument meanings and error messages:
 *   CpuEmbeddingLookupTransform   (data/kernels/cpu_embedding/
 *                                  cpu_embedding_lookup_transform.{h,cc})
 *   DenseCpuEmbeddingLookupTransform (dense_cpu_embedding_lookup_transform.
 *                                  {h,cc})
 *   CpuEmbeddingEngineResource    (cpu_embedding_resource.{h,cc})
 * Inputs and outputs are host buffers (XSE HostBuffer: dtype, shape, base
 * pointer; runtime/core/host_buffer.h:134-400); the operators stage them to
 * the GPU, run the engine's kernels and return host outputs. Status codes and
 * xse_last_error() work as in xse_emb.h.
 */
#ifndef XSE_OPS_H_
#define XSE_OPS_H_

#include <stdint.h>

#include "xse_emb.h"

#ifdef __cplusplus
extern "C" {
#endif

/* Element types of host buffers (xla::ifrt::DType kinds used on this path).
 * XSE_HB_INVALID marks an uninitialized ("Empty host buffer"). */
enum {
  XSE_HB_INVALID = 0,
  XSE_HB_S32 = 1,
  XSE_HB_S64 = 2,
  XSE_HB_F32 = 3,
};

#define XSE_HB_MAX_RANK 8

/* A host tensor view. Buffers made by xse_host_buffer_alloc (and every
 * operator output) live in pinned memory owned by the library. */
typedef struct {
  void* data;
  int32_t dtype; /* XSE_HB_* */
  int32_t rank;
  int64_t dims[XSE_HB_MAX_RANK];
} xse_host_buffer;

/* Allocates a pinned host buffer (64-byte aligned, as HostBuffer::flat<T>
 * requires, runtime/core/host_buffer.h:279-330). */
int xse_host_buffer_alloc(int32_t dtype, int32_t rank, const int64_t* dims,
                          xse_host_buffer* out);
/* Frees a buffer from xse_host_buffer_alloc or an operator output. */
void xse_host_buffer_free(xse_host_buffer* buffer);

/* ---------------------------------------------------------------------------
 * CpuEmbeddingEngineResource (cpu_embedding_resource.{h,cc}).
 * ------------------------------------------------------------------------- */
typedef struct xse_resource xse_resource;

/* LoadImpl (cpu_embedding_resource.cc:229-253): assets are (name, path)
 * pairs; the one named "__jce_manifest__" is the CpuEmbeddingManifest text
 * proto, every other asset a raw little-endian table "<name>.bin" of
 * vocab_size x embedding_dim elements. The manifest's optional per-table
 * `data_type` field (FLOAT32 default, BFLOAT16, INT8_ROWWISE) extends the
 * reference's fp32-only format; an INT8_ROWWISE asset holds the int8 rows
 * followed by vocab_size fp32 scales and vocab_size fp32 biases. Tables are
 * loaded into HBM of `device`. */
int xse_resource_load(const char* const* asset_names,
                      const char* const* asset_paths, int32_t num_assets,
                      int32_t device, xse_resource** out);
/* Placement of a resource's tables over the ranks of a sharded job, and the
 * host -> HBM upload. The reference loads every table into one host
 * (cpu_embedding_resource.cc:97-225); here rank `rank` of `world` keeps:
 *   XSE_SHARD_NONE      every table whole (world and rank ignored);
 *   XSE_SHARD_TABLEWISE table i of the manifest (in manifest order) when
 *                       i mod world == rank -- the features of other ranks'
 *                       tables are not registered, their embedding
 *                       dimensions still answer GetEmbeddingDim;
 *   XSE_SHARD_ROWWISE   rows [vocab r / world, vocab (r+1) / world) of every
 *                       table (the engine's shard window), read from the
 *                       asset at that offset.
 * Rows are read from the asset file (pread) into pinned staging buffers of
 * chunk_bytes (0: 32 MiB; < 0: one pageable cudaMemcpy per table from the
 * memory-mapped asset) by upload_threads host threads (0: 8),
 * double-buffered so that reading the file overlaps the DMA of the previous
 * chunk. */
enum { XSE_SHARD_NONE = 0, XSE_SHARD_TABLEWISE = 1, XSE_SHARD_ROWWISE = 2 };
typedef struct {
  int32_t world;
  int32_t rank;
  int32_t sharding;       /* XSE_SHARD_* */
  int32_t upload_threads;
  int64_t chunk_bytes;
} xse_load_options;

/* xse_resource_load with a placement and upload options (NULL: as
 * xse_resource_load). */
int xse_resource_load_sharded(const char* const* asset_names,
                              const char* const* asset_paths,
                              int32_t num_assets, int32_t device,
                              const xse_load_options* options,
                              xse_resource** out);
/* An empty resource whose engine is filled through xse_resource_engine
 * (the reference's tests build resources this way). */
int xse_resource_create(int32_t device, xse_resource** out);
void xse_resource_destroy(xse_resource* resource);
/* The engine the resource owns (CpuEmbeddingEngineResource::Get). */
xse_engine* xse_resource_engine(xse_resource* resource);
/* GetEmbeddingDim (cpu_embedding_resource.cc:255-263). */
int xse_resource_embedding_dim(xse_resource* resource, const char* feature,
                               int32_t* dim);
/* RegisterEmbeddingDimForTest (cpu_embedding_resource.h:42-45). */
int xse_resource_register_embedding_dim(xse_resource* resource,
                                        const char* feature, int32_t dim);

/* ---------------------------------------------------------------------------
 * CpuEmbeddingLookupTransform (cpu_embedding_lookup_transform.{h,cc}).
 * ------------------------------------------------------------------------- */
typedef struct xse_lookup_transform xse_lookup_transform;

/* Create (cpu_embedding_lookup_transform.cc:87-151). */
int xse_lookup_transform_create(xse_resource* resource,
                                const char* const* feature_names,
                                int32_t num_features, int32_t dense_lookup,
                                const char* const* output_feature_names,
                                int32_t num_output_names,
                                int64_t embedding_dim,
                                xse_lookup_transform** out);
void xse_lookup_transform_destroy(xse_lookup_transform* transform);

/* operator()(ids, row_pointers, weights) (cpu_embedding_lookup_transform.cc:
 * 244-356, checks as ValidateLookupInputs :159-242): one entry per feature in each list (row_pointers and weights
 * are ignored with dense_lookup). On success writes num_features pinned F32
 * outputs of shape [batch, dim] into outputs (free each with
 * xse_host_buffer_free). `stream` is the CUDA stream to run on (NULL: the
 * legacy default stream). */
int xse_lookup_transform_run(xse_lookup_transform* transform,
                             const xse_host_buffer* ids, int32_t num_ids,
                             const xse_host_buffer* row_pointers,
                             int32_t num_row_pointers,
                             const xse_host_buffer* weights,
                             int32_t num_weights, xse_host_buffer* outputs,
                             void* stream);

/* ---------------------------------------------------------------------------
 * DenseCpuEmbeddingLookupTransform (dense_cpu_embedding_lookup_transform.
 * {h,cc}).
 * ------------------------------------------------------------------------- */
typedef struct xse_dense_lookup_transform xse_dense_lookup_transform;

/* Create (dense_cpu_embedding_lookup_transform.cc:76-99). */
int xse_dense_lookup_transform_create(xse_resource* resource,
                                      const char* const* feature_names,
                                      int32_t num_features, int64_t pad_value,
                                      const char* const* output_feature_names,
                                      int32_t num_output_names,
                                      xse_dense_lookup_transform** out);
void xse_dense_lookup_transform_destroy(xse_dense_lookup_transform* t);

/* operator()(dense_ids_list) (dense_cpu_embedding_lookup_transform.cc:
 * 148-268): per feature a [batch, seq] S32/S64 buffer; ids equal to
 * pad_value are dropped and an all-pad row keeps one pad_value id. Writes
 * num_features pinned F32 [batch, dim] outputs. */
int xse_dense_lookup_transform_run(xse_dense_lookup_transform* transform,
                                   const xse_host_buffer* dense_ids,
                                   int32_t num_inputs,
                                   xse_host_buffer* outputs, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* XSE_OPS_H_ */
