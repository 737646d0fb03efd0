/* Peer-memory exchange between the GPUs of one node (one process per GPU).
 *
 * No counterpart in the reference (its engine runs in one host process,
 * data/cpu_embedding/cc/cpu_embedding_engine.h:41-103). Table-wise sharded
 * pooling returns every sample block to the rank that owns the sample. Here
 * the pooling kernel does that itself: each rank maps the other ranks'
 * receive buffers (CUDA IPC over NVLink) and its bag requests write pooled
 * rows straight into the owner's buffer, so the exchange is the pooling
 * kernel's own stores and overlaps its gathers row by row. A flag barrier
 * then tells every rank that all blocks addressed to it have landed.
 *
 * Each rank creates a group (one cudaMalloc'd buffer holding the barrier
 * flags and `buffer_bytes` of data), passes its handle to every other rank
 * (any host channel), and connects with all handles in rank order. All calls
 * are stream-ordered; a barrier that waits longer than its spin limit (a
 * rank that never arrives) gives up, records the failure on the device and
 * returns, and xse_peer_group_check() then reports DEADLINE_EXCEEDED.
 * Status codes and xse_last_error() as in xse_emb.h.
 */
#ifndef XSE_PEER_H_
#define XSE_PEER_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define XSE_PEER_MAX_RANKS 8

typedef struct {
  unsigned char bytes[64]; /* a cudaIpcMemHandle_t */
} xse_ipc_handle;

typedef struct xse_peer_group xse_peer_group;

/* Allocates this rank's buffer on `device` (flags zeroed) and writes its IPC
 * handle to *handle. world <= XSE_PEER_MAX_RANKS. */
int xse_peer_group_create(int32_t device, int32_t world, int32_t rank,
                          int64_t buffer_bytes, xse_peer_group** out,
                          xse_ipc_handle* handle);
/* Maps the buffers of the other ranks: handles[q] is rank q's handle. */
int xse_peer_group_connect(xse_peer_group* group,
                           const xse_ipc_handle* handles, int32_t world);
/* Rank `peer`'s data region as mapped in this process (this rank's own
 * buffer for peer == rank); NULL before connect or for a bad rank. */
void* xse_peer_group_buffer(xse_peer_group* group, int32_t peer);
/* Stream-ordered barrier over all ranks: work queued on `stream` before it
 * (on every rank) happens before work queued after it (on every rank),
 * including stores into peer buffers. Each call advances the epoch; every
 * rank must call it the same number of times. spin_limit bounds the polls
 * of each wait (about 1 us each); 0 selects the default (about 2 s). */
int xse_peer_group_barrier(xse_peer_group* group, int64_t spin_limit,
                           void* stream);
/* Waits for `stream` and reports DEADLINE_EXCEEDED if any barrier so far
 * gave up waiting (the flag stays set). */
int xse_peer_group_check(xse_peer_group* group, void* stream);
/* Unmaps the peers' buffers and frees this rank's. Every rank must be done
 * with the others' buffers first (a host barrier). */
void xse_peer_group_destroy(xse_peer_group* group);

#ifdef __cplusplus
}
#endif

#endif /* XSE_PEER_H_ */
