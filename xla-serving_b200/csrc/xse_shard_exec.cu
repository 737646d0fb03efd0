// Sharded execution (include/xse_shard.h): an NCCL communicator per rank
// and the table-wise / row-wise exchange of one step, driven from C++.
//
// A step pools this rank's tables through the engine's ordinary group
// execution (validation + pooling kernels, asynchronous status ring) with
// requests whose outputs point where each sample block must end up:
//   PEER       the owner's output slot, mapped over NVLink (the pooling
//              kernel's stores are the exchange), then the flag barrier of
//              xse_peer.cu on a side stream;
//   A2A        this rank's own block straight into the output, the other
//              blocks into a send buffer; one grouped NCCL send/recv and a
//              reorder of the received blocks into the output;
//   PIPELINED  the same per destination block, each block's send/recv on
//              a communication stream while the next block is pooled;
//   ROW        partial sums of every sample block, reduce-scattered by
//              NCCL per chunk on the communication stream.
// Requests over a sample block are the whole-batch request with its offsets
// pointer advanced to the block's first bag (absolute CSR offsets), so no
// input is copied.
//
// NCCL is resolved at run time with dlopen: the process usually has
// torch's copy loaded already, and the engine must not pin a second one.

#include <cuda_runtime.h>
#include <dlfcn.h>
#include <nccl.h>
#include <stdint.h>

#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/xse_emb.h"
#include "../../include/xse_peer.h"
#include "../../include/xse_shard.h"
#include "xse_internal.h"

namespace xse {
namespace {

int ShardFail(int code, const char* fmt, ...)
    __attribute__((format(printf, 2, 3)));
int ShardFail(int code, const char* fmt, ...) {
  char buf[512];
  va_list args;
  va_start(args, fmt);
  vsnprintf(buf, sizeof(buf), fmt, args);
  va_end(args);
  SetLastErrorMessage(buf);
  return code;
}

int ShardOk() {
  SetLastErrorMessage("");
  return XSE_OK;
}

// The NCCL entry points the exchange uses.
struct NcclApi {
  bool loaded = false;
  std::string error;
  ncclResult_t (*GetUniqueId)(ncclUniqueId*) = nullptr;
  ncclResult_t (*CommInitRank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*CommDestroy)(ncclComm_t) = nullptr;
  ncclResult_t (*CommAbort)(ncclComm_t) = nullptr;
  ncclResult_t (*CommGetAsyncError)(ncclComm_t, ncclResult_t*) = nullptr;
  const char* (*GetErrorString)(ncclResult_t) = nullptr;
  ncclResult_t (*GroupStart)() = nullptr;
  ncclResult_t (*GroupEnd)() = nullptr;
  ncclResult_t (*Send)(const void*, size_t, ncclDataType_t, int, ncclComm_t,
                       cudaStream_t) = nullptr;
  ncclResult_t (*Recv)(void*, size_t, ncclDataType_t, int, ncclComm_t,
                       cudaStream_t) = nullptr;
  ncclResult_t (*ReduceScatter)(const void*, void*, size_t, ncclDataType_t,
                                ncclRedOp_t, ncclComm_t,
                                cudaStream_t) = nullptr;
  ncclResult_t (*AllGather)(const void*, void*, size_t, ncclDataType_t,
                            ncclComm_t, cudaStream_t) = nullptr;
};

template <typename F>
bool Resolve(void* lib, const char* name, F* fn, std::string* error) {
  *fn = reinterpret_cast<F>(dlsym(lib, name));
  if (*fn == nullptr && error->empty()) {
    *error = std::string("libnccl.so.2 lacks ") + name;
  }
  return *fn != nullptr;
}

const NcclApi& Nccl() {
  static NcclApi api = [] {
    NcclApi a;
    void* lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (lib == nullptr) lib = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (lib == nullptr) {
      const char* why = dlerror();
      a.error = std::string("cannot load libnccl.so.2: ") +
                (why != nullptr ? why : "unknown error");
      return a;
    }
    bool ok = Resolve(lib, "ncclGetUniqueId", &a.GetUniqueId, &a.error);
    ok &= Resolve(lib, "ncclCommInitRank", &a.CommInitRank, &a.error);
    ok &= Resolve(lib, "ncclCommDestroy", &a.CommDestroy, &a.error);
    ok &= Resolve(lib, "ncclCommAbort", &a.CommAbort, &a.error);
    ok &= Resolve(lib, "ncclCommGetAsyncError", &a.CommGetAsyncError,
                  &a.error);
    ok &= Resolve(lib, "ncclGetErrorString", &a.GetErrorString, &a.error);
    ok &= Resolve(lib, "ncclGroupStart", &a.GroupStart, &a.error);
    ok &= Resolve(lib, "ncclGroupEnd", &a.GroupEnd, &a.error);
    ok &= Resolve(lib, "ncclSend", &a.Send, &a.error);
    ok &= Resolve(lib, "ncclRecv", &a.Recv, &a.error);
    ok &= Resolve(lib, "ncclReduceScatter", &a.ReduceScatter, &a.error);
    ok &= Resolve(lib, "ncclAllGather", &a.AllGather, &a.error);
    a.loaded = ok;
    return a;
  }();
  return api;
}

int NcclFail(ncclResult_t r, const char* what) {
  const NcclApi& n = Nccl();
  return ShardFail(XSE_INTERNAL, "NCCL %s: %s", what,
                   n.GetErrorString != nullptr ? n.GetErrorString(r)
                                               : "error");
}

int CudaFail(cudaError_t e, const char* what) {
  return ShardFail(XSE_INTERNAL, "%s: %s", what, cudaGetErrorString(e));
}

struct DeviceScope {
  int prev = -1;
  explicit DeviceScope(int device) {
    cudaGetDevice(&prev);
    if (prev != device) cudaSetDevice(device);
  }
  ~DeviceScope() {
    int cur = -1;
    cudaGetDevice(&cur);
    if (prev >= 0 && cur != prev) cudaSetDevice(prev);
  }
};

// Received blocks [q][block][T_q][dim] -> sample-major out[b][q + k W][dim]
// for every source q except `skip` (whose rows were pooled into out
// directly). One warp per (q, b, k) row, 16-byte copies.
__global__ void ReorderBlocksKernel(const float* __restrict__ recv,
                                    float* __restrict__ out, int64_t block,
                                    int32_t world, int32_t num_tables,
                                    int32_t dim, int32_t skip) {
  const int lane = threadIdx.x & 31;
  const int64_t warps =
      static_cast<int64_t>(gridDim.x) * (blockDim.x / 32);
  const int64_t rows = block * num_tables;  // over all sources
  const int vecs = dim / 4;
  for (int64_t w = static_cast<int64_t>(blockIdx.x) * (blockDim.x / 32) +
                   threadIdx.x / 32;
       w < rows; w += warps) {
    // Row w walks the receive buffer in order: source q's block holds
    // block * T_q rows, T_q = number of tables q owns.
    int64_t at = w;
    int32_t q = 0;
    int64_t base = 0;
    for (; q < world; ++q) {
      const int32_t tq = (num_tables - q + world - 1) / world;
      const int64_t n = block * tq;
      if (at < n) break;
      at -= n;
      base += n;
    }
    if (q >= world || q == skip) continue;
    const int32_t tq = (num_tables - q + world - 1) / world;
    const int64_t b = at / tq;
    const int32_t k = static_cast<int32_t>(at % tq);
    const int32_t g = q + k * world;
    const float4* src =
        reinterpret_cast<const float4*>(recv + (base + at) * dim);
    float4* dst = reinterpret_cast<float4*>(out + (b * num_tables + g) * dim);
    for (int c = lane; c < vecs; c += 32) dst[c] = src[c];
  }
}

}  // namespace
}  // namespace xse

struct xse_shard_comm {
  ncclComm_t comm = nullptr;
  bool owned = false;
  int32_t device = 0, world = 1, rank = 0;
};

struct xse_shard_exchange {
  xse_engine* engine = nullptr;
  xse_shard_comm* comm = nullptr;
  xse_shard_plan plan{};
  int32_t world = 1, rank = 0, num_local = 0, chunks = 1;
  int64_t block = 0, piece = 0;
  std::vector<int32_t> counts;      // tables per rank (table-wise)
  std::vector<int64_t> recv_off;    // float offset of source q's block
  int64_t out_floats = 0;           // block * num_tables * dim
  // Output slots: PEER rotates 3 slots of the mapped buffer.
  int32_t slots = 1;
  float* out_local = nullptr;       // non-PEER output (cudaMalloc)
  xse_peer_group* peers = nullptr;
  float* send = nullptr;            // A2A / PIPELINED: [W][block][T_l][D]
  float* recv = nullptr;            // A2A / PIPELINED: [q][block][T_q][D]
  float* partial = nullptr;         // ROW, W > 1: [chunks][W][piece][T][D]
  xse_status* status = nullptr;
  cudaStream_t side = nullptr;      // PEER barrier / NCCL stream
  cudaEvent_t pooled = nullptr;
  std::vector<cudaEvent_t> done;    // per slot (PEER) / last NCCL step
  std::vector<bool> done_valid;
  int64_t step = -1;
  int32_t slot = 0;
  bool pending_ready = false;
  std::vector<xse_bag_request> reqs;  // sample blocks of the feature requests
  std::vector<int32_t> owner;          // feature request of each block
  std::vector<float*> block_base;      // peer mode: destinations' slots
  std::vector<int64_t> block_offset;   // peer mode: feature k's column
};

namespace {

using xse::ShardFail;
using xse::ShardOk;

int64_t OffsetBytes(const xse_bag_request& r) {
  return r.offsets_type == XSE_INDEX_I64 ? 8 : 4;
}

// The request of bags [b0, b0 + bags) of `f`, written to out with stride.
xse_bag_request Slice(const xse_bag_request& f, int64_t b0, int64_t bags,
                      float* out, int64_t stride) {
  xse_bag_request r = f;
  r.offsets = static_cast<const char*>(f.offsets) + b0 * OffsetBytes(f);
  r.num_offsets = bags + 1;
  r.output = out;
  r.output_stride = stride;
  return r;
}

float* OutSlot(xse_shard_exchange* ex, int32_t peer, int32_t slot) {
  if (ex->peers == nullptr) return ex->out_local;
  char* base = static_cast<char*>(xse_peer_group_buffer(ex->peers, peer));
  return reinterpret_cast<float*>(base) + slot * ex->out_floats;
}

void ClearBlocks(xse_shard_exchange* ex) {
  ex->reqs.clear();
  ex->owner.clear();
}

void AddBlock(xse_shard_exchange* ex, int32_t k, const xse_bag_request& r) {
  ex->reqs.push_back(r);
  ex->owner.push_back(k);
}

// Pools the blocks in ex->reqs. The feature requests `f` are the execution's
// requests: errors name feature k, and the validation pass (when `validate`;
// the first execution of a step) reads each feature's ids once, however many
// blocks it is cut into.
int Execute(xse_shard_exchange* ex, const xse_bag_request* f, int32_t n,
            bool validate, cudaStream_t stream) {
  xse::PartSet parts{ex->reqs.data(), ex->owner.data(),
                     static_cast<int32_t>(ex->reqs.size()), validate};
  return xse::ExecuteParts(ex->engine, f, n, parts, stream, XSE_EXEC_ASYNC,
                           ex->status);
}

// Peer mode: every feature's block for destination d lands in d's slot at
// the feature's column, so the kernels take one blocked descriptor per
// feature (instead of one per feature and destination).
int ExecuteBlocked(xse_shard_exchange* ex, const xse_bag_request* f,
                   int32_t n, cudaStream_t stream) {
  xse::PartSet parts{ex->reqs.data(), ex->owner.data(),
                     static_cast<int32_t>(ex->reqs.size()), true};
  if (ex->world > 1 && ex->world <= xse::kMaxOutBlocks) {
    parts.blocks = ex->world;
    parts.block_bags = ex->block;
    parts.block_base = ex->block_base.data();
    parts.block_offset = ex->block_offset.data();
    parts.block_stride =
        static_cast<int64_t>(ex->plan.num_tables) * ex->plan.dim;
  }
  return xse::ExecuteParts(ex->engine, f, n, parts, stream, XSE_EXEC_ASYNC,
                           ex->status);
}

int SideAfter(xse_shard_exchange* ex, cudaStream_t stream) {
  cudaError_t e = cudaEventRecord(ex->pooled, stream);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(ex->side, ex->pooled, 0);
  return e == cudaSuccess ? XSE_OK : xse::CudaFail(e, "stream ordering");
}

int StreamAfterSide(xse_shard_exchange* ex, cudaStream_t stream) {
  cudaError_t e = cudaEventRecord(ex->done[0], ex->side);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(stream, ex->done[0], 0);
  return e == cudaSuccess ? XSE_OK : xse::CudaFail(e, "stream ordering");
}

int RunPeer(xse_shard_exchange* ex, const xse_bag_request* f, int32_t flags,
            cudaStream_t stream, float** out) {
  const int64_t i = ex->step + 1;
  const int32_t slot = static_cast<int32_t>(i % ex->slots);
  // Step i overwrites, on every rank, the slot of step i - 3. Each rank
  // queued that step's readers before its pooling of step i - 2, which the
  // barrier of step i - 2 waited for on every rank.
  const int32_t prev = static_cast<int32_t>((i + 1) % ex->slots);
  // A barrier that has already completed needs no wait node on the stream.
  if (i >= 2 && ex->done_valid[prev] &&
      cudaEventQuery(ex->done[prev]) != cudaSuccess) {
    (void)cudaGetLastError();  // cudaErrorNotReady is not an error here
    cudaError_t e = cudaStreamWaitEvent(stream, ex->done[prev], 0);
    if (e != cudaSuccess) return xse::CudaFail(e, "slot reuse wait");
  }
  const int32_t w = ex->world, d_ = ex->plan.dim, t = ex->plan.num_tables;
  ClearBlocks(ex);
  ex->block_base.assign(static_cast<size_t>(w), nullptr);
  ex->block_offset.assign(static_cast<size_t>(ex->num_local), 0);
  for (int32_t k = 0; k < ex->num_local; ++k) {
    ex->block_offset[k] = static_cast<int64_t>(ex->rank + k * w) * d_;
  }
  for (int32_t dest = 0; dest < w; ++dest) {
    float* slot_base = OutSlot(ex, dest, slot);
    ex->block_base[dest] = slot_base;
    for (int32_t k = 0; k < ex->num_local; ++k) {
      AddBlock(ex, k,
               Slice(f[k], dest * ex->block, ex->block,
                     slot_base + ex->block_offset[k],
                     static_cast<int64_t>(t) * d_));
    }
  }
  int code = ExecuteBlocked(ex, f, ex->num_local, stream);
  if (code != XSE_OK) return code;
  if (w > 1) {
    code = SideAfter(ex, stream);
    if (code != XSE_OK) return code;
    code = xse_peer_group_barrier(ex->peers, ex->plan.spin_limit, ex->side);
    if (code != XSE_OK) return code;
    cudaError_t e = cudaEventRecord(ex->done[slot], ex->side);
    if (e != cudaSuccess) return xse::CudaFail(e, "barrier event");
    ex->done_valid[slot] = true;
    if ((flags & XSE_SHARD_DEFER_WAIT) == 0) {
      e = cudaStreamWaitEvent(stream, ex->done[slot], 0);
      if (e != cudaSuccess) return xse::CudaFail(e, "barrier wait");
      ex->pending_ready = false;
    } else {
      ex->pending_ready = true;
    }
  }
  ex->step = i;
  ex->slot = slot;
  if (out != nullptr) *out = OutSlot(ex, ex->rank, slot);
  return ShardOk();
}

// Grouped send of block `dest` of the send buffer and receive of source
// `src`'s block, on `s`.
int SendRecv(xse_shard_exchange* ex, int32_t dest, int32_t src,
             cudaStream_t s) {
  const xse::NcclApi& n = xse::Nccl();
  const int64_t send_floats =
      ex->block * ex->num_local * static_cast<int64_t>(ex->plan.dim);
  ncclResult_t r = n.GroupStart();
  if (r == ncclSuccess) {
    r = n.Send(ex->send + dest * send_floats, send_floats, ncclFloat32, dest,
               ex->comm->comm, s);
  }
  if (r == ncclSuccess) {
    r = n.Recv(ex->recv + ex->recv_off[src],
               ex->block * ex->counts[src] * static_cast<int64_t>(ex->plan.dim),
               ncclFloat32, src, ex->comm->comm, s);
  }
  const ncclResult_t end = n.GroupEnd();
  if (r == ncclSuccess) r = end;
  return r == ncclSuccess ? XSE_OK : xse::NcclFail(r, "send/recv");
}

int Reorder(xse_shard_exchange* ex, cudaStream_t stream) {
  const int64_t rows = ex->block * ex->plan.num_tables;
  const int64_t blocks = std::min<int64_t>((rows + 7) / 8, 148 * 16);
  xse::ReorderBlocksKernel<<<static_cast<int>(std::max<int64_t>(blocks, 1)),
                             256, 0, stream>>>(
      ex->recv, ex->out_local, ex->block, ex->world, ex->plan.num_tables,
      ex->plan.dim, ex->rank);
  const cudaError_t e = cudaGetLastError();
  return e == cudaSuccess ? XSE_OK : xse::CudaFail(e, "reorder launch");
}

// Requests of destination block `dest`: the own block straight into the
// output (sample-major), the others into their send block.
void BlockRequests(xse_shard_exchange* ex, const xse_bag_request* f,
                   int32_t dest) {
  const int32_t w = ex->world, d_ = ex->plan.dim, t = ex->plan.num_tables;
  for (int32_t k = 0; k < ex->num_local; ++k) {
    if (dest == ex->rank) {
      const int32_t g = ex->rank + k * w;
      AddBlock(ex, k,
               Slice(f[k], dest * ex->block, ex->block,
                     ex->out_local + static_cast<int64_t>(g) * d_,
                     static_cast<int64_t>(t) * d_));
    } else {
      float* base = ex->send + dest * ex->block * ex->num_local * d_;
      AddBlock(ex, k,
               Slice(f[k], dest * ex->block, ex->block,
                     base + static_cast<int64_t>(k) * d_,
                     static_cast<int64_t>(ex->num_local) * d_));
    }
  }
}

int RunA2A(xse_shard_exchange* ex, const xse_bag_request* f,
           cudaStream_t stream) {
  ClearBlocks(ex);
  for (int32_t dest = 0; dest < ex->world; ++dest) {
    BlockRequests(ex, f, dest);
  }
  int code = Execute(ex, f, ex->num_local, true, stream);
  if (code != XSE_OK || ex->world == 1) return code;
  const xse::NcclApi& n = xse::Nccl();
  const int64_t send_floats =
      ex->block * ex->num_local * static_cast<int64_t>(ex->plan.dim);
  ncclResult_t r = n.GroupStart();
  for (int32_t q = 0; q < ex->world && r == ncclSuccess; ++q) {
    if (q == ex->rank) continue;
    r = n.Send(ex->send + q * send_floats, send_floats, ncclFloat32, q,
               ex->comm->comm, stream);
    if (r == ncclSuccess) {
      r = n.Recv(ex->recv + ex->recv_off[q],
                 ex->block * ex->counts[q] * static_cast<int64_t>(ex->plan.dim),
                 ncclFloat32, q, ex->comm->comm, stream);
    }
  }
  const ncclResult_t end = n.GroupEnd();
  if (r == ncclSuccess) r = end;
  if (r != ncclSuccess) return xse::NcclFail(r, "all-to-all");
  return Reorder(ex, stream);
}

int RunPipelined(xse_shard_exchange* ex, const xse_bag_request* f,
                 cudaStream_t stream) {
  const int32_t w = ex->world, r = ex->rank;
  for (int32_t j = 1; j < w; ++j) {
    const int32_t dest = (r + j) % w;
    const int32_t src = (r - j + w) % w;
    ClearBlocks(ex);
    BlockRequests(ex, f, dest);
    int code = Execute(ex, f, ex->num_local, j == 1, stream);
    if (code == XSE_OK) code = SideAfter(ex, stream);
    if (code == XSE_OK) code = SendRecv(ex, dest, src, ex->side);
    if (code != XSE_OK) return code;
  }
  ClearBlocks(ex);
  BlockRequests(ex, f, r);
  int code = Execute(ex, f, ex->num_local, w == 1, stream);
  if (code != XSE_OK || w == 1) return code;
  code = StreamAfterSide(ex, stream);
  if (code != XSE_OK) return code;
  return Reorder(ex, stream);
}

int RunRow(xse_shard_exchange* ex, const xse_bag_request* f,
           cudaStream_t stream) {
  const int32_t w = ex->world, t = ex->plan.num_tables, d_ = ex->plan.dim;
  const int64_t row = static_cast<int64_t>(t) * d_;
  if (w == 1) {
    ClearBlocks(ex);
    for (int32_t k = 0; k < t; ++k) {
      AddBlock(ex, k, Slice(f[k], 0, ex->block, ex->out_local + k * d_, row));
    }
    return Execute(ex, f, t, true, stream);
  }
  const xse::NcclApi& n = xse::Nccl();
  for (int32_t c = 0; c < ex->chunks; ++c) {
    float* part = ex->partial + c * w * ex->piece * row;
    ClearBlocks(ex);
    for (int32_t s = 0; s < w; ++s) {
      const int64_t b0 = s * ex->block + c * ex->piece;
      for (int32_t k = 0; k < t; ++k) {
        AddBlock(ex, k, Slice(f[k], b0, ex->piece,
                              part + s * ex->piece * row + k * d_, row));
      }
    }
    int code = Execute(ex, f, t, c == 0, stream);
    if (code == XSE_OK) code = SideAfter(ex, stream);
    if (code != XSE_OK) return code;
    const ncclResult_t res = n.ReduceScatter(
        part, ex->out_local + c * ex->piece * row, ex->piece * row,
        ncclFloat32, ncclSum, ex->comm->comm, ex->side);
    if (res != ncclSuccess) return xse::NcclFail(res, "reduce-scatter");
  }
  return StreamAfterSide(ex, stream);
}

}  // namespace

extern "C" {

int xse_shard_unique_id(unsigned char id[XSE_SHARD_ID_BYTES]) {
  const xse::NcclApi& n = xse::Nccl();
  if (!n.loaded) return ShardFail(XSE_FAILED_PRECONDITION, "%s", n.error.c_str());
  if (id == nullptr) return ShardFail(XSE_INVALID_ARGUMENT, "null id buffer");
  static_assert(sizeof(ncclUniqueId) == XSE_SHARD_ID_BYTES, "NCCL id size");
  ncclUniqueId uid;
  const ncclResult_t r = n.GetUniqueId(&uid);
  if (r != ncclSuccess) return xse::NcclFail(r, "unique id");
  std::memcpy(id, &uid, sizeof(uid));
  return ShardOk();
}

int xse_shard_comm_create(int32_t device, int32_t world, int32_t rank,
                          const unsigned char id[XSE_SHARD_ID_BYTES],
                          xse_shard_comm** out) {
  const xse::NcclApi& n = xse::Nccl();
  if (!n.loaded) return ShardFail(XSE_FAILED_PRECONDITION, "%s", n.error.c_str());
  if (out == nullptr || id == nullptr) {
    return ShardFail(XSE_INVALID_ARGUMENT, "null argument");
  }
  *out = nullptr;
  if (world < 1 || world > XSE_SHARD_MAX_RANKS || rank < 0 || rank >= world) {
    return ShardFail(XSE_INVALID_ARGUMENT,
                     "communicator needs 1 <= world <= %d and 0 <= rank < "
                     "world (world %d, rank %d)",
                     XSE_SHARD_MAX_RANKS, world, rank);
  }
  xse::DeviceScope scope(device);
  ncclUniqueId uid;
  std::memcpy(&uid, id, sizeof(uid));
  ncclComm_t comm = nullptr;
  const ncclResult_t r = n.CommInitRank(&comm, world, uid, rank);
  if (r != ncclSuccess) return xse::NcclFail(r, "communicator init");
  auto* c = new xse_shard_comm();
  c->comm = comm;
  c->owned = true;
  c->device = device;
  c->world = world;
  c->rank = rank;
  *out = c;
  return ShardOk();
}

int xse_shard_comm_adopt(void* nccl_comm, int32_t device, int32_t world,
                         int32_t rank, xse_shard_comm** out) {
  if (out == nullptr || nccl_comm == nullptr) {
    return ShardFail(XSE_INVALID_ARGUMENT, "null argument");
  }
  if (world < 1 || world > XSE_SHARD_MAX_RANKS || rank < 0 || rank >= world) {
    return ShardFail(XSE_INVALID_ARGUMENT, "bad world %d / rank %d", world,
                     rank);
  }
  const xse::NcclApi& n = xse::Nccl();
  if (!n.loaded) return ShardFail(XSE_FAILED_PRECONDITION, "%s", n.error.c_str());
  auto* c = new xse_shard_comm();
  c->comm = static_cast<ncclComm_t>(nccl_comm);
  c->owned = false;
  c->device = device;
  c->world = world;
  c->rank = rank;
  *out = c;
  return ShardOk();
}

int xse_shard_comm_abort(xse_shard_comm* comm) {
  if (comm == nullptr || comm->comm == nullptr) {
    return ShardFail(XSE_INVALID_ARGUMENT, "null communicator");
  }
  const xse::NcclApi& n = xse::Nccl();
  const ncclResult_t r = n.CommAbort(comm->comm);
  comm->comm = nullptr;
  return r == ncclSuccess ? ShardOk() : xse::NcclFail(r, "abort");
}

void xse_shard_comm_destroy(xse_shard_comm* comm) {
  if (comm == nullptr) return;
  if (comm->owned && comm->comm != nullptr) {
    xse::DeviceScope scope(comm->device);
    xse::Nccl().CommDestroy(comm->comm);
  }
  delete comm;
}

void xse_shard_exchange_destroy(xse_shard_exchange* ex) {
  if (ex == nullptr) return;
  {
    xse::DeviceScope scope(ex->comm != nullptr ? ex->comm->device : 0);
    if (ex->side != nullptr) cudaStreamSynchronize(ex->side);
    cudaDeviceSynchronize();
    if (ex->peers != nullptr) xse_peer_group_destroy(ex->peers);
    cudaFree(ex->out_local);
    cudaFree(ex->send);
    cudaFree(ex->recv);
    cudaFree(ex->partial);
    if (ex->status != nullptr) xse_status_destroy(ex->status);
    if (ex->pooled != nullptr) cudaEventDestroy(ex->pooled);
    for (cudaEvent_t e : ex->done) cudaEventDestroy(e);
    if (ex->side != nullptr) cudaStreamDestroy(ex->side);
  }
  delete ex;
}

int xse_shard_exchange_create(xse_engine* engine, xse_shard_comm* comm,
                              const xse_shard_plan* plan,
                              xse_shard_exchange** out) {
  if (engine == nullptr || comm == nullptr || plan == nullptr ||
      out == nullptr) {
    return ShardFail(XSE_INVALID_ARGUMENT, "null argument");
  }
  *out = nullptr;
  if (comm->comm == nullptr) {
    return ShardFail(XSE_FAILED_PRECONDITION, "communicator was aborted");
  }
  const int32_t w = comm->world;
  const int32_t chunks = plan->chunks > 1 ? plan->chunks : 1;
  if (plan->mode < XSE_SHARD_TABLE_PEER || plan->mode > XSE_SHARD_ROW) {
    return ShardFail(XSE_INVALID_ARGUMENT, "unknown exchange mode %d",
                     plan->mode);
  }
  if (plan->num_tables < 1 || plan->dim < 1 || plan->dim % 4 != 0 ||
      plan->batch < 1 || plan->batch % w != 0 ||
      (plan->mode == XSE_SHARD_ROW && (plan->batch / w) % chunks != 0)) {
    return ShardFail(XSE_INVALID_ARGUMENT,
                     "shard plan needs tables >= 1, a dimension that is a "
                     "multiple of 4 and a batch divisible by the world size "
                     "%d (row-wise: by world * chunks) (tables %d, dim %d, "
                     "batch %lld, chunks %d)",
                     w, plan->num_tables, plan->dim,
                     static_cast<long long>(plan->batch), chunks);
  }
  if (plan->mode != XSE_SHARD_ROW && plan->num_tables < w) {
    return ShardFail(XSE_INVALID_ARGUMENT,
                     "table-wise sharding needs at least one table per rank "
                     "(%d tables, %d ranks)",
                     plan->num_tables, w);
  }
  xse::DeviceScope scope(comm->device);
  auto* ex = new xse_shard_exchange();
  ex->engine = engine;
  ex->comm = comm;
  ex->plan = *plan;
  ex->world = w;
  ex->rank = comm->rank;
  ex->chunks = chunks;
  ex->block = plan->batch / w;
  ex->piece = ex->block / chunks;
  const int64_t d = plan->dim, t = plan->num_tables;
  ex->out_floats = ex->block * t * d;
  int64_t at = 0;
  for (int32_t q = 0; q < w; ++q) {
    const int32_t tq = plan->mode == XSE_SHARD_ROW
                           ? plan->num_tables
                           : (plan->num_tables - q + w - 1) / w;
    ex->counts.push_back(tq);
    ex->recv_off.push_back(at);
    at += ex->block * tq * d;
  }
  ex->num_local = ex->counts[ex->rank];
  int capacity = ex->num_local;
  if (plan->mode == XSE_SHARD_TABLE_PEER || plan->mode == XSE_SHARD_TABLE_A2A) {
    capacity = ex->num_local * w;
  } else if (plan->mode == XSE_SHARD_ROW) {
    capacity = static_cast<int>(t) * w;
  }
  auto fail = [&](int code) {
    xse_shard_exchange_destroy(ex);
    return code;
  };
  int code = xse_status_create(capacity, &ex->status);
  if (code != XSE_OK) return fail(code);
  cudaError_t e = cudaStreamCreateWithFlags(&ex->side, cudaStreamNonBlocking);
  if (e == cudaSuccess) {
    e = cudaEventCreateWithFlags(&ex->pooled, cudaEventDisableTiming);
  }
  ex->slots = plan->mode == XSE_SHARD_TABLE_PEER ? 3 : 1;
  for (int32_t s = 0; s < ex->slots && e == cudaSuccess; ++s) {
    cudaEvent_t ev = nullptr;
    e = cudaEventCreateWithFlags(&ev, cudaEventDisableTiming);
    ex->done.push_back(ev);
    ex->done_valid.push_back(false);
  }
  if (e != cudaSuccess) return fail(xse::CudaFail(e, "exchange streams"));
  const size_t out_bytes = static_cast<size_t>(ex->out_floats) * 4;
  if (plan->mode == XSE_SHARD_TABLE_PEER) {
    xse_ipc_handle mine;
    code = xse_peer_group_create(comm->device, w, ex->rank,
                                 static_cast<int64_t>(out_bytes) * ex->slots,
                                 &ex->peers, &mine);
    if (code != XSE_OK) return fail(code);
    if (w > 1) {
      // Every rank's IPC handle through the communicator.
      unsigned char* dev = nullptr;
      std::vector<xse_ipc_handle> all(w);
      e = cudaMalloc(&dev, sizeof(xse_ipc_handle) * (w + 1));
      if (e == cudaSuccess) {
        e = cudaMemcpy(dev + sizeof(xse_ipc_handle) * w, &mine, sizeof(mine),
                       cudaMemcpyHostToDevice);
      }
      if (e != cudaSuccess) {
        cudaFree(dev);
        return fail(xse::CudaFail(e, "handle exchange buffer"));
      }
      const ncclResult_t r = xse::Nccl().AllGather(
          dev + sizeof(xse_ipc_handle) * w, dev, sizeof(xse_ipc_handle),
          ncclUint8, comm->comm, ex->side);
      if (r == ncclSuccess) {
        e = cudaMemcpyAsync(all.data(), dev, sizeof(xse_ipc_handle) * w,
                            cudaMemcpyDeviceToHost, ex->side);
        if (e == cudaSuccess) e = cudaStreamSynchronize(ex->side);
      }
      cudaFree(dev);
      if (r != ncclSuccess) return fail(xse::NcclFail(r, "handle exchange"));
      if (e != cudaSuccess) return fail(xse::CudaFail(e, "handle exchange"));
      code = xse_peer_group_connect(ex->peers, all.data(), w);
      if (code != XSE_OK) return fail(code);
    } else {
      code = xse_peer_group_connect(ex->peers, &mine, 1);
      if (code != XSE_OK) return fail(code);
    }
  } else {
    e = cudaMalloc(&ex->out_local, out_bytes);
    if (e == cudaSuccess && w > 1 && plan->mode != XSE_SHARD_ROW) {
      e = cudaMalloc(&ex->send, static_cast<size_t>(w) * ex->block *
                                    ex->num_local * d * 4);
      if (e == cudaSuccess) e = cudaMalloc(&ex->recv, out_bytes);
    }
    if (e == cudaSuccess && w > 1 && plan->mode == XSE_SHARD_ROW) {
      e = cudaMalloc(&ex->partial,
                     static_cast<size_t>(chunks) * w * ex->piece * t * d * 4);
    }
    if (e != cudaSuccess) return fail(xse::CudaFail(e, "exchange buffers"));
  }
  *out = ex;
  return ShardOk();
}

int xse_shard_exchange_run(xse_shard_exchange* ex,
                           const xse_bag_request* features, int32_t n,
                           int32_t flags, void* stream, float** out) {
  xse::TraceRange trace("xse.shard_exchange");
  if (ex == nullptr || features == nullptr) {
    return ShardFail(XSE_INVALID_ARGUMENT, "null argument");
  }
  if (ex->comm->comm == nullptr) {
    return ShardFail(XSE_FAILED_PRECONDITION, "communicator was aborted");
  }
  const int32_t want =
      ex->plan.mode == XSE_SHARD_ROW ? ex->plan.num_tables : ex->num_local;
  if (n != want) {
    return ShardFail(XSE_INVALID_ARGUMENT,
                     "rank %d pools %d tables; got %d feature requests",
                     ex->rank, want, n);
  }
  for (int32_t k = 0; k < n; ++k) {
    if (features[k].num_offsets != ex->plan.batch + 1 ||
        features[k].offsets == nullptr) {
      return ShardFail(XSE_INVALID_ARGUMENT,
                       "feature request %d has %lld row pointers; the batch "
                       "needs %lld",
                       k, static_cast<long long>(features[k].num_offsets),
                       static_cast<long long>(ex->plan.batch + 1));
    }
  }
  xse::DeviceScope scope(ex->comm->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int code = XSE_OK;
  switch (ex->plan.mode) {
    case XSE_SHARD_TABLE_PEER:
      return RunPeer(ex, features, flags, s, out);
    case XSE_SHARD_TABLE_A2A:
      code = RunA2A(ex, features, s);
      break;
    case XSE_SHARD_TABLE_PIPELINED:
      code = RunPipelined(ex, features, s);
      break;
    default:
      code = RunRow(ex, features, s);
      break;
  }
  if (code != XSE_OK) return code;
  ++ex->step;
  if (out != nullptr) *out = ex->out_local;
  return ShardOk();
}

int xse_shard_exchange_ready(xse_shard_exchange* ex, void* stream) {
  if (ex == nullptr) return ShardFail(XSE_INVALID_ARGUMENT, "null exchange");
  if (ex->pending_ready && ex->done_valid[ex->slot]) {
    xse::DeviceScope scope(ex->comm->device);
    const cudaError_t e = cudaStreamWaitEvent(
        static_cast<cudaStream_t>(stream), ex->done[ex->slot], 0);
    if (e != cudaSuccess) return xse::CudaFail(e, "barrier wait");
    ex->pending_ready = false;
  }
  return ShardOk();
}

int xse_shard_exchange_check(xse_shard_exchange* ex, void* stream) {
  if (ex == nullptr) return ShardFail(XSE_INVALID_ARGUMENT, "null exchange");
  xse::DeviceScope scope(ex->comm->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaStreamSynchronize(s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(ex->side);
  if (e != cudaSuccess) return xse::CudaFail(e, "exchange synchronize");
  int code = xse_status_wait(ex->status, stream);
  if (code != XSE_OK) return code;
  if (ex->peers != nullptr) {
    code = xse_peer_group_check(ex->peers, stream);
    if (code != XSE_OK) return code;
  }
  if (ex->comm->comm != nullptr && ex->world > 1) {
    ncclResult_t async = ncclSuccess;
    const ncclResult_t r = xse::Nccl().CommGetAsyncError(ex->comm->comm,
                                                         &async);
    if (r != ncclSuccess) return xse::NcclFail(r, "async error query");
    if (async != ncclSuccess && async != ncclInProgress) {
      return xse::NcclFail(async, "asynchronous error");
    }
  }
  return ShardOk();
}

}  // extern "C"
