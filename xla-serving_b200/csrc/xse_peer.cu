// Peer-memory exchange group and its flag barrier (include/xse_peer.h).
//
// Each rank's buffer starts with a 256-byte header: flags[q] (uint32) at
// 4q is written by rank q when it reaches a barrier, and the error word at
// byte 128 is set by this rank's barrier when a wait gives up. Data starts at
// byte 256, so it keeps the allocation's 256-byte alignment.
//
// The barrier is one kernel of `world` threads per rank. Thread q first makes
// this rank's earlier work visible system-wide (the stream order already
// finished it; the fence orders it before the signal), then stores the new
// epoch into rank q's flags[rank] with release semantics at system scope, and
// then polls flags[q] of its own header with acquire loads until rank q's
// epoch arrives or the spin limit runs out (the first polls run back to
// back, later ones 1 us apart). Epochs only grow, by one per barrier, so a
// flag at or past the epoch means that rank got here. A group whose barrier
// gave up is out of step and must be destroyed.

#include <cuda_runtime.h>
#include <stdint.h>

#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <mutex>

#include "../../include/xse_emb.h"
#include "../../include/xse_peer.h"
#include "xse_internal.h"

namespace xse {
namespace {

constexpr int64_t kHeaderBytes = 256;
constexpr int64_t kErrorOffset = 128;
constexpr int64_t kDefaultSpinLimit = 2000000;  // ~1 us per poll

int Fail(int code, const char* fmt, ...)
    __attribute__((format(printf, 2, 3)));
int Fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list args;
  va_start(args, fmt);
  vsnprintf(buf, sizeof(buf), fmt, args);
  va_end(args);
  SetLastErrorMessage(buf);
  return code;
}

struct BarrierParams {
  uint32_t* flags[XSE_PEER_MAX_RANKS];  // every rank's header, mapped here
  int32_t* error;                       // this rank's error word
  int64_t spin_limit;
  uint32_t epoch;
  int32_t world;
  int32_t rank;
};

__device__ __forceinline__ void StoreRelease(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v)
               : "memory");
}

__device__ __forceinline__ uint32_t LoadAcquire(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];"
               : "=r"(v)
               : "l"(p)
               : "memory");
  return v;
}

__global__ void PeerBarrierKernel(BarrierParams p) {
  const int q = threadIdx.x;
  if (q >= p.world) return;
  __threadfence_system();
  StoreRelease(p.flags[q] + p.rank, p.epoch);
  const uint32_t* mine = p.flags[p.rank] + q;
  for (int64_t spins = 0;; ++spins) {
    if (static_cast<int32_t>(LoadAcquire(mine) - p.epoch) >= 0) break;
    if (spins >= p.spin_limit) {
      atomicExch(p.error, 1);  // gave up: rank q never arrived
      break;
    }
    if (spins >= 256) __nanosleep(1000);
  }
}

}  // namespace
}  // namespace xse

struct xse_peer_group {
  int32_t device = 0, world = 0, rank = 0;
  int64_t buffer_bytes = 0;
  char* own = nullptr;  // this rank's allocation (header + data)
  char* mapped[XSE_PEER_MAX_RANKS] = {};
  bool connected = false;
  uint32_t epoch = 0;
  std::mutex mu;
};

namespace {

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

}  // namespace

extern "C" int xse_peer_group_create(int32_t device, int32_t world,
                                     int32_t rank, int64_t buffer_bytes,
                                     xse_peer_group** out,
                                     xse_ipc_handle* handle) {
  using xse::Fail;
  if (out == nullptr || handle == nullptr) {
    return Fail(XSE_INVALID_ARGUMENT, "null output argument");
  }
  *out = nullptr;
  if (world < 1 || world > XSE_PEER_MAX_RANKS || rank < 0 || rank >= world ||
      buffer_bytes < 0) {
    return Fail(XSE_INVALID_ARGUMENT,
                "peer group needs 1 <= world <= %d, 0 <= rank < world and a "
                "non-negative size (world %d, rank %d)",
                XSE_PEER_MAX_RANKS, world, rank);
  }
  DeviceScope scope(device);
  auto* g = new xse_peer_group();
  g->device = device;
  g->world = world;
  g->rank = rank;
  g->buffer_bytes = buffer_bytes;
  void* ptr = nullptr;
  cudaError_t e = cudaMalloc(&ptr, xse::kHeaderBytes + buffer_bytes);
  if (e == cudaSuccess) e = cudaMemset(ptr, 0, xse::kHeaderBytes);
  cudaIpcMemHandle_t h;
  if (e == cudaSuccess) e = cudaIpcGetMemHandle(&h, ptr);
  if (e == cudaSuccess) e = cudaDeviceSynchronize();
  if (e != cudaSuccess) {
    if (ptr != nullptr) cudaFree(ptr);
    delete g;
    return Fail(XSE_RESOURCE_EXHAUSTED, "peer buffer of %lld bytes: %s",
                static_cast<long long>(buffer_bytes), cudaGetErrorString(e));
  }
  static_assert(sizeof(h) <= sizeof(handle->bytes), "IPC handle size");
  std::memset(handle->bytes, 0, sizeof(handle->bytes));
  std::memcpy(handle->bytes, &h, sizeof(h));
  g->own = static_cast<char*>(ptr);
  g->mapped[rank] = g->own;
  *out = g;
  xse::SetLastErrorMessage("");
  return XSE_OK;
}

extern "C" int xse_peer_group_connect(xse_peer_group* g,
                                      const xse_ipc_handle* handles,
                                      int32_t world) {
  using xse::Fail;
  if (g == nullptr || handles == nullptr || world != g->world) {
    return Fail(XSE_INVALID_ARGUMENT,
                "connect needs the group and one handle per rank");
  }
  std::lock_guard<std::mutex> lock(g->mu);
  if (g->connected) return Fail(XSE_FAILED_PRECONDITION, "already connected");
  DeviceScope scope(g->device);
  for (int32_t q = 0; q < world; ++q) {
    if (q == g->rank) continue;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handles[q].bytes, sizeof(h));
    void* ptr = nullptr;
    const cudaError_t e =
        cudaIpcOpenMemHandle(&ptr, h, cudaIpcMemLazyEnablePeerAccess);
    if (e != cudaSuccess) {
      for (int32_t k = 0; k < q; ++k) {
        if (k != g->rank && g->mapped[k] != nullptr) {
          cudaIpcCloseMemHandle(g->mapped[k]);
          g->mapped[k] = nullptr;
        }
      }
      return Fail(XSE_INTERNAL, "mapping rank %d's buffer: %s", q,
                  cudaGetErrorString(e));
    }
    g->mapped[q] = static_cast<char*>(ptr);
  }
  g->connected = true;
  xse::SetLastErrorMessage("");
  return XSE_OK;
}

extern "C" void* xse_peer_group_buffer(xse_peer_group* g, int32_t peer) {
  if (g == nullptr || peer < 0 || peer >= g->world) return nullptr;
  if (!g->connected && peer != g->rank) return nullptr;
  return g->mapped[peer] + xse::kHeaderBytes;
}

extern "C" int xse_peer_group_barrier(xse_peer_group* g, int64_t spin_limit,
                                      void* stream) {
  using xse::Fail;
  if (g == nullptr) return Fail(XSE_INVALID_ARGUMENT, "null group");
  std::lock_guard<std::mutex> lock(g->mu);
  if (!g->connected) {
    return Fail(XSE_FAILED_PRECONDITION, "barrier before connect");
  }
  DeviceScope scope(g->device);
  xse::BarrierParams p = {};
  for (int32_t q = 0; q < g->world; ++q) {
    p.flags[q] = reinterpret_cast<uint32_t*>(g->mapped[q]);
  }
  p.error = reinterpret_cast<int32_t*>(g->own + xse::kErrorOffset);
  p.spin_limit = spin_limit > 0 ? spin_limit : xse::kDefaultSpinLimit;
  p.epoch = ++g->epoch;
  p.world = g->world;
  p.rank = g->rank;
  xse::PeerBarrierKernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(p);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    return Fail(XSE_INTERNAL, "barrier launch: %s", cudaGetErrorString(e));
  }
  xse::SetLastLaunchCount(1);
  xse::SetLastErrorMessage("");
  return XSE_OK;
}

extern "C" int xse_peer_group_check(xse_peer_group* g, void* stream) {
  using xse::Fail;
  if (g == nullptr) return Fail(XSE_INVALID_ARGUMENT, "null group");
  DeviceScope scope(g->device);
  int32_t error = 0;
  cudaError_t e = cudaMemcpyAsync(&error, g->own + xse::kErrorOffset,
                                  sizeof(error), cudaMemcpyDeviceToHost,
                                  static_cast<cudaStream_t>(stream));
  if (e == cudaSuccess) e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    return Fail(XSE_INTERNAL, "reading the barrier status: %s",
                cudaGetErrorString(e));
  }
  if (error != 0) {
    return Fail(XSE_DEADLINE_EXCEEDED,
                "a peer barrier gave up waiting for another rank");
  }
  xse::SetLastErrorMessage("");
  return XSE_OK;
}

extern "C" void xse_peer_group_destroy(xse_peer_group* g) {
  if (g == nullptr) return;
  {
    DeviceScope scope(g->device);
    for (int32_t q = 0; q < g->world; ++q) {
      if (q != g->rank && g->mapped[q] != nullptr) {
        cudaIpcCloseMemHandle(g->mapped[q]);
      }
    }
    if (g->own != nullptr) cudaFree(g->own);
  }
  delete g;
}
