// C ABI of the engine (declared in include/xse_emb.h).
//
// The engine mirrors CpuEmbeddingEngine (data/cpu_embedding/cc/
// cpu_embedding_engine.{h,cc}): a registry of tables and feature specs under
// two mutexes taken in the order specs -> tables. Tables live in HBM. A group
// execution follows internal::ExecuteEmbeddingBagBatch (embedding_bag.cc:
// 477-535): validate the whole group, check output isolation, then pool; the
// validation of offsets and ids runs on the device and its result gates the
// pooling kernel, so a failing group writes nothing.

#include <cuda_runtime.h>
#include <stdint.h>

#include <unistd.h>

#include <algorithm>
#include <atomic>
#include <cerrno>
#include <cinttypes>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <tuple>
#include <unordered_map>
#include <vector>

#include "../../include/xse_dlrm.h"
#include "../../include/xse_emb.h"
#include "xse_internal.h"

extern "C" int xse_synth_table_impl(void*, float*, float*, int32_t, uint64_t,
                                    uint64_t, int64_t, int64_t, int32_t,
                                    cudaStream_t);
extern "C" int xse_synth_lengths_impl(int64_t*, int64_t, int32_t, int32_t,
                                      uint64_t, uint64_t, cudaStream_t);
extern "C" int xse_synth_ids_impl(int64_t*, int64_t, int64_t, double,
                                  uint64_t, uint64_t, uint64_t, uint64_t,
                                  int64_t, cudaStream_t);
extern "C" int xse_synth_weights_impl(float*, int64_t, uint64_t, uint64_t,
                                      int64_t, cudaStream_t);

namespace {

thread_local std::string g_last_error;
thread_local int32_t g_last_launches = 0;

int SetError(int code, const char* fmt, ...) {
  char buf[1024];
  va_list args;
  va_start(args, fmt);
  vsnprintf(buf, sizeof(buf), fmt, args);
  va_end(args);
  g_last_error = buf;
  return code;
}

int Ok() {
  g_last_error.clear();
  return XSE_OK;
}

int CudaError(cudaError_t e, const char* what) {
  return SetError(XSE_INTERNAL, "%s: %s", what, cudaGetErrorString(e));
}

}  // namespace

namespace xse {
void SetLastErrorMessage(const char* message) {
  g_last_error = message != nullptr ? message : "";
}
void SetLastLaunchCount(int32_t launches) { g_last_launches = launches; }
}  // namespace xse

namespace {

struct Table {
  std::string name;
  int32_t dtype = 0, combine = 1, dim = 0;
  int64_t vocab = 0, row_begin = 0, row_end = 0;
  void* rows = nullptr;          // device
  float2* scale_bias = nullptr;  // device, int8 rows
  bool owns_rows = false;
  int device = 0;
  ~Table() {
    if (rows == nullptr && scale_bias == nullptr) return;
    int prev = 0;
    cudaGetDevice(&prev);
    cudaSetDevice(device);
    if (owns_rows && rows != nullptr) cudaFree(rows);
    if (scale_bias != nullptr) cudaFree(scale_bias);
    cudaSetDevice(prev);
  }
};

struct Feature {
  std::string table;
  int32_t max_sequence_length = 0;
};

size_t ElemBytes(int32_t dtype) {
  return dtype == XSE_DT_F32 ? 4 : dtype == XSE_DT_BF16 ? 2 : 1;
}

// Host-detectable error of one request, ordered as the checks of
// ValidateEmbeddingBagInput (embedding_bag.cc:89-144).
enum HostStage {
  kStageNone = 0,
  kStageEarly = 1,      // before the offset checks
  kStageIdsNull = 2,    // after the offset/size checks, before id bounds
  kStageWeightsNull = 3,
};

struct RequestMeta {
  int stage = kStageNone;
  int code = XSE_OK;
  std::string message;
  const void* ids = nullptr;
  int32_t ids64 = 1;
  int64_t vocab = 0;
};

}  // namespace

namespace {

// What the host knows about one execution recorded in a status slot.
struct StatusSlot {
  std::vector<RequestMeta> meta;
  int32_t n = 0;
  int early_code = XSE_OK;  // host-side failure decided at launch time
  std::string early_message;
};

}  // namespace

// A ring of device status slots, one per execution. Synchronous executions
// use slot 0 and read it back at once. Asynchronous executions fill slots in
// turn with no per-execution memset or read-back: the ring is cleared with
// one memset when it starts over and read back in one copy at
// xse_status_wait, which reports the first failing execution.
struct xse_status {
  int device = 0;
  int32_t capacity = 0;  // requests per execution
  int32_t ring = 1;      // slots
  size_t slot_bytes = 0;
  char* dev = nullptr;
  char* host = nullptr;  // pinned mirror
  std::vector<StatusSlot> slots;
  int32_t used = 0;        // slots filled since the last read-back
  bool need_reset = true;  // slots 1.. may hold old results
  int deferred_code = XSE_OK;  // first error of a read-back forced by a full ring
  std::string deferred_message;

  xse::DevStatus* dev_slot(int k) {
    return reinterpret_cast<xse::DevStatus*>(dev + slot_bytes * k);
  }
  xse::DevStatus* host_slot(int k) {
    return reinterpret_cast<xse::DevStatus*>(host + slot_bytes * k);
  }
};

// One timed trial launch of the pooling-kernel tuner.
struct PoolTrial {
  int32_t choice;  // xse::kPoolStreaming or xse::kPoolStaged
  cudaEvent_t start, end;
};

// Pooling-kernel choice for one launch signature (see ChoosePoolKernel).
struct PoolTuner {
  int32_t decided = xse::kPoolAuto;
  int64_t launched = 0;       // trial launches issued
  int32_t done[2] = {0, 0};   // completed timings: streaming, staged
  float ms[2] = {0.0f, 0.0f};  // fastest of each kernel's timings
  std::vector<PoolTrial> pending;
};

struct xse_engine {
  int device = 0;
  std::mutex specs_mu;
  std::mutex tables_mu;
  std::unordered_map<std::string, Feature> features;
  std::unordered_map<std::string, std::shared_ptr<Table>> tables;
  std::mutex default_status_mu;
  xse_status* default_status = nullptr;
  // Kernel timing of every profile_period-th execution (0: off): events
  // before the validation kernels (when they run), before the pooling
  // kernels and after them.
  struct ProfileEvents {
    cudaEvent_t validate = nullptr, pool = nullptr, end = nullptr;
    bool validated = false;
  };
  std::mutex profile_mu;
  int32_t profile_period = 0;
  int64_t profile_calls = 0;
  std::vector<ProfileEvents> profile_events;
  size_t profile_used = 0;
  // Pooling-kernel tuner, keyed by launch signature.
  std::mutex tune_mu;
  std::unordered_map<uint64_t, PoolTuner> tuners;
};

namespace {

// Resolves the errors of the execution in slot k in request order, mirroring
// the order of the reference's per-request checks. Returns the status code.
int ResolveSlot(xse_status* st, int k) {
  const StatusSlot& slot = st->slots[k];
  const xse::DevStatus* host = st->host_slot(k);
  for (int32_t i = 0; i < slot.n; ++i) {
    if (host->req[i].flags & xse::kErrDeviceWait) {
      return SetError(XSE_INTERNAL,
                      "A device-side wait of the fused interaction ran out.");
    }
  }
  for (int32_t i = 0; i < slot.n; ++i) {
    const RequestMeta& m = slot.meta[i];
    if (m.stage == kStageEarly) return SetError(m.code, "%s", m.message.c_str());
    const unsigned int flags = host->req[i].flags;
    const char* msg = nullptr;
    if (flags & xse::kErrBadOffsets) {
      msg = "Row pointers must be non-negative and monotonic.";
    } else if (flags & xse::kErrLastExceedsIds) {
      msg = "Final row pointer exceeds embedding IDs size.";
    } else if (flags & xse::kErrLastExceedsWeights) {
      msg = "Final row pointer exceeds weights size.";
    }
    if (msg != nullptr) {
      return SetError(XSE_INVALID_ARGUMENT,
                      "FP32 embedding-bag request %d: %s", i, msg);
    }
    if (m.stage == kStageIdsNull || m.stage == kStageWeightsNull) {
      return SetError(m.code, "%s", m.message.c_str());
    }
    if (flags & xse::kErrBadId) {
      const int64_t index =
          static_cast<int64_t>(~host->req[i].inv_min_bad_index);
      int64_t id = 0;
      if (m.ids64) {
        cudaMemcpy(&id, static_cast<const int64_t*>(m.ids) + index,
                   sizeof(id), cudaMemcpyDeviceToHost);
      } else {
        int32_t id32 = 0;
        cudaMemcpy(&id32, static_cast<const int32_t*>(m.ids) + index,
                   sizeof(id32), cudaMemcpyDeviceToHost);
        id = id32;
      }
      return SetError(XSE_INVALID_ARGUMENT,
                      "FP32 embedding-bag request %d: Embedding ID (%" PRId64
                      ") at index %" PRId64 " is out of bounds [0, %" PRId64
                      ").",
                      i, id, index, m.vocab);
    }
  }
  if (slot.early_code != XSE_OK) {
    return SetError(slot.early_code, "%s", slot.early_message.c_str());
  }
  return Ok();
}

// Waits for the stream, reads back every filled slot and returns the first
// error among them (or one deferred by an earlier forced read-back).
int SettleStatus(xse_status* st, cudaStream_t stream) {
  cudaError_t e = cudaStreamSynchronize(stream);
  if (e != cudaSuccess) return SetError(XSE_INTERNAL, "stream synchronize: %s",
                                        cudaGetErrorString(e));
  int code = XSE_OK;
  std::string message;
  if (st->used > 0) {
    e = cudaMemcpy(st->host, st->dev, st->slot_bytes * st->used,
                   cudaMemcpyDeviceToHost);
    if (e != cudaSuccess) {
      return SetError(XSE_INTERNAL, "status read-back: %s",
                      cudaGetErrorString(e));
    }
    for (int32_t k = 0; k < st->used && code == XSE_OK; ++k) {
      code = ResolveSlot(st, k);
      if (code != XSE_OK) message = g_last_error;
    }
  }
  st->used = 0;
  st->need_reset = true;
  if (st->deferred_code != XSE_OK) {
    code = st->deferred_code;
    message = st->deferred_message;
    st->deferred_code = XSE_OK;
    st->deferred_message.clear();
  }
  return code == XSE_OK ? Ok() : SetError(code, "%s", message.c_str());
}

// A set of `count` byte intervals [base + k*stride, base + k*stride + width).
// Contiguous buffers have count 1. Outputs may be strided (one table's
// column block of an interleaved [batch, tables, dim] buffer), which the
// reference's contiguous outputs never are.
struct Range {
  int64_t base, stride, width, count;
  int32_t request;
  const char* kind;
  int64_t end() const { return base + (count - 1) * stride + width; }
};

int64_t FloorDiv(int64_t a, int64_t b) {
  const int64_t q = a / b;
  return (a % b != 0 && ((a < 0) != (b < 0))) ? q - 1 : q;
}

// Exact overlap test when both ranges share one stride (or either is a
// single interval); a conservative hull test otherwise.
bool Overlaps(const Range& a, const Range& b) {
  if (a.count == 1 && b.count == 1) {
    return a.base < b.base + b.width && b.base < a.base + a.width;
  }
  if (a.end() <= b.base || b.end() <= a.base) return false;
  const Range& s = a.count >= b.count ? a : b;  // strided
  const Range& o = a.count >= b.count ? b : a;
  if (o.count == 1) {
    // Rows k of s meet [o.base, o.base + o.width) iff
    // o.base - width < s.base + k*stride < o.base + o.width.
    const int64_t k_lo = FloorDiv(o.base - s.width - s.base, s.stride) + 1;
    const int64_t k_hi =
        -FloorDiv(-(o.base + o.width - s.base), s.stride) - 1;
    return std::max<int64_t>(k_lo, 0) <= std::min<int64_t>(k_hi, s.count - 1);
  }
  if (a.stride != b.stride) return true;
  // Rows k of a and j of b meet iff m = k - j satisfies
  // d - a.width < m*stride < d + b.width with d = b.base - a.base.
  const int64_t d = b.base - a.base;
  const int64_t m_lo = FloorDiv(d - a.width, a.stride) + 1;
  const int64_t m_hi = -FloorDiv(-(d + b.width), a.stride) - 1;
  return std::max<int64_t>(m_lo, -(b.count - 1)) <=
         std::min<int64_t>(m_hi, a.count - 1);
}

void AddRange(const void* p, int64_t bytes, int32_t request, const char* kind,
              std::vector<Range>* out) {
  if (p == nullptr || bytes <= 0) return;
  out->push_back({static_cast<int64_t>(reinterpret_cast<uintptr_t>(p)), bytes,
                  bytes, 1, request, kind});
}

// ValidateOutputIsolation (embedding_bag.cc:304-351) over device ranges.
int CheckIsolation(const xse_bag_request* reqs,
                   const std::vector<std::shared_ptr<Table>>& tables,
                   int32_t n, std::string* message) {
  std::vector<Range> outputs, inputs;
  for (int32_t i = 0; i < n; ++i) {
    const xse_bag_request& r = reqs[i];
    const Table& t = *tables[i];
    const int64_t bags = r.num_offsets - 1;
    const int64_t stride = r.output_stride > 0 ? r.output_stride : t.dim;
    if (bags > 0 && r.output != nullptr) {
      outputs.push_back(
          {static_cast<int64_t>(reinterpret_cast<uintptr_t>(r.output)),
           stride * 4, static_cast<int64_t>(t.dim) * 4, bags, i, "output"});
    }
    AddRange(r.ids, r.num_ids * (r.ids_type == XSE_INDEX_I64 ? 8 : 4), i,
             "embedding-ID", &inputs);
    AddRange(r.offsets,
             r.num_offsets * (r.offsets_type == XSE_INDEX_I64 ? 8 : 4), i,
             "row-pointer", &inputs);
    AddRange(r.weights, r.num_weights * 4, i, "weight", &inputs);
    AddRange(t.rows,
             (t.row_end - t.row_begin) * t.dim *
                 static_cast<int64_t>(ElemBytes(t.dtype)),
             i, "embedding-table", &inputs);
  }
  // Sorted by start, outputs are compared pairwise while their hulls can
  // still meet (strided outputs interleave, so neighbours are not enough).
  std::sort(outputs.begin(), outputs.end(),
            [](const Range& a, const Range& b) { return a.base < b.base; });
  char buf[256];
  for (size_t k = 0; k < outputs.size(); ++k) {
    for (size_t j = k + 1;
         j < outputs.size() && outputs[j].base < outputs[k].end(); ++j) {
      if (Overlaps(outputs[k], outputs[j])) {
        const int32_t lo = std::min(outputs[k].request, outputs[j].request);
        const int32_t hi = std::max(outputs[k].request, outputs[j].request);
        snprintf(buf, sizeof(buf),
                 "FP32 embedding-bag request outputs %d and %d overlap.", lo,
                 hi);
        *message = buf;
        return XSE_INVALID_ARGUMENT;
      }
    }
  }
  // Inputs sorted by start, with the running maximum of their ends: an
  // output is tested only against inputs that start before its end, walking
  // down while some input at or below the position still reaches past the
  // output's start. Of the inputs an output meets, the first in request
  // order is reported, as a scan of the inputs in request order would.
  // (A sharded step holds 8 tables x W destinations of requests; the plain
  // outputs x inputs scan took about 50 us at W = 8.)
  std::vector<int32_t> order(inputs.size());
  for (size_t i = 0; i < order.size(); ++i) order[i] = static_cast<int32_t>(i);
  std::sort(order.begin(), order.end(), [&](int32_t a, int32_t b) {
    return inputs[a].base < inputs[b].base;
  });
  std::vector<int64_t> reach(order.size());
  int64_t far = INT64_MIN;
  for (size_t k = 0; k < order.size(); ++k) {
    far = std::max(far, inputs[order[k]].end());
    reach[k] = far;
  }
  for (const Range& o : outputs) {
    const int64_t o_end = o.end();
    const size_t hi =
        std::lower_bound(order.begin(), order.end(), o_end,
                         [&](int32_t idx, int64_t v) {
                           return inputs[idx].base < v;
                         }) -
        order.begin();
    int32_t hit = -1;
    for (size_t k = hi; k-- > 0 && reach[k] > o.base;) {
      const int32_t idx = order[k];
      if ((hit < 0 || idx < hit) && Overlaps(o, inputs[idx])) hit = idx;
    }
    if (hit >= 0) {
      const Range& in = inputs[hit];
      snprintf(buf, sizeof(buf),
               "FP32 embedding-bag request %d output overlaps request %d %s "
               "storage.",
               o.request, in.request, in.kind);
      *message = buf;
      return XSE_INVALID_ARGUMENT;
    }
  }
  return XSE_OK;
}

// ---------------------------------------------------------------------------
// Pooling-kernel tuner. Launches of 16-byte-vector rows larger than one wave
// of PoolStagedKernel can run either it or PoolVecKernel, with bit-identical
// results; which is faster depends on the id stream (the staged kernel wins
// when skewed ids make most rows cache hits -- the Zipf(1.1) table-wise
// slice 1.08 -> 0.90 ms -- and loses badly on uniform ids over tables
// larger than L2: 70 -> 123 us on the multi-table workload), which the
// engine cannot see. So per launch signature (layout, tables and their
// weighting modes, request count, log2 of the bag count) the first
// executions alternate the two kernels with CUDA events around each launch,
// and once each kernel has kTuneTrials completed timings the one with the
// faster best time is used from then on. Events are read without waiting
// (cudaEventQuery) on later executions of the same signature.
constexpr int kTuneTrials = 2;
constexpr size_t kTuneMaxPending = 4 * kTuneTrials;
// Signatures beyond this many take the fixed rule (bounds the map when
// batch shapes or table sets keep changing).
constexpr size_t kTuneMaxSignatures = 4096;

uint64_t TuneKey(const xse::Layout& l, const xse::PoolParams& p) {
  uint64_t h = 1469598103934665603ull;  // FNV-1a
  auto mix = [&h](uint64_t v) {
    h ^= v;
    h *= 1099511628211ull;
  };
  mix(static_cast<uint64_t>(l.dtype));
  mix(static_cast<uint64_t>(l.g));
  mix(static_cast<uint64_t>(l.v));
  mix(static_cast<uint64_t>(l.exact));
  mix(static_cast<uint64_t>(p.n));
  for (int32_t k = 0; k < p.n; ++k) {
    mix(static_cast<uint64_t>(reinterpret_cast<uintptr_t>(p.d[k].rows)));
    mix(static_cast<uint64_t>(xse::WeightModeOf(p.d[k])));
  }
  int bucket = 0;
  for (int64_t t = p.total_tasks; t > 1; t >>= 1) ++bucket;
  mix(static_cast<uint64_t>(bucket));
  return h;
}

// Folds the trial timings that have completed into `t` (tune_mu held).
void PollTrials(PoolTuner* t) {
  size_t keep = 0;
  for (size_t i = 0; i < t->pending.size(); ++i) {
    PoolTrial& trial = t->pending[i];
    const cudaError_t q = cudaEventQuery(trial.end);
    if (q == cudaErrorNotReady) {
      // Not an error: clear it from the runtime's last-error slot.
      if (cudaPeekAtLastError() == cudaErrorNotReady) (void)cudaGetLastError();
      t->pending[keep++] = trial;
      continue;
    }
    float ms = 0.0f;
    const cudaError_t te =
        q == cudaSuccess ? cudaEventElapsedTime(&ms, trial.start, trial.end)
                         : q;
    // A trial whose events failed is dropped; its error must not surface as
    // the last error of an unrelated later call.
    if (te != cudaSuccess) (void)cudaGetLastError();
    if (te == cudaSuccess) {
      // The fastest timing of each kernel: a first launch can carry one-off
      // costs (module loading, cold caches) that later ones do not.
      const int k = trial.choice == xse::kPoolStaged ? 1 : 0;
      t->ms[k] = t->done[k] == 0 ? ms : std::min(t->ms[k], ms);
      ++t->done[k];
    }
    cudaEventDestroy(trial.start);
    cudaEventDestroy(trial.end);
  }
  t->pending.resize(keep);
  if (t->decided == xse::kPoolAuto && t->done[0] >= kTuneTrials &&
      t->done[1] >= kTuneTrials) {
    t->decided =
        t->ms[1] < t->ms[0] ? xse::kPoolStaged : xse::kPoolStreaming;
  }
}

// Sets p->kernel_choice for a launch of `engine`; returns the trial to time
// (events created, choice set) or a trial with null events.
// XSE_POOL_KERNEL=streaming or =staged in the environment fixes the choice
// for every tunable launch (profiling one kernel on purpose: under a
// profiler that serialises kernels the tuner's timings mean nothing).
int32_t ForcedPoolKernel() {
  static const int32_t forced = [] {
    const char* v = std::getenv("XSE_POOL_KERNEL");
    if (v == nullptr) return static_cast<int32_t>(xse::kPoolAuto);
    if (std::strcmp(v, "streaming") == 0) return static_cast<int32_t>(xse::kPoolStreaming);
    if (std::strcmp(v, "staged") == 0) return static_cast<int32_t>(xse::kPoolStaged);
    return static_cast<int32_t>(xse::kPoolAuto);
  }();
  return forced;
}

PoolTrial ChoosePoolKernel(xse_engine* engine, const xse::Layout& l,
                           xse::PoolParams* p, uint64_t* key) {
  PoolTrial trial{xse::kPoolAuto, nullptr, nullptr};
  if (!xse::PoolKernelTunable(l, p->total_tasks)) return trial;
  if (ForcedPoolKernel() != xse::kPoolAuto) {
    p->kernel_choice = ForcedPoolKernel();
    return trial;
  }
  *key = TuneKey(l, *p);
  std::lock_guard<std::mutex> lock(engine->tune_mu);
  if (engine->tuners.size() >= kTuneMaxSignatures &&
      engine->tuners.find(*key) == engine->tuners.end()) {
    return trial;
  }
  PoolTuner& t = engine->tuners[*key];
  if (!t.pending.empty()) PollTrials(&t);
  if (t.decided != xse::kPoolAuto) {
    p->kernel_choice = t.decided;
    return trial;
  }
  if (t.pending.size() >= kTuneMaxPending) return trial;  // static rule
  const int32_t choice =
      t.launched % 2 == 0 ? xse::kPoolStaged : xse::kPoolStreaming;
  if (cudaEventCreate(&trial.start) != cudaSuccess) {
    (void)cudaGetLastError();
    return PoolTrial{xse::kPoolAuto, nullptr, nullptr};
  }
  if (cudaEventCreate(&trial.end) != cudaSuccess) {
    (void)cudaGetLastError();
    cudaEventDestroy(trial.start);
    return PoolTrial{xse::kPoolAuto, nullptr, nullptr};
  }
  ++t.launched;
  trial.choice = choice;
  p->kernel_choice = choice;
  return trial;
}

void AddTrial(xse_engine* engine, uint64_t key, const PoolTrial& trial) {
  std::lock_guard<std::mutex> lock(engine->tune_mu);
  engine->tuners[key].pending.push_back(trial);
}

class DeviceGuard {
 public:
  explicit DeviceGuard(int device) {
    cudaGetDevice(&prev_);
    if (prev_ != device) cudaSetDevice(device);
    device_ = device;
  }
  ~DeviceGuard() {
    if (prev_ != device_) cudaSetDevice(prev_);
  }

 private:
  int prev_ = 0, device_ = 0;
};

// `inter` non-null: the pooled rows feed the dot interaction (the requests'
// outputs are not used) -- the fused kernel where one serves the layout,
// else pooling into scratch and the interaction kernel. `parts` non-null:
// the parts are pooled instead of `reqs` (whose outputs are not used), and
// `reqs` are validated only when parts->validate asks for it.
int ExecuteBatch(xse_engine* engine, const xse_bag_request* reqs, int32_t n,
                 cudaStream_t stream, int32_t flags, xse_status* st,
                 const xse::InteractArgs* inter = nullptr,
                 const xse::PartSet* parts = nullptr) {
  g_last_launches = 0;
  if (n <= 0 || reqs == nullptr) {
    return SetError(XSE_INVALID_ARGUMENT,
                    "Embedding batch requires at least one request.");
  }
  if (n > st->capacity) {
    return SetError(XSE_INVALID_ARGUMENT,
                    "Embedding batch has %d requests; the status block holds "
                    "%d.",
                    n, st->capacity);
  }
  // Resolve specs and tables under the same lock order as Clear
  // (cpu_embedding_engine.cc:174-200).
  std::vector<std::shared_ptr<Table>> tables(static_cast<size_t>(n));
  {
    std::lock_guard<std::mutex> spec_lock(engine->specs_mu);
    std::lock_guard<std::mutex> table_lock(engine->tables_mu);
    for (int32_t i = 0; i < n; ++i) {
      const char* fname = reqs[i].feature_name ? reqs[i].feature_name : "";
      auto spec = engine->features.find(fname);
      if (spec == engine->features.end()) {
        return SetError(XSE_NOT_FOUND, "Feature spec not found for: %s", fname);
      }
      if (spec->second.max_sequence_length != 0) {
        return SetError(XSE_UNIMPLEMENTED,
                        "Batch request %d requires a non-sequence feature "
                        "specification.",
                        i);
      }
      auto table = engine->tables.find(spec->second.table);
      if (table == engine->tables.end()) {
        return SetError(XSE_NOT_FOUND, "Table not found for: %s",
                        spec->second.table.c_str());
      }
      tables[i] = table->second;
    }
  }

  DeviceGuard guard(engine->device);
  const bool async = (flags & XSE_EXEC_ASYNC) != 0;
  // A synchronous execution first settles earlier asynchronous ones; an
  // asynchronous one settles the ring only when it is full (an error found
  // then is reported by the next wait).
  if (st->used > 0 && (!async || st->used == st->ring)) {
    const int code = SettleStatus(st, stream);
    if (code != XSE_OK) {
      if (!async) return code;
      st->deferred_code = code;
      st->deferred_message = g_last_error;
    }
  }
  const int slot_index = st->used;
  StatusSlot& slot = st->slots[slot_index];
  slot.n = n;
  slot.early_code = XSE_OK;
  slot.early_message.clear();
  slot.meta.assign(static_cast<size_t>(n), RequestMeta());
  xse::DevStatus* const dev_status = st->dev_slot(slot_index);

  // Host-side checks (PrepareRequest, embedding_bag.cc:235-251).
  std::vector<xse::BagDesc> descs;
  descs.reserve(static_cast<size_t>(n));
  bool any_early = false;
  char buf[512];
  for (int32_t i = 0; i < n; ++i) {
    const xse_bag_request& r = reqs[i];
    const Table& t = *tables[i];
    RequestMeta& m = slot.meta[i];
    m.ids = r.ids;
    m.ids64 = r.ids_type == XSE_INDEX_I64;
    m.vocab = t.vocab;
    auto early = [&](int stage, int code, const char* text, bool prefix) {
      if (prefix) {
        snprintf(buf, sizeof(buf), "FP32 embedding-bag request %d: %s", i,
                 text);
      } else {
        snprintf(buf, sizeof(buf), text, i);
      }
      m.stage = stage;
      m.code = code;
      m.message = buf;
    };
    if (r.output == nullptr && inter == nullptr && parts == nullptr) {
      early(kStageEarly, XSE_INVALID_ARGUMENT,
            "FP32 embedding-bag request %d requires an output allocator.",
            false);
    } else if ((r.ids_type != XSE_INDEX_I32 && r.ids_type != XSE_INDEX_I64) ||
               (r.offsets_type != XSE_INDEX_I32 &&
                r.offsets_type != XSE_INDEX_I64)) {
      early(kStageEarly, XSE_INVALID_ARGUMENT,
            "Embedding IDs and row pointers must be int32 or int64.", true);
    } else if (r.num_offsets < 2 || r.offsets == nullptr) {
      early(kStageEarly, XSE_INVALID_ARGUMENT,
            "Row pointers must contain at least two elements.", true);
    } else if (r.num_ids < 0 || r.num_weights < 0 ||
               (r.output_stride != 0 && r.output_stride < t.dim)) {
      early(kStageEarly, XSE_INVALID_ARGUMENT,
            "Request sizes must be non-negative and the output stride at "
            "least the embedding dimension.",
            true);
    } else if (r.ids == nullptr && r.num_ids > 0) {
      early(kStageIdsNull, XSE_INVALID_ARGUMENT,
            "Embedding-ID storage must be non-null.", true);
    } else if (r.weights == nullptr && r.num_weights > 0) {
      early(kStageWeightsNull, XSE_INVALID_ARGUMENT,
            "Weight storage must be non-null.", true);
    }
    if (m.stage == kStageEarly) {
      any_early = true;
      continue;
    }
    xse::BagDesc d{};
    d.rows = t.rows;
    d.scale_bias = t.scale_bias;
    d.ids = m.stage == kStageIdsNull ? nullptr : r.ids;
    d.offsets = r.offsets;
    d.weights = (r.num_weights > 0 && m.stage != kStageWeightsNull)
                    ? r.weights
                    : nullptr;
    d.out = r.output;
    d.out_stride = r.output_stride > 0 ? r.output_stride : t.dim;
    d.vocab = t.vocab;
    d.row_begin = t.row_begin;
    d.row_end = t.row_end;
    d.num_ids = r.num_ids;
    d.num_weights = r.num_weights;
    d.num_bags = r.num_offsets - 1;
    d.dim = t.dim;
    d.slot = i;
    d.combine = static_cast<int8_t>(t.combine);
    d.ids64 = static_cast<int8_t>(r.ids_type == XSE_INDEX_I64);
    d.offs64 = static_cast<int8_t>(r.offsets_type == XSE_INDEX_I64);
    d.vec_out = static_cast<int8_t>(
        (reinterpret_cast<uintptr_t>(r.output) & 15u) == 0 &&
        d.out_stride % 4 == 0);
    descs.push_back(d);
  }
  // The first request's early error wins outright when no earlier request
  // can fail on the device.
  if (any_early && slot.meta[0].stage == kStageEarly) {
    return SetError(slot.meta[0].code, "%s", slot.meta[0].message.c_str());
  }
  if (inter != nullptr && !any_early) {
    const int dim = tables[0]->dim;
    const int64_t width =
        dim + static_cast<int64_t>(n + 1) * n / 2;
    for (int32_t i = 0; i < n; ++i) {
      const Table& t = *tables[i];
      if (t.dim != dim) {
        return SetError(XSE_INVALID_ARGUMENT,
                        "Interaction request %d has dimension %d; request 0 "
                        "has %d.",
                        i, t.dim, dim);
      }
      if (reqs[i].num_offsets - 1 != inter->batch) {
        return SetError(XSE_INVALID_ARGUMENT,
                        "Interaction request %d has %lld bags; the batch has "
                        "%lld samples.",
                        i, static_cast<long long>(reqs[i].num_offsets - 1),
                        static_cast<long long>(inter->batch));
      }
      if (t.row_begin != 0 || t.row_end != t.vocab) {
        return SetError(XSE_INVALID_ARGUMENT,
                        "Interaction request %d reads a row-wise shard "
                        "window; the interaction needs whole tables.",
                        i);
      }
    }
    if (inter->dense_stride < dim || inter->out_stride < width) {
      return SetError(XSE_INVALID_ARGUMENT,
                      "Interaction strides too small: dense %lld (dimension "
                      "%d), output %lld (width %lld).",
                      static_cast<long long>(inter->dense_stride), dim,
                      static_cast<long long>(inter->out_stride),
                      static_cast<long long>(width));
    }
  }
  // The parts' descriptors: their whole request's, with the part's bags
  // and output (a part's slot is its whole request's).
  std::vector<xse::BagDesc> part_descs;
  std::vector<std::shared_ptr<Table>> part_tables;
  if (parts != nullptr && !any_early) {
    part_descs.reserve(static_cast<size_t>(parts->n));
    part_tables.reserve(static_cast<size_t>(parts->n));
    for (int32_t j = 0; j < parts->n; ++j) {
      const xse_bag_request& r = parts->reqs[j];
      const int32_t o = parts->owner[j];
      if (o < 0 || o >= n || r.output == nullptr || r.offsets == nullptr ||
          r.num_offsets < 2 || r.offsets_type != reqs[o].offsets_type ||
          r.output_stride < 0 ||
          (r.output_stride != 0 && r.output_stride < tables[o]->dim)) {
        return SetError(XSE_INTERNAL, "malformed part %d of an execution", j);
      }
      xse::BagDesc d = descs[static_cast<size_t>(o)];
      d.offsets = r.offsets;
      d.num_bags = r.num_offsets - 1;
      d.out = r.output;
      d.out_stride = r.output_stride > 0 ? r.output_stride : tables[o]->dim;
      d.vec_out = static_cast<int8_t>(
          (reinterpret_cast<uintptr_t>(r.output) & 15u) == 0 &&
          d.out_stride % 4 == 0);
      part_descs.push_back(d);
      part_tables.push_back(tables[o]);
    }
    if (parts->blocks > 0) {
      // One blocked descriptor per whole request instead of one per part.
      if (parts->blocks > xse::kMaxOutBlocks || parts->block_bags <= 0 ||
          parts->block_base == nullptr || parts->block_offset == nullptr ||
          parts->block_stride <= 0 ||
          parts->block_bags * parts->blocks > INT32_MAX) {
        return SetError(XSE_INTERNAL, "malformed blocked execution");
      }
      bool aligned = parts->block_stride % 4 == 0;
      for (int32_t j = 0; j < parts->blocks; ++j) {
        aligned = aligned &&
                  (reinterpret_cast<uintptr_t>(parts->block_base[j]) & 15u) == 0;
      }
      part_descs.clear();
      for (int32_t k = 0; k < n; ++k) {
        xse::BagDesc d = descs[static_cast<size_t>(k)];
        if (d.num_bags != parts->block_bags * parts->blocks ||
            parts->block_stride < d.dim) {
          return SetError(XSE_INTERNAL, "malformed blocked execution");
        }
        d.block_bags = parts->block_bags;
        d.out_offset = parts->block_offset[k];
        d.out = parts->block_base[0] + d.out_offset;
        d.out_stride = parts->block_stride;
        d.vec_out = static_cast<int8_t>(aligned && d.out_offset % 4 == 0);
        part_descs.push_back(d);
      }
    }
  }
  std::string iso_message;
  int iso_code = XSE_OK;
  if (!any_early && inter == nullptr) {
    iso_code = parts != nullptr
                   ? CheckIsolation(parts->reqs, part_tables, parts->n,
                                    &iso_message)
                   : CheckIsolation(reqs, tables, n, &iso_message);
  }

  // Clear this execution's slot: the whole ring when an asynchronous run of
  // executions starts, only slot 0 for a synchronous one.
  cudaError_t e = cudaSuccess;
  if (async && slot_index == 0) {
    e = cudaMemsetAsync(st->dev, 0, st->slot_bytes * st->ring, stream);
    st->need_reset = false;
  } else if (!async || st->need_reset) {
    e = cudaMemsetAsync(dev_status, 0, xse::DevStatusBytes(n), stream);
  }
  if (e != cudaSuccess) return CudaError(e, "status reset");
  const bool fused = (flags & XSE_EXEC_FUSED) != 0;
  const bool validate_only = any_early || iso_code != XSE_OK;
  const bool any_soft = std::any_of(
      slot.meta.begin(), slot.meta.end(),
      [](const RequestMeta& m) { return m.stage != kStageNone; });

  // Validation pass over every descriptor (strict mode, or whenever the
  // group is known to fail and only its error order is needed).
  int launches = 0;
  const bool validate =
      parts == nullptr || parts->validate || validate_only || any_soft;
  const bool run_validation = (!fused || validate_only || any_soft) && validate;
  // Kernel timing (a copy of the engine's event set: the vector may grow
  // under another caller).
  xse_engine::ProfileEvents timing{};
  if (!validate_only && !any_soft) {
    std::lock_guard<std::mutex> lock(engine->profile_mu);
    if (engine->profile_period > 0 &&
        engine->profile_calls++ % engine->profile_period == 0) {
      if (engine->profile_used == engine->profile_events.size()) {
        xse_engine::ProfileEvents ev;
        cudaEventCreate(&ev.validate);
        cudaEventCreate(&ev.pool);
        cudaEventCreate(&ev.end);
        engine->profile_events.push_back(ev);
      }
      xse_engine::ProfileEvents& ev =
          engine->profile_events[engine->profile_used++];
      ev.validated = run_validation;
      timing = ev;
    }
  }
  if (timing.validate != nullptr && run_validation) {
    cudaEventRecord(timing.validate, stream);
  }
  if (run_validation) {
    for (size_t base = 0; base < descs.size();
         base += xse::kMaxDescsPerLaunch) {
      xse::PoolParams p{};
      p.status = dev_status;
      int64_t work = 0;
      const size_t cnt =
          std::min<size_t>(xse::kMaxDescsPerLaunch, descs.size() - base);
      for (size_t k = 0; k < cnt; ++k) {
        p.d[k] = descs[base + k];
        p.d[k].work_begin = work;
        work += xse::ValidationWork(p.d[k].num_bags, p.d[k].num_ids);
      }
      p.n = static_cast<int32_t>(cnt);
      e = xse::LaunchValidate(p, work, stream);
      if (e != cudaSuccess) return CudaError(e, "validation launch");
      ++launches;
    }
  }
  if (!validate_only && !any_soft) {
    if (timing.pool != nullptr) cudaEventRecord(timing.pool, stream);
    auto layout_of = [&](const xse::BagDesc& d) {
      xse::Layout l = xse::ChooseLayout(tables[d.slot]->dtype, d.dim, d.rows);
      if (tables[d.slot]->dtype == XSE_DT_I8_ROWWISE &&
          d.scale_bias == nullptr) {
        l.v = 0;  // an empty int8 window: the element-wise kernel
        l.exact = false;
      }
      return l;
    };
    // Pooling launches: descriptors grouped by kernel layout, request order
    // kept within each group.
    auto launch_groups = [&]() -> cudaError_t {
      std::map<std::tuple<int, int, int, bool, int>,
               std::vector<xse::BagDesc>>
          groups;
      for (const xse::BagDesc& d : parts != nullptr ? part_descs : descs) {
        const xse::Layout l = layout_of(d);
        // One launch per layout; its weighting modes share it.
        groups[{l.dtype, l.g, l.v, l.exact, l.wide ? 1 : 0}].push_back(d);
      }
      for (auto& [key, list] : groups) {
        const xse::Layout l{std::get<0>(key), std::get<1>(key),
                            std::get<2>(key), std::get<3>(key), 0,
                            std::get<4>(key) != 0};
        for (size_t base = 0; base < list.size();
             base += xse::kMaxDescsPerLaunch) {
          xse::PoolParams p{};
          p.status = dev_status;
          p.fused_checks = fused ? 1 : 0;
          if (parts != nullptr && parts->blocks > 0) {
            for (int32_t j = 0; j < parts->blocks; ++j) {
              p.block_base[j] = parts->block_base[j];
            }
          }
          const size_t cnt =
              std::min<size_t>(xse::kMaxDescsPerLaunch, list.size() - base);
          int64_t tasks = 0;
          for (size_t k = 0; k < cnt; ++k) {
            p.d[k] = list[base + k];
            p.d[k].task_begin = tasks;
            tasks += xse::TasksFor(l, p.d[k].num_bags);
          }
          p.n = static_cast<int32_t>(cnt);
          p.total_tasks = tasks;
          uint64_t key = 0;
          const PoolTrial trial = ChoosePoolKernel(engine, l, &p, &key);
          // A failed record only spoils the trial (PollTrials drops it).
          if (trial.start != nullptr &&
              cudaEventRecord(trial.start, stream) != cudaSuccess) {
            (void)cudaGetLastError();
          }
          cudaError_t le = xse::LaunchPool(l, p, stream, &launches);
          if (trial.start != nullptr) {
            if (cudaEventRecord(trial.end, stream) != cudaSuccess) {
              (void)cudaGetLastError();
            }
            AddTrial(engine, key, trial);
          }
          if (le != cudaSuccess) return le;
        }
      }
      return cudaSuccess;
    };
    if (inter == nullptr) {
      e = launch_groups();
      if (e != cudaSuccess) return CudaError(e, "pooling launch");
    } else {
      // Fused when every request has the layout of request 0 and a fused
      // kernel serves it.
      const xse::Layout l0 = layout_of(descs[0]);
      bool same = descs.size() <= static_cast<size_t>(xse::kMaxDescsPerLaunch);
      for (const xse::BagDesc& d : descs) {
        const xse::Layout l = layout_of(d);
        same = same && l.dtype == l0.dtype && l.g == l0.g && l.v == l0.v &&
               l.exact == l0.exact && l.wide == l0.wide;
      }
      e = cudaErrorNotSupported;
      if (same) {
        xse::PoolParams p{};
        p.status = dev_status;
        p.fused_checks = fused ? 1 : 0;
        for (size_t k = 0; k < descs.size(); ++k) p.d[k] = descs[k];
        p.n = static_cast<int32_t>(descs.size());
        e = xse::LaunchPoolInteract(l0, p, *inter, stream);
        if (e == cudaSuccess) ++launches;
      }
      if (e == cudaErrorNotSupported) {
        (void)cudaGetLastError();
        // Unfused: pool into scratch, then the interaction kernel.
        const int dim = descs[0].dim;
        const int64_t width = static_cast<int64_t>(n) * dim;
        float* scratch = nullptr;
        const size_t bytes = static_cast<size_t>(
            std::max<int64_t>(inter->batch * width, 4) * sizeof(float));
        e = cudaMallocAsync(reinterpret_cast<void**>(&scratch), bytes, stream);
        if (e != cudaSuccess) return CudaError(e, "interaction scratch");
        for (size_t k = 0; k < descs.size(); ++k) {
          descs[k].out = scratch + k * dim;
          descs[k].out_stride = width;
          descs[k].vec_out = static_cast<int8_t>(dim % 4 == 0);
        }
        e = launch_groups();
        if (e == cudaSuccess) {
          e = xse::LaunchDotInteraction(inter->dense, inter->dense_stride,
                                        scratch, width, inter->batch, n, dim,
                                        inter->out, inter->out_stride,
                                        stream);
          ++launches;
        }
        if (e == cudaSuccess && inter->out_lo != nullptr) {
          // The split operands in place (hi over the values).
          if (xse_tf32_split(inter->out, inter->batch,
                             static_cast<int32_t>(inter->out_stride),
                             inter->out_stride, inter->out, inter->out_lo,
                             stream) != XSE_OK) {
            e = cudaErrorLaunchFailure;
          }
          ++launches;
        }
        cudaError_t fe = cudaFreeAsync(scratch, stream);
        if (e == cudaSuccess) e = fe;
      }
      if (e != cudaSuccess) return CudaError(e, "interaction launch");
    }
    if (timing.end != nullptr) cudaEventRecord(timing.end, stream);
  }
  g_last_launches = launches;
  if (iso_code != XSE_OK) {
    slot.early_code = iso_code;
    slot.early_message = iso_message;
  }
  st->used = slot_index + 1;
  if (async && !validate_only && !any_soft) return Ok();
  // Synchronous, or the group is known to fail: read the result now.
  const int code = SettleStatus(st, stream);
  if (code == XSE_OK && (any_early || any_soft)) {
    // Unreachable: an early or soft error always resolves to a failure.
    return SetError(XSE_INTERNAL, "unresolved request error");
  }
  return code;
}

// Asynchronous executions recorded before a read-back is forced.
constexpr int32_t kStatusRing = 64;

// Status blocks of `ring` slots of `capacity` requests each.
int CreateStatus(int device, int32_t capacity, int32_t ring,
                 xse_status** out) {
  auto st = std::make_unique<xse_status>();
  st->device = device;
  st->capacity = capacity;
  st->ring = ring;
  st->slot_bytes = (xse::DevStatusBytes(capacity) + 255) / 256 * 256;
  st->slots.resize(static_cast<size_t>(ring));
  const size_t bytes = st->slot_bytes * ring;
  cudaError_t e = cudaMalloc(&st->dev, bytes);
  if (e != cudaSuccess) return CudaError(e, "status allocation");
  e = cudaMallocHost(&st->host, bytes);
  if (e != cudaSuccess) {
    cudaFree(st->dev);
    return CudaError(e, "status allocation");
  }
  std::memset(st->host, 0, bytes);
  *out = st.release();
  return XSE_OK;
}

}  // namespace

extern "C" {

const char* xse_last_error(void) { return g_last_error.c_str(); }
int32_t xse_abi_version(void) { return XSE_ABI_VERSION; }
int32_t xse_last_launch_count(void) { return g_last_launches; }

int xse_engine_create(const xse_engine_options* options, xse_engine** out) {
  if (out == nullptr) return SetError(XSE_INVALID_ARGUMENT, "out is null");
  int count = 0;
  cudaError_t e = cudaGetDeviceCount(&count);
  if (e != cudaSuccess || count <= 0) {
    return SetError(XSE_FAILED_PRECONDITION,
                    "No CUDA device is available for the embedding engine.");
  }
  auto engine = std::make_unique<xse_engine>();
  engine->device = options ? options->device : 0;
  if (engine->device < 0 || engine->device >= count) {
    return SetError(XSE_INVALID_ARGUMENT, "Device %d does not exist.",
                    engine->device);
  }
  DeviceGuard guard(engine->device);
  const int code =
      CreateStatus(engine->device, 256, 1, &engine->default_status);
  if (code != XSE_OK) return code;
  *out = engine.release();
  return Ok();
}

void xse_status_destroy(xse_status* status) {
  if (status == nullptr) return;
  DeviceGuard guard(status->device);
  cudaFree(status->dev);
  cudaFreeHost(status->host);
  delete status;
}

void xse_engine_destroy(xse_engine* engine) {
  if (engine == nullptr) return;
  {
    DeviceGuard guard(engine->device);
    cudaDeviceSynchronize();
  }
  xse_status_destroy(engine->default_status);
  for (auto& ev : engine->profile_events) {
    cudaEventDestroy(ev.validate);
    cudaEventDestroy(ev.pool);
    cudaEventDestroy(ev.end);
  }
  for (auto& [key, tuner] : engine->tuners) {
    (void)key;
    for (const PoolTrial& trial : tuner.pending) {
      cudaEventDestroy(trial.start);
      cudaEventDestroy(trial.end);
    }
  }
  delete engine;
}

int xse_engine_set_profiling(xse_engine* engine, int32_t period) {
  if (engine == nullptr) return SetError(XSE_INVALID_ARGUMENT, "null engine");
  if (period < 0) {
    return SetError(XSE_INVALID_ARGUMENT, "profiling period must be >= 0");
  }
  std::lock_guard<std::mutex> lock(engine->profile_mu);
  engine->profile_period = period;
  engine->profile_calls = 0;
  engine->profile_used = 0;
  return Ok();
}

int xse_engine_profile_read_stages(xse_engine* engine, double* validate_ms,
                                   int64_t* validated, double* pool_ms,
                                   int64_t* executions, int64_t* calls) {
  if (engine == nullptr || pool_ms == nullptr || executions == nullptr) {
    return SetError(XSE_INVALID_ARGUMENT, "arguments must be non-null");
  }
  DeviceGuard guard(engine->device);
  std::lock_guard<std::mutex> lock(engine->profile_mu);
  double total = 0.0, vtotal = 0.0;
  int64_t vcount = 0;
  for (size_t k = 0; k < engine->profile_used; ++k) {
    const auto& ev = engine->profile_events[k];
    cudaError_t e = cudaEventSynchronize(ev.end);
    if (e != cudaSuccess) return CudaError(e, "profile event");
    float ms = 0.0f;
    e = cudaEventElapsedTime(&ms, ev.pool, ev.end);
    if (e != cudaSuccess) return CudaError(e, "profile elapsed time");
    total += ms;
    if (ev.validated) {
      e = cudaEventElapsedTime(&ms, ev.validate, ev.pool);
      if (e != cudaSuccess) return CudaError(e, "profile elapsed time");
      vtotal += ms;
      ++vcount;
    }
  }
  *pool_ms = total;
  *executions = static_cast<int64_t>(engine->profile_used);
  if (validate_ms != nullptr) *validate_ms = vtotal;
  if (validated != nullptr) *validated = vcount;
  if (calls != nullptr) *calls = engine->profile_calls;
  engine->profile_used = 0;
  engine->profile_calls = 0;
  return Ok();
}

int xse_engine_profile_read(xse_engine* engine, double* pool_ms,
                            int64_t* executions, int64_t* calls) {
  return xse_engine_profile_read_stages(engine, nullptr, nullptr, pool_ms,
                                        executions, calls);
}

}  // extern "C"

namespace xse {

// Host -> HBM copy of table rows through pinned staging: chunk k is filled
// into pinned buffer k % 2 by `threads` host threads while chunk k - 1's DMA
// runs, so reading and PCIe overlap. The fill reads the file `fd` at
// file_offset with pread (no page faults on a mapping) when fd >= 0, else
// copies from `src` (pageable memory). chunk <= 0 copies straight from
// `src` (one pageable cudaMemcpy).
cudaError_t UploadFromHost(void* dst, const void* src, size_t bytes,
                           int64_t chunk, int threads, int fd,
                           int64_t file_offset) {
  if (bytes == 0) return cudaSuccess;
  if (chunk <= 0) return cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice);
  cudaPointerAttributes attr{};
  if (fd < 0 && cudaPointerGetAttributes(&attr, src) == cudaSuccess &&
      attr.type == cudaMemoryTypeHost) {  // already pinned
    return cudaMemcpy(dst, src, bytes, cudaMemcpyHostToDevice);
  }
  (void)cudaGetLastError();
  std::atomic<bool> read_failed{false};
  // Fills n bytes at dst from source offset `at`.
  auto fill = [&](char* to, size_t at, size_t n) {
    if (fd < 0) {
      std::memcpy(to, static_cast<const char*>(src) + at, n);
      return;
    }
    while (n > 0) {
      const ssize_t r = pread(fd, to, n, static_cast<off_t>(file_offset + at));
      if (r < 0 && errno == EINTR) continue;
      if (r <= 0) {
        read_failed = true;
        return;
      }
      to += r;
      at += static_cast<size_t>(r);
      n -= static_cast<size_t>(r);
    }
  };
  const size_t step = std::min<size_t>(static_cast<size_t>(chunk), bytes);
  if (threads < 1) threads = 1;
  void* pinned[2] = {nullptr, nullptr};
  cudaEvent_t done[2] = {nullptr, nullptr};
  cudaStream_t stream = nullptr;
  cudaError_t e = cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking);
  for (int b = 0; b < 2 && e == cudaSuccess; ++b) {
    e = cudaHostAlloc(&pinned[b], step, cudaHostAllocDefault);
    if (e == cudaSuccess) {
      e = cudaEventCreateWithFlags(&done[b], cudaEventDisableTiming);
    }
  }
  char* to = static_cast<char*>(dst);
  for (size_t off = 0, k = 0; off < bytes && e == cudaSuccess;
       off += step, ++k) {
    const size_t len = std::min(step, bytes - off);
    const int b = static_cast<int>(k & 1);
    if (k >= 2) e = cudaEventSynchronize(done[b]);  // buffer b is free
    if (e != cudaSuccess) break;
    // Parallel fill of the staging buffer (4 KiB-aligned slices).
    const size_t per = std::max<size_t>((len / threads + 4095) / 4096 * 4096,
                                        4096);
    char* stage = static_cast<char*>(pinned[b]);
    std::vector<std::thread> pool;
    for (int i = 1; i < threads && per * i < len; ++i) {
      pool.emplace_back([&, i]() {
        const size_t lo = per * i, hi = std::min(len, per * (i + 1));
        fill(stage + lo, off + lo, hi - lo);
      });
    }
    fill(stage, off, std::min(len, per));
    for (auto& th : pool) th.join();
    if (read_failed) {
      e = cudaErrorFileNotFound;
      break;
    }
    e = cudaMemcpyAsync(to + off, pinned[b], len, cudaMemcpyHostToDevice,
                        stream);
    if (e == cudaSuccess) e = cudaEventRecord(done[b], stream);
  }
  const cudaError_t se = stream ? cudaStreamSynchronize(stream) : cudaSuccess;
  if (e == cudaSuccess) e = se;
  for (int b = 0; b < 2; ++b) {
    if (done[b]) cudaEventDestroy(done[b]);
    if (pinned[b]) cudaFreeHost(pinned[b]);
  }
  if (stream) cudaStreamDestroy(stream);
  return e;
}

int AddTable(xse_engine* engine, const xse_table_desc* desc,
             int64_t upload_chunk, int upload_threads, int fd,
             int64_t file_offset) {
  if (engine == nullptr || desc == nullptr) {
    return SetError(XSE_INVALID_ARGUMENT, "engine and table must be non-null");
  }
  if (desc->name == nullptr || desc->name[0] == '\0') {
    return SetError(XSE_INVALID_ARGUMENT,
                    "Embedding table name cannot be empty.");
  }
  if (desc->dtype < XSE_DT_F32 || desc->dtype > XSE_DT_I8_ROWWISE) {
    return SetError(XSE_INVALID_ARGUMENT, "Unsupported data type: %d",
                    desc->dtype);
  }
  if (desc->combine < XSE_COMBINE_SUM || desc->combine > XSE_COMBINE_SQRTN) {
    return SetError(XSE_INVALID_ARGUMENT, "Unknown combine mode for table: %s",
                    desc->name);
  }
  if (desc->vocab <= 0 || desc->dim <= 0) {
    return SetError(XSE_INVALID_ARGUMENT,
                    "Table dimensions must be strictly positive. Got "
                    "vocab_size: %" PRId64 ", embedding_dim: %d",
                    desc->vocab, desc->dim);
  }
  int64_t row_begin = desc->row_begin, row_end = desc->row_end;
  if (row_begin == 0 && row_end == 0) row_end = desc->vocab;
  if (row_begin < 0 || row_end > desc->vocab || row_end < row_begin) {
    return SetError(XSE_INVALID_ARGUMENT,
                    "Shard window [%" PRId64 ", %" PRId64
                    ") is outside the table's %" PRId64 " rows.",
                    row_begin, row_end, desc->vocab);
  }
  const int64_t rows = row_end - row_begin;
  if (rows > 0 && desc->rows == nullptr) {
    return SetError(XSE_INVALID_ARGUMENT, "Table rows must be non-null.");
  }
  if (desc->dtype == XSE_DT_I8_ROWWISE && rows > 0 &&
      (desc->scale == nullptr || desc->bias == nullptr)) {
    return SetError(XSE_INVALID_ARGUMENT,
                    "Int8 row-wise tables need per-row scale and bias.");
  }
  {
    std::lock_guard<std::mutex> lock(engine->tables_mu);
    if (engine->tables.count(desc->name)) {
      return SetError(XSE_ALREADY_EXISTS, "Table already exists: %s",
                      desc->name);
    }
  }
  DeviceGuard guard(engine->device);
  auto t = std::make_shared<Table>();
  t->name = desc->name;
  t->dtype = desc->dtype;
  t->combine = desc->combine;
  t->dim = desc->dim;
  t->vocab = desc->vocab;
  t->row_begin = row_begin;
  t->row_end = row_end;
  t->device = engine->device;
  const size_t bytes =
      static_cast<size_t>(rows) * desc->dim * ElemBytes(desc->dtype);
  cudaError_t e = cudaSuccess;
  if (desc->placement == XSE_PLACE_ADOPT_DEVICE) {
    t->rows = const_cast<void*>(desc->rows);
  } else if (bytes > 0) {
    e = cudaMalloc(&t->rows, bytes);
    if (e != cudaSuccess) return CudaError(e, "table allocation");
    t->owns_rows = true;
    e = desc->placement == XSE_PLACE_COPY_FROM_HOST
            ? UploadFromHost(t->rows, desc->rows, bytes, upload_chunk,
                             upload_threads, fd, file_offset)
            : cudaMemcpy(t->rows, desc->rows, bytes,
                         cudaMemcpyDeviceToDevice);
    if (e != cudaSuccess) return CudaError(e, "table upload");
  }
  if (desc->dtype == XSE_DT_I8_ROWWISE && rows > 0) {
    e = cudaMalloc(&t->scale_bias, sizeof(float2) * rows);
    if (e != cudaSuccess) return CudaError(e, "scale/bias allocation");
    if (desc->placement == XSE_PLACE_COPY_FROM_HOST) {
      std::vector<float2> sb(static_cast<size_t>(rows));
      for (int64_t r = 0; r < rows; ++r) {
        sb[r] = make_float2(desc->scale[r], desc->bias[r]);
      }
      e = cudaMemcpy(t->scale_bias, sb.data(), sizeof(float2) * rows,
                     cudaMemcpyHostToDevice);
    } else {
      e = xse::LaunchInterleaveScaleBias(desc->scale, desc->bias,
                                         t->scale_bias, rows, nullptr);
      if (e == cudaSuccess) e = cudaDeviceSynchronize();
    }
    if (e != cudaSuccess) return CudaError(e, "scale/bias upload");
  }
  std::lock_guard<std::mutex> lock(engine->tables_mu);
  auto [it, inserted] = engine->tables.emplace(t->name, t);
  if (!inserted) {
    return SetError(XSE_ALREADY_EXISTS, "Table already exists: %s",
                    desc->name);
  }
  return Ok();
}

}  // namespace xse

extern "C" {

int xse_engine_add_table(xse_engine* engine, const xse_table_desc* desc) {
  return xse::AddTable(engine, desc, xse::kDefaultUploadChunk,
                       xse::kDefaultUploadThreads, -1, 0);
}

int xse_engine_register_feature(xse_engine* engine, const char* feature,
                                const char* table,
                                int32_t max_sequence_length) {
  if (engine == nullptr || feature == nullptr || table == nullptr) {
    return SetError(XSE_INVALID_ARGUMENT, "arguments must be non-null");
  }
  std::lock_guard<std::mutex> lock(engine->specs_mu);
  auto [it, inserted] = engine->features.emplace(
      feature, Feature{table, max_sequence_length});
  if (!inserted) {
    return SetError(XSE_ALREADY_EXISTS, "Feature spec already registered: %s",
                    feature);
  }
  return Ok();
}

int xse_engine_clear(xse_engine* engine) {
  if (engine == nullptr) return SetError(XSE_INVALID_ARGUMENT, "null engine");
  std::lock_guard<std::mutex> spec_lock(engine->specs_mu);
  std::lock_guard<std::mutex> table_lock(engine->tables_mu);
  engine->features.clear();
  engine->tables.clear();
  return Ok();
}

int xse_engine_table_info(xse_engine* engine, const char* table,
                          xse_table_info* out) {
  if (engine == nullptr || table == nullptr || out == nullptr) {
    return SetError(XSE_INVALID_ARGUMENT, "arguments must be non-null");
  }
  std::lock_guard<std::mutex> lock(engine->tables_mu);
  auto it = engine->tables.find(table);
  if (it == engine->tables.end()) {
    return SetError(XSE_NOT_FOUND, "Table not found for table: %s", table);
  }
  const Table& t = *it->second;
  out->dtype = t.dtype;
  out->combine = t.combine;
  out->dim = t.dim;
  out->reserved = 0;
  out->vocab = t.vocab;
  out->row_begin = t.row_begin;
  out->row_end = t.row_end;
  out->rows = t.rows;
  return Ok();
}

int xse_engine_feature_table(xse_engine* engine, const char* feature,
                             char* buf, int32_t buflen,
                             int32_t* max_sequence_length) {
  if (engine == nullptr || feature == nullptr) {
    return SetError(XSE_INVALID_ARGUMENT, "arguments must be non-null");
  }
  std::lock_guard<std::mutex> lock(engine->specs_mu);
  auto it = engine->features.find(feature);
  if (it == engine->features.end()) {
    return SetError(XSE_NOT_FOUND, "Feature spec not found for feature: %s",
                    feature);
  }
  if (buf != nullptr && buflen > 0) {
    snprintf(buf, static_cast<size_t>(buflen), "%s", it->second.table.c_str());
  }
  if (max_sequence_length != nullptr) {
    *max_sequence_length = it->second.max_sequence_length;
  }
  return Ok();
}

int xse_status_create(int32_t max_requests, xse_status** out) {
  if (out == nullptr || max_requests <= 0) {
    return SetError(XSE_INVALID_ARGUMENT,
                    "max_requests must be positive and out non-null");
  }
  int device = 0;
  cudaGetDevice(&device);
  const int code = CreateStatus(device, max_requests, kStatusRing, out);
  return code == XSE_OK ? Ok() : code;
}

int xse_engine_execute_batch(xse_engine* engine, const xse_bag_request* reqs,
                             int32_t n, void* stream, int32_t flags,
                             xse_status* status) {
  xse::TraceRange trace("xse.execute_batch");
  if (engine == nullptr) return SetError(XSE_INVALID_ARGUMENT, "null engine");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (status != nullptr) {
    return ExecuteBatch(engine, reqs, n, s, flags, status);
  }
  if ((flags & XSE_EXEC_ASYNC) != 0) {
    return SetError(XSE_INVALID_ARGUMENT,
                    "Asynchronous execution needs a caller-owned status.");
  }
  std::lock_guard<std::mutex> lock(engine->default_status_mu);
  return ExecuteBatch(engine, reqs, n, s, flags, engine->default_status);
}

int xse_engine_execute_interaction(xse_engine* engine,
                                   const xse_bag_request* reqs, int32_t n,
                                   const float* dense, int64_t dense_stride,
                                   int64_t batch, float* out,
                                   int64_t out_stride, void* stream,
                                   int32_t flags, xse_status* status) {
  return xse_engine_execute_interaction_tf32(engine, reqs, n, dense,
                                             dense_stride, batch, out,
                                             nullptr, out_stride, stream,
                                             flags, status);
}

int xse_engine_execute_interaction_tf32(
    xse_engine* engine, const xse_bag_request* reqs, int32_t n,
    const float* dense, int64_t dense_stride, int64_t batch, float* out_hi,
    float* out_lo, int64_t out_stride, void* stream, int32_t flags,
    xse_status* status) {
  xse::TraceRange trace("xse.execute_interaction");
  float* out = out_hi;
  if (engine == nullptr) return SetError(XSE_INVALID_ARGUMENT, "null engine");
  if (dense == nullptr || out == nullptr || batch < 0) {
    return SetError(XSE_INVALID_ARGUMENT,
                    "Interaction needs dense rows, an output and a "
                    "non-negative batch.");
  }
  xse::InteractArgs a{};
  a.dense = dense;
  a.dense_stride = dense_stride;
  a.out = out;
  a.out_lo = out_lo;
  a.out_stride = out_stride;
  a.batch = batch;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (status != nullptr) {
    return ExecuteBatch(engine, reqs, n, s, flags, status, &a);
  }
  if ((flags & XSE_EXEC_ASYNC) != 0) {
    return SetError(XSE_INVALID_ARGUMENT,
                    "Asynchronous execution needs a caller-owned status.");
  }
  std::lock_guard<std::mutex> lock(engine->default_status_mu);
  return ExecuteBatch(engine, reqs, n, s, flags, engine->default_status, &a);
}

int xse_status_wait(xse_status* status, void* stream) {
  if (status == nullptr) return SetError(XSE_INVALID_ARGUMENT, "null status");
  DeviceGuard guard(status->device);
  return SettleStatus(status, static_cast<cudaStream_t>(stream));
}

int xse_dot_interaction(const float* dense, const float* pooled,
                        int64_t batch, int32_t num_tables, int32_t dim,
                        float* out, void* stream) {
  const int64_t rows = static_cast<int64_t>(num_tables) + 1;
  return xse_dot_interaction_strided(
      dense, dim, pooled, static_cast<int64_t>(num_tables) * dim, batch,
      num_tables, dim, out, dim + rows * (rows - 1) / 2, stream);
}

int xse_dot_interaction_strided(const float* dense, int64_t dense_stride,
                                const float* pooled, int64_t pooled_stride,
                                int64_t batch, int32_t num_tables,
                                int32_t dim, float* out, int64_t out_stride,
                                void* stream) {
  g_last_launches = 0;
  if (batch < 0 || num_tables < 1 || dim < 1) {
    return SetError(XSE_INVALID_ARGUMENT,
                    "Interaction needs batch >= 0, at least one table and a "
                    "positive dimension.");
  }
  const int64_t rows = static_cast<int64_t>(num_tables) + 1;
  const int64_t width = dim + rows * (rows - 1) / 2;
  if (dense_stride < dim || pooled_stride < static_cast<int64_t>(num_tables) * dim ||
      out_stride < width) {
    return SetError(XSE_INVALID_ARGUMENT,
                    "Interaction strides must cover a row: dense >= %d, "
                    "pooled >= %lld, out >= %lld.", dim,
                    static_cast<long long>(num_tables) * dim,
                    static_cast<long long>(width));
  }
  if (batch > 0 && (dense == nullptr || pooled == nullptr || out == nullptr)) {
    return SetError(XSE_INVALID_ARGUMENT, "Interaction buffers must be non-null.");
  }
  const cudaError_t e = xse::LaunchDotInteraction(
      dense, dense_stride, pooled, pooled_stride, batch, num_tables, dim, out,
      out_stride, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return CudaError(e, "interaction launch");
  g_last_launches = batch > 0 ? 1 : 0;
  return Ok();
}

int xse_synth_table(void* rows, float* scale, float* bias, int32_t dtype,
                    uint64_t seed, uint64_t table, int64_t row0,
                    int64_t nrows, int32_t dim, void* stream) {
  if (dtype < XSE_DT_F32 || dtype > XSE_DT_I8_ROWWISE || nrows < 0 ||
      dim <= 0 || row0 < 0 || (nrows > 0 && rows == nullptr) ||
      (dtype == XSE_DT_I8_ROWWISE && nrows > 0 &&
       (scale == nullptr || bias == nullptr))) {
    return SetError(XSE_INVALID_ARGUMENT, "invalid synthetic table request");
  }
  const int rc = xse_synth_table_impl(rows, scale, bias, dtype, seed, table,
                                      row0, nrows, dim,
                                      static_cast<cudaStream_t>(stream));
  return rc == 0 ? Ok() : SetError(rc, "synthetic table launch failed");
}

int xse_synth_lengths(int64_t* lengths, int64_t n, int32_t lo, int32_t hi,
                      uint64_t seed, uint64_t table, void* stream) {
  if (n < 0 || lo < 0 || hi < lo || (n > 0 && lengths == nullptr)) {
    return SetError(XSE_INVALID_ARGUMENT, "invalid synthetic lengths request");
  }
  const int rc = xse_synth_lengths_impl(lengths, n, lo, hi, seed, table,
                                        static_cast<cudaStream_t>(stream));
  return rc == 0 ? Ok() : SetError(rc, "synthetic lengths launch failed");
}

int xse_synth_ids(int64_t* ids, int64_t n, int64_t vocab, double zipf_alpha,
                  uint64_t perm_mul, uint64_t perm_add, uint64_t seed,
                  uint64_t table, int64_t index0, void* stream) {
  if (n < 0 || vocab <= 0 || vocab >= (1ll << 31) ||
      perm_mul >= (1ull << 32) || perm_add >= (1ull << 32) ||
      (n > 0 && ids == nullptr) || index0 < 0) {
    return SetError(XSE_INVALID_ARGUMENT, "invalid synthetic ids request");
  }
  const int rc = xse_synth_ids_impl(ids, n, vocab, zipf_alpha, perm_mul,
                                    perm_add, seed, table, index0,
                                    static_cast<cudaStream_t>(stream));
  return rc == 0 ? Ok() : SetError(rc, "synthetic ids launch failed");
}

int xse_synth_weights(float* weights, int64_t n, uint64_t seed,
                      uint64_t table, int64_t index0, void* stream) {
  if (n < 0 || (n > 0 && weights == nullptr) || index0 < 0) {
    return SetError(XSE_INVALID_ARGUMENT, "invalid synthetic weights request");
  }
  const int rc = xse_synth_weights_impl(weights, n, seed, table, index0,
                                        static_cast<cudaStream_t>(stream));
  return rc == 0 ? Ok() : SetError(rc, "synthetic weights launch failed");
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free execution (xse_engine_execute_batch_noalloc).
//
// The status that xse_engine_execute_batch keeps in an allocated block lives
// here in one fixed device array. Everything else the call needs on the host
// (resolved tables, descriptors, the kernel parameter block, the status
// read-back) sits on the stack, so the call allocates nothing.

namespace {

constexpr int32_t kNoAllocMaxRequests = XSE_NOALLOC_MAX_REQUESTS;
static_assert(kNoAllocMaxRequests <= xse::kMaxDescsPerLaunch,
              "one validation launch covers the whole group");
constexpr size_t kNoAllocStatusBytes =
    sizeof(xse::DevStatus) +
    sizeof(xse::DevRequestStatus) * (kNoAllocMaxRequests - 1);

}  // namespace

// Device scratch of the allocation-free call: every GPU that loads this
// library holds one copy until the process exits. Host code only sees a
// stand-in for it; its device address comes from cudaGetSymbolAddress.
static __device__ __align__(256) unsigned char
    g_noalloc_status[kNoAllocStatusBytes];

namespace {

constexpr int kNoAllocMaxDevices = 64;
std::mutex g_noalloc_mu;
void* g_noalloc_address[kNoAllocMaxDevices] = {};

// Device address of the scratch array on `device` (which must be current),
// looked up on the first call per device.
int NoAllocScratch(int device, xse::DevStatus** out) {
  if (device < 0 || device >= kNoAllocMaxDevices) {
    return SetError(XSE_FAILED_PRECONDITION,
                    "Device %d is beyond the %d devices the allocation-free "
                    "call supports.",
                    device, kNoAllocMaxDevices);
  }
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_address[device] == nullptr) {
    void* address = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&address, g_noalloc_status);
    if (e != cudaSuccess) return CudaError(e, "scratch symbol address");
    g_noalloc_address[device] = address;
  }
  *out = static_cast<xse::DevStatus*>(g_noalloc_address[device]);
  return XSE_OK;
}

}  // namespace

extern "C" int xse_engine_execute_batch_noalloc(xse_engine* engine,
                                                const xse_bag_request* reqs,
                                                int32_t n, void* stream) {
  g_last_launches = 0;
  if (engine == nullptr) return SetError(XSE_INVALID_ARGUMENT, "null engine");
  if (n <= 0 || reqs == nullptr) {
    return SetError(XSE_INVALID_ARGUMENT,
                    "Embedding batch requires at least one request.");
  }
  if (n > kNoAllocMaxRequests) {
    return SetError(XSE_INVALID_ARGUMENT,
                    "The allocation-free call takes at most %d requests; got "
                    "%d. Split the group or use xse_engine_execute_batch.",
                    kNoAllocMaxRequests, n);
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  std::shared_ptr<Table> tables[kNoAllocMaxRequests];
  {
    std::lock_guard<std::mutex> spec_lock(engine->specs_mu);
    std::lock_guard<std::mutex> table_lock(engine->tables_mu);
    for (int32_t i = 0; i < n; ++i) {
      const char* fname = reqs[i].feature_name ? reqs[i].feature_name : "";
      // A scan instead of find(): find would build a std::string key.
      auto spec = engine->features.begin();
      while (spec != engine->features.end() &&
             std::strcmp(spec->first.c_str(), fname) != 0) {
        ++spec;
      }
      if (spec == engine->features.end()) {
        return SetError(XSE_NOT_FOUND, "Feature spec not found for: %s", fname);
      }
      if (spec->second.max_sequence_length != 0) {
        return SetError(XSE_UNIMPLEMENTED,
                        "Batch request %d requires a non-sequence feature "
                        "specification.",
                        i);
      }
      auto table = engine->tables.find(spec->second.table);
      if (table == engine->tables.end()) {
        return SetError(XSE_NOT_FOUND, "Table not found for: %s",
                        spec->second.table.c_str());
      }
      tables[i] = table->second;
    }
  }

  DeviceGuard guard(engine->device);
  xse::DevStatus* scratch = nullptr;
  int code = NoAllocScratch(engine->device, &scratch);
  if (code != XSE_OK) return code;

  // Host checks (PrepareRequest, embedding_bag.cc:235-251), kept per request
  // in stack arrays: a request's host-detectable error is reported only when
  // every earlier request has passed its device checks, as
  // xse_engine_execute_batch (and the reference's per-request loop,
  // embedding_bag.cc:493-497) order them.
  xse::PoolParams params{};  // kernel parameter block (~9 KB, on the stack)
  xse::BagDesc* descs = params.d;
  int32_t nd = 0;
  int8_t stage[kNoAllocMaxRequests] = {};
  const char* problem[kNoAllocMaxRequests] = {};
  bool any_early = false, any_soft = false;
  for (int32_t i = 0; i < n; ++i) {
    const xse_bag_request& r = reqs[i];
    const Table& t = *tables[i];
    if (r.output == nullptr) {
      stage[i] = kStageEarly;  // unprefixed message, formatted below
    } else if ((r.ids_type != XSE_INDEX_I32 && r.ids_type != XSE_INDEX_I64) ||
               (r.offsets_type != XSE_INDEX_I32 &&
                r.offsets_type != XSE_INDEX_I64)) {
      stage[i] = kStageEarly;
      problem[i] = "Embedding IDs and row pointers must be int32 or int64.";
    } else if (r.num_offsets < 2 || r.offsets == nullptr) {
      stage[i] = kStageEarly;
      problem[i] = "Row pointers must contain at least two elements.";
    } else if (r.num_ids < 0 || r.num_weights < 0 ||
               (r.output_stride != 0 && r.output_stride < t.dim)) {
      stage[i] = kStageEarly;
      problem[i] =
          "Request sizes must be non-negative and the output stride at least "
          "the embedding dimension.";
    } else if (r.ids == nullptr && r.num_ids > 0) {
      stage[i] = kStageIdsNull;
      problem[i] = "Embedding-ID storage must be non-null.";
    } else if (r.weights == nullptr && r.num_weights > 0) {
      stage[i] = kStageWeightsNull;
      problem[i] = "Weight storage must be non-null.";
    }
    if (stage[i] != kStageNone) any_soft = true;
    if (stage[i] == kStageEarly) {
      any_early = true;
      continue;
    }
    xse::BagDesc d{};
    d.rows = t.rows;
    d.scale_bias = t.scale_bias;
    d.ids = stage[i] == kStageIdsNull ? nullptr : r.ids;
    d.offsets = r.offsets;
    d.weights = (r.num_weights > 0 && stage[i] != kStageWeightsNull)
                    ? r.weights
                    : nullptr;
    d.out = r.output;
    d.out_stride = r.output_stride > 0 ? r.output_stride : t.dim;
    d.vocab = t.vocab;
    d.row_begin = t.row_begin;
    d.row_end = t.row_end;
    d.num_ids = r.num_ids;
    d.num_weights = r.num_weights;
    d.num_bags = r.num_offsets - 1;
    d.dim = t.dim;
    d.slot = i;
    d.combine = static_cast<int8_t>(t.combine);
    d.ids64 = static_cast<int8_t>(r.ids_type == XSE_INDEX_I64);
    d.offs64 = static_cast<int8_t>(r.offsets_type == XSE_INDEX_I64);
    d.vec_out = static_cast<int8_t>(
        (reinterpret_cast<uintptr_t>(r.output) & 15u) == 0 &&
        d.out_stride % 4 == 0);
    descs[nd++] = d;
  }
  auto early_error = [&](int32_t i) {
    if (problem[i] == nullptr) {
      return SetError(XSE_INVALID_ARGUMENT,
                      "FP32 embedding-bag request %d requires an output "
                      "allocator.",
                      i);
    }
    return SetError(XSE_INVALID_ARGUMENT, "FP32 embedding-bag request %d: %s",
                    i, problem[i]);
  };
  // Request 0's early error wins outright: no earlier request can fail.
  if (stage[0] == kStageEarly) return early_error(0);

  // Output isolation (embedding_bag.cc:304-351) on fixed arrays, with the
  // outputs visited in address order as CheckIsolation visits them. Checked
  // only when no request failed its early checks (as the regular call); an
  // isolation error is reported after every request's own errors.
  char iso_message[256];
  bool iso_failed = false;
  if (!any_early) {
    Range outputs[kNoAllocMaxRequests];
    Range inputs[kNoAllocMaxRequests * 4];
    int32_t n_out = 0, n_in = 0;
    for (int32_t i = 0; i < n; ++i) {
      const xse_bag_request& r = reqs[i];
      const Table& t = *tables[i];
      const int64_t bags = r.num_offsets - 1;
      const int64_t stride = r.output_stride > 0 ? r.output_stride : t.dim;
      if (bags > 0 && r.output != nullptr) {
        Range o{static_cast<int64_t>(reinterpret_cast<uintptr_t>(r.output)),
                stride * 4, static_cast<int64_t>(t.dim) * 4, bags, i,
                "output"};
        int32_t k = n_out++;  // insertion by base address
        while (k > 0 && outputs[k - 1].base > o.base) {
          outputs[k] = outputs[k - 1];
          --k;
        }
        outputs[k] = o;
      }
      auto add = [&](const void* p, int64_t bytes, const char* kind) {
        if (p != nullptr && bytes > 0) {
          inputs[n_in++] = {
              static_cast<int64_t>(reinterpret_cast<uintptr_t>(p)), bytes,
              bytes, 1, i, kind};
        }
      };
      add(r.ids, r.num_ids * (r.ids_type == XSE_INDEX_I64 ? 8 : 4),
          "embedding-ID");
      add(r.offsets, r.num_offsets * (r.offsets_type == XSE_INDEX_I64 ? 8 : 4),
          "row-pointer");
      add(r.weights, r.num_weights * 4, "weight");
      add(t.rows,
          (t.row_end - t.row_begin) * t.dim *
              static_cast<int64_t>(ElemBytes(t.dtype)),
          "embedding-table");
    }
    for (int32_t a = 0; a < n_out && !iso_failed; ++a) {
      for (int32_t b = a + 1; b < n_out && outputs[b].base < outputs[a].end();
           ++b) {
        if (Overlaps(outputs[a], outputs[b])) {
          snprintf(iso_message, sizeof(iso_message),
                   "FP32 embedding-bag request outputs %d and %d overlap.",
                   std::min(outputs[a].request, outputs[b].request),
                   std::max(outputs[a].request, outputs[b].request));
          iso_failed = true;
          break;
        }
      }
    }
    // Of the inputs an output meets, the first in request order is named.
    for (int32_t a = 0; a < n_out && !iso_failed; ++a) {
      for (int32_t b = 0; b < n_in; ++b) {
        if (Overlaps(outputs[a], inputs[b])) {
          snprintf(iso_message, sizeof(iso_message),
                   "FP32 embedding-bag request %d output overlaps request %d "
                   "%s storage.",
                   outputs[a].request, inputs[b].request, inputs[b].kind);
          iso_failed = true;
          break;
        }
      }
    }
  }

  // The array keeps the previous call's status: clear this call's part.
  cudaError_t e = cudaMemsetAsync(scratch, 0, xse::DevStatusBytes(n), s);
  if (e != cudaSuccess) return CudaError(e, "scratch reset");
  int launches = 0;
  {
    // The validation pass runs even when the group is known to fail, so
    // that an earlier request's device-detected error is the one reported.
    int64_t work = 0;
    for (int32_t k = 0; k < nd; ++k) {
      descs[k].work_begin = work;
      work += xse::ValidationWork(descs[k].num_bags, descs[k].num_ids);
    }
    params.n = nd;
    params.fused_checks = 0;
    params.status = scratch;
    e = xse::LaunchValidate(params, work, s);
    if (e != cudaSuccess) return CudaError(e, "validation launch");
    ++launches;
  }
  if (!any_soft && !iso_failed) {
    // One pooling launch per kernel layout, requests kept in order.
    xse::PoolParams group{};
    bool launched[kNoAllocMaxRequests] = {};
    for (int32_t i = 0; i < nd; ++i) {
      if (launched[i]) continue;
      const Table& ti = *tables[descs[i].slot];
      xse::Layout li = xse::ChooseLayout(ti.dtype, descs[i].dim, descs[i].rows);
      if (ti.dtype == XSE_DT_I8_ROWWISE && descs[i].scale_bias == nullptr) {
        li.v = 0;
        li.exact = false;
      }
      li.wmode = li.v == 0 ? 0 : xse::WeightModeOf(descs[i]);
      group.n = 0;
      group.fused_checks = 0;
      group.status = scratch;
      int64_t tasks = 0;
      for (int32_t j = i; j < nd; ++j) {
        if (launched[j]) continue;
        const Table& tj = *tables[descs[j].slot];
        xse::Layout lj =
            xse::ChooseLayout(tj.dtype, descs[j].dim, descs[j].rows);
        if (tj.dtype == XSE_DT_I8_ROWWISE && descs[j].scale_bias == nullptr) {
          lj.v = 0;
          lj.exact = false;
        }
        lj.wmode = lj.v == 0 ? 0 : xse::WeightModeOf(descs[j]);
        if (lj.dtype != li.dtype || lj.g != li.g || lj.v != li.v ||
            lj.exact != li.exact || lj.wide != li.wide) {
          continue;  // weighting modes share a launch
        }
        launched[j] = true;
        group.d[group.n] = descs[j];
        group.d[group.n].task_begin = tasks;
        tasks += descs[j].num_bags;
        ++group.n;
      }
      group.total_tasks = tasks;
      e = xse::LaunchPool(li, group, s, &launches);
      if (e != cudaSuccess) return CudaError(e, "pooling launch");
    }
  }
  g_last_launches = launches;

  // Read back this call's status into stack memory and resolve it in the
  // reference's order of checks: per request, its early error, its offset
  // errors, its null ids or weights, its out-of-range ids; then isolation.
  alignas(16) unsigned char host_buf[kNoAllocStatusBytes];
  e = cudaMemcpyAsync(host_buf, scratch, xse::DevStatusBytes(n),
                      cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return CudaError(e, "scratch read-back");
  const xse::DevStatus* st = reinterpret_cast<const xse::DevStatus*>(host_buf);
  for (int32_t i = 0; i < n; ++i) {
    if (stage[i] == kStageEarly) return early_error(i);
    const unsigned int flags = st->req[i].flags;
    const char* msg = nullptr;
    if (flags & xse::kErrBadOffsets) {
      msg = "Row pointers must be non-negative and monotonic.";
    } else if (flags & xse::kErrLastExceedsIds) {
      msg = "Final row pointer exceeds embedding IDs size.";
    } else if (flags & xse::kErrLastExceedsWeights) {
      msg = "Final row pointer exceeds weights size.";
    }
    if (msg != nullptr) {
      return SetError(XSE_INVALID_ARGUMENT, "FP32 embedding-bag request %d: %s",
                      i, msg);
    }
    if (stage[i] == kStageIdsNull || stage[i] == kStageWeightsNull) {
      return SetError(XSE_INVALID_ARGUMENT, "FP32 embedding-bag request %d: %s",
                      i, problem[i]);
    }
    if (flags & xse::kErrBadId) {
      const int64_t index = static_cast<int64_t>(~st->req[i].inv_min_bad_index);
      const bool ids64 = reqs[i].ids_type == XSE_INDEX_I64;
      int64_t id = 0;
      if (ids64) {
        e = cudaMemcpy(&id, static_cast<const int64_t*>(reqs[i].ids) + index,
                       sizeof(id), cudaMemcpyDeviceToHost);
      } else {
        int32_t id32 = 0;
        e = cudaMemcpy(&id32,
                       static_cast<const int32_t*>(reqs[i].ids) + index,
                       sizeof(id32), cudaMemcpyDeviceToHost);
        id = id32;
      }
      if (e != cudaSuccess) return CudaError(e, "id read-back");
      return SetError(XSE_INVALID_ARGUMENT,
                      "FP32 embedding-bag request %d: Embedding ID (%" PRId64
                      ") at index %" PRId64 " is out of bounds [0, %" PRId64
                      ").",
                      i, id, index, tables[i]->vocab);
    }
  }
  if (iso_failed) return SetError(XSE_INVALID_ARGUMENT, "%s", iso_message);
  return Ok();
}

// ---------------------------------------------------------------------------
// Legacy per-feature path (CpuEmbeddingEngine::Execute).

namespace {

int64_t ReadIndex(const void* base, int is64, int64_t i) {
  int64_t v = 0;
  if (is64) {
    cudaMemcpy(&v, static_cast<const int64_t*>(base) + i, sizeof(v),
               cudaMemcpyDeviceToHost);
  } else {
    int32_t v32 = 0;
    cudaMemcpy(&v32, static_cast<const int32_t*>(base) + i, sizeof(v32),
               cudaMemcpyDeviceToHost);
    v = v32;
  }
  return v;
}

}  // namespace

extern "C" int xse_engine_execute_legacy(xse_engine* engine,
                                         const xse_bag_request* reqs,
                                         int32_t n, void* stream) {
  g_last_launches = 0;
  if (engine == nullptr) return SetError(XSE_INVALID_ARGUMENT, "null engine");
  if (n < 0 || (n > 0 && reqs == nullptr)) {
    return SetError(XSE_INVALID_ARGUMENT, "bad request list");
  }
  if (n > xse::kMaxDescsPerLaunch) {
    return SetError(XSE_INVALID_ARGUMENT,
                    "At most %d features per legacy execution, got %d.",
                    xse::kMaxDescsPerLaunch, n);
  }
  // FeatureBatchCsrInput::Create's host-visible check
  // (feature_batch_csr_input.cc:36-39).
  for (int32_t i = 0; i < n; ++i) {
    if (reqs[i].num_offsets < 2) {
      return SetError(XSE_INVALID_ARGUMENT,
                      "Row pointers must have at least 2 elements.");
    }
  }
  // Specs, then tables (cpu_embedding_engine.cc:98-124).
  std::vector<Feature> specs(static_cast<size_t>(n));
  std::vector<std::shared_ptr<Table>> tables(static_cast<size_t>(n));
  {
    std::lock_guard<std::mutex> spec_lock(engine->specs_mu);
    for (int32_t i = 0; i < n; ++i) {
      const char* fname = reqs[i].feature_name ? reqs[i].feature_name : "";
      auto it = engine->features.find(fname);
      if (it == engine->features.end()) {
        return SetError(XSE_NOT_FOUND, "Feature spec not found for: %s", fname);
      }
      specs[i] = it->second;
    }
  }
  {
    std::lock_guard<std::mutex> table_lock(engine->tables_mu);
    for (int32_t i = 0; i < n; ++i) {
      auto it = engine->tables.find(specs[i].table);
      if (it == engine->tables.end()) {
        return SetError(XSE_NOT_FOUND, "Table not found for: %s",
                        specs[i].table.c_str());
      }
      tables[i] = it->second;
    }
  }
  xse::LegacyParams p = {};
  p.n = n;
  int64_t tasks = 0;
  for (int32_t i = 0; i < n; ++i) {
    const xse_bag_request& r = reqs[i];
    const Table& t = *tables[i];
    const bool sequence = specs[i].max_sequence_length > 0;
    if (t.dtype != XSE_DT_F32 && t.dtype != XSE_DT_BF16) {
      return SetError(XSE_INVALID_ARGUMENT, "Unsupported data type: %d",
                      t.dtype);
    }
    if (t.row_begin != 0 || t.row_end != t.vocab) {
      return SetError(XSE_FAILED_PRECONDITION,
                      "Table %s holds a row-wise shard; the per-feature path "
                      "needs whole tables.", t.name.c_str());
    }
    if (sequence && r.num_weights > 0) {
      return SetError(XSE_INVALID_ARGUMENT,
                      "Weights should be empty for sequence assembly.");
    }
    if ((r.num_ids > 0 && r.ids == nullptr) || r.offsets == nullptr ||
        r.output == nullptr || (r.num_weights > 0 && r.weights == nullptr)) {
      return SetError(XSE_INVALID_ARGUMENT,
                      "Legacy request %d has a null buffer.", i);
    }
    xse::LegacyDesc& d = p.d[i];
    d.rows = t.rows;
    d.ids = r.ids;
    d.offsets = r.offsets;
    d.weights = r.num_weights > 0 ? r.weights : nullptr;
    d.out = r.output;
    d.vocab = t.vocab;
    d.num_ids = r.num_ids;
    d.num_weights = r.num_weights;
    d.num_bags = r.num_offsets - 1;
    d.task_begin = tasks;
    d.max_seq = sequence ? specs[i].max_sequence_length : 0;
    d.dim = t.dim;
    d.slot = i;
    d.combine = static_cast<int8_t>(t.combine);
    d.ids64 = r.ids_type == XSE_INDEX_I64 ? 1 : 0;
    d.offs64 = r.offsets_type == XSE_INDEX_I64 ? 1 : 0;
    d.dtype = t.dtype == XSE_DT_F32 ? 0 : 1;
    d.kind = sequence ? xse::kLegacySequence
                      : (d.dtype == 0 ? xse::kLegacyPoolF32
                                      : xse::kLegacyPoolBf16);
    tasks += d.num_bags;
  }
  p.total_tasks = tasks;
  DeviceGuard guard(engine->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const size_t status_bytes = xse::DevStatusBytes(n > 0 ? n : 1);
  void* dev_status = nullptr;
  cudaError_t e = cudaMallocAsync(&dev_status, status_bytes, s);
  if (e != cudaSuccess) return CudaError(e, "legacy status allocation");
  e = cudaMemsetAsync(dev_status, 0, status_bytes, s);
  p.status = static_cast<xse::DevStatus*>(dev_status);
  if (e == cudaSuccess) e = xse::LaunchLegacy(p, s);
  std::vector<unsigned char> host(status_bytes);
  if (e == cudaSuccess) {
    e = cudaMemcpyAsync(host.data(), dev_status, status_bytes,
                        cudaMemcpyDeviceToHost, s);
  }
  cudaFreeAsync(dev_status, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return CudaError(e, "legacy execution");
  g_last_launches = tasks > 0 ? 2 : 0;
  const auto* st = reinterpret_cast<const xse::DevStatus*>(host.data());
  if (st->group_error == 0) return Ok();
  // FeatureBatchCsrInput's checks first (they precede Execute in the
  // reference), in request order (feature_batch_csr_input.cc:36-54).
  for (int32_t i = 0; i < n; ++i) {
    const unsigned int f = st->req[i].flags;
    const xse::LegacyDesc& d = p.d[i];
    if (f & (xse::kLegacySizeMismatch | xse::kLegacyNotSorted |
             xse::kLegacyWeights)) {
      const int64_t last = ReadIndex(d.offsets, d.offs64, d.num_bags);
      if (f & xse::kLegacySizeMismatch) {
        return SetError(XSE_INVALID_ARGUMENT,
                        "Embedding ids size (%" PRId64
                        ") does not match last element of row pointers "
                        "(%" PRId64 ")",
                        d.num_ids, last);
      }
      if (f & xse::kLegacyNotSorted) {
        return SetError(XSE_INVALID_ARGUMENT, "Row pointers are not sorted.");
      }
      return SetError(XSE_INVALID_ARGUMENT,
                      "Weights size (%" PRId64
                      ") does not match expected size (%" PRId64 ")",
                      d.num_weights, last);
    }
  }
  // Then the bounds scans (compute_activations.cc:89-98, 205-213).
  for (int32_t i = 0; i < n; ++i) {
    if ((st->req[i].flags & xse::kLegacyBadId) == 0) continue;
    const xse::LegacyDesc& d = p.d[i];
    const int64_t pos = static_cast<int64_t>(~st->req[i].inv_min_bad_index);
    const int64_t id = ReadIndex(d.ids, d.ids64, pos);
    int64_t index = pos;
    if (d.kind == xse::kLegacySequence) {  // position within its sample
      std::vector<int64_t> rp(static_cast<size_t>(d.num_bags) + 1);
      for (int64_t b = 0; b <= d.num_bags; ++b) {
        rp[b] = ReadIndex(d.offsets, d.offs64, b);
      }
      const auto it = std::upper_bound(rp.begin(), rp.end(), pos);
      index = pos - *(it - 1);
    }
    return SetError(XSE_INVALID_ARGUMENT,
                    "Embedding ID (%" PRId64 ") at index %" PRId64
                    " is out of bounds [0, %" PRId64 ") for table %s.",
                    id, index, d.vocab, tables[i]->name.c_str());
  }
  return SetError(XSE_INTERNAL, "legacy execution failed");
}

namespace xse {

int ExecuteParts(xse_engine* engine, const xse_bag_request* whole, int32_t n,
                 const PartSet& parts, cudaStream_t stream, int32_t flags,
                 xse_status* status) {
  TraceRange trace("xse.execute_parts");
  if (engine == nullptr || status == nullptr || parts.reqs == nullptr ||
      parts.owner == nullptr) {
    return SetError(XSE_INVALID_ARGUMENT, "null argument");
  }
  return ExecuteBatch(engine, whole, n, stream, flags, status, nullptr,
                      &parts);
}

}  // namespace xse
