// CPU oracle for the embedding-bag / DLRM interaction path.
//
// TEST INFRASTRUCTURE ONLY: the results the CUDA path is tested against and
// the timed CPU baseline. It restates, in plain C++17, the reference CPU engine of
// openxla/xla-serving. Each function cites the reference file:line it follows.
// Compiled with -ffp-contract=off so that every multiply and add rounds
// separately, in the order the reference's scalar semantics give.
//
// Parity pins: the reference needs Bazel, abseil and Eigen to build, none of
// which exist here, so this restatement is pinned against the reference's own
// known-answer tests (tests/golden/known_answers.json) and against the
// reference's numpy lookup run on seeded inputs (tests/golden/make_golden.py).

#include "xse_oracle.h"

#include <sched.h>

#include <algorithm>
#include <atomic>
#include <cinttypes>
#include <cmath>
#include <condition_variable>
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <functional>
#include <limits>
#include <memory>
#include <mutex>
#include <string>
#include <thread>
#include <vector>

namespace {

int Fail(int code, char* err, int32_t errlen, const char* fmt, ...) {
  if (err != nullptr && errlen > 0) {
    va_list args;
    va_start(args, fmt);
    vsnprintf(err, static_cast<size_t>(errlen), fmt, args);
    va_end(args);
  }
  return code;
}

// ---------------------------------------------------------------------------
// bf16 helpers (round to nearest even, as Eigen::bfloat16's float ctor does).
float Bf16ToFloat(uint16_t bits) {
  uint32_t word = static_cast<uint32_t>(bits) << 16;
  float value;
  std::memcpy(&value, &word, sizeof(value));
  return value;
}

uint16_t FloatToBf16(float value) {
  uint32_t word;
  std::memcpy(&word, &value, sizeof(word));
  if ((word & 0x7fffffffu) > 0x7f800000u) {  // NaN: keep it a quiet NaN.
    return static_cast<uint16_t>((word >> 16) | 0x0040u);
  }
  const uint32_t rounding = 0x7fffu + ((word >> 16) & 1u);
  return static_cast<uint16_t>((word + rounding) >> 16);
}

// ---------------------------------------------------------------------------
// One request, resolved.
struct Request {
  const oracle_request* raw;
  int64_t num_bags;
};

int64_t Offset(const oracle_request& r, int64_t i) {
  return r.offsets_i64 ? static_cast<const int64_t*>(r.offsets)[i]
                       : static_cast<const int32_t*>(r.offsets)[i];
}

// Row element c of row `id`, widened to fp32 (dequantized for int8 rows).
float RowValue(const oracle_request& r, int64_t id, int64_t c) {
  const int64_t at = id * r.dim + c;
  switch (r.dtype) {
    case ORACLE_F32:
      return static_cast<const float*>(r.table)[at];
    case ORACLE_BF16:
      return Bf16ToFloat(static_cast<const uint16_t*>(r.table)[at]);
    default: {
      // Row-wise dequantisation to an fp32 row, then the fp32 bag: the
      // product float(q) * scale and the sum with bias are rounded
      // separately (the file is compiled with -ffp-contract=off, so neither
      // expression becomes an fma).
      const float q = static_cast<float>(static_cast<const int8_t*>(r.table)[at]);
      const float scaled = q * r.scale[id];
      return scaled + r.bias[id];
    }
  }
}

// ValidateEmbeddingBagInput (embedding_bag.cc:89-144), widened to int64
// offsets and to the bf16 / int8-rowwise table types.
int ValidateRequest(const oracle_request& r, char* err, int32_t errlen) {
  if (r.table == nullptr) {
    return Fail(ORACLE_INVALID_ARGUMENT, err, errlen,
                "Embedding table must be non-null.");
  }
  const bool known_dtype = r.dtype == ORACLE_F32 || r.dtype == ORACLE_BF16 ||
                           r.dtype == ORACLE_I8_ROWWISE;
  const bool known_mode = r.combine == ORACLE_SUM || r.combine == ORACLE_MEAN ||
                          r.combine == ORACLE_SQRTN;
  if (!known_dtype || !known_mode || r.dim <= 0 || r.vocab < 0 ||
      (r.dtype == ORACLE_I8_ROWWISE &&
       (r.scale == nullptr || r.bias == nullptr))) {
    return Fail(ORACLE_FAILED_PRECONDITION, err, errlen,
                "Grouped execution requires a non-sequence FP32 SUM, MEAN, or "
                "SQRT_N table without a custom combiner.");
  }
  if (r.num_offsets < 2 || r.offsets == nullptr) {
    return Fail(ORACLE_INVALID_ARGUMENT, err, errlen,
                "Row pointers must contain at least two elements.");
  }
  bool sorted = Offset(r, 0) >= 0;
  for (int64_t i = 1; sorted && i < r.num_offsets; ++i) {
    sorted = Offset(r, i - 1) <= Offset(r, i);
  }
  if (!sorted) {
    return Fail(ORACLE_INVALID_ARGUMENT, err, errlen,
                "Row pointers must be non-negative and monotonic.");
  }
  const int64_t first = Offset(r, 0);
  const int64_t last = Offset(r, r.num_offsets - 1);
  if (last > r.num_ids) {
    return Fail(ORACLE_INVALID_ARGUMENT, err, errlen,
                "Final row pointer exceeds embedding IDs size.");
  }
  if (r.num_weights > 0 && last > r.num_weights) {
    return Fail(ORACLE_INVALID_ARGUMENT, err, errlen,
                "Final row pointer exceeds weights size.");
  }
  if (first != last && r.ids == nullptr) {
    return Fail(ORACLE_INVALID_ARGUMENT, err, errlen,
                "Embedding-ID storage must be non-null.");
  }
  if (r.num_weights > 0 && r.weights == nullptr) {
    return Fail(ORACLE_INVALID_ARGUMENT, err, errlen,
                "Weight storage must be non-null.");
  }
  for (int64_t index = first; index < last; ++index) {
    const int64_t id = r.ids[index];
    if (id < 0 || id >= r.vocab) {
      return Fail(ORACLE_INVALID_ARGUMENT, err, errlen,
                  "Embedding ID (%" PRId64 ") at index %" PRId64
                  " is out of bounds [0, %" PRId64 ").",
                  id, index, r.vocab);
    }
  }
  return ORACLE_OK;
}

// BagScale (embedding_bag.cc:146-167): applied as a multiply; weighted
// denominators are summed in CSR order.
float BagScale(const oracle_request& r, int64_t bag) {
  const int64_t begin = Offset(r, bag);
  const int64_t end = Offset(r, bag + 1);
  const int64_t size = end - begin;
  if (size == 0 || r.combine == ORACLE_SUM) return 1.0f;
  if (r.num_weights == 0) {
    return r.combine == ORACLE_MEAN
               ? 1.0f / static_cast<float>(size)
               : 1.0f / std::sqrt(static_cast<float>(size));
  }
  float denominator = 0.0f;
  for (int64_t p = begin; p < end; ++p) {
    const float w = r.weights[p];
    denominator += r.combine == ORACLE_MEAN ? w : w * w;
  }
  return r.combine == ORACLE_MEAN ? 1.0f / denominator
                                  : 1.0f / std::sqrt(denominator);
}

// ReducePortable (embedding_bag.cc:170-194): zero the bag, add rows (or
// weight*row) in CSR order element by element, then scale non-empty bags of
// non-SUM tables.
void ReduceBags(const oracle_request& r, int64_t bag_begin, int64_t bag_end) {
  const int64_t dim = r.dim;
  for (int64_t bag = bag_begin; bag < bag_end; ++bag) {
    float* out = r.out + bag * dim;
    std::fill(out, out + dim, 0.0f);
    const int64_t begin = Offset(r, bag);
    const int64_t end = Offset(r, bag + 1);
    for (int64_t p = begin; p < end; ++p) {
      const int64_t id = r.ids[p];
      if (r.num_weights == 0) {
        for (int64_t c = 0; c < dim; ++c) out[c] += RowValue(r, id, c);
      } else {
        const float w = r.weights[p];
        for (int64_t c = 0; c < dim; ++c) {
          const float term = w * RowValue(r, id, c);
          out[c] += term;
        }
      }
    }
    if (begin != end && r.combine != ORACLE_SUM) {
      const float scale = BagScale(r, bag);
      for (int64_t c = 0; c < dim; ++c) out[c] *= scale;
    }
  }
}

// ValidateOutputIsolation (embedding_bag.cc:268-351): no output overlaps
// another output or any input range.
struct Range {
  uintptr_t begin, end;
  int32_t request;
  const char* kind;
};

bool Overlaps(const Range& a, const Range& b) {
  return a.begin < b.end && b.begin < a.end;
}

void AddRange(const void* data, int64_t elements, size_t elem_size,
              int32_t request, const char* kind, std::vector<Range>* ranges) {
  if (elements <= 0 || data == nullptr) return;
  const uintptr_t begin = reinterpret_cast<uintptr_t>(data);
  ranges->push_back(
      {begin, begin + static_cast<uintptr_t>(elements) * elem_size, request,
       kind});
}

size_t TableElementBytes(int32_t dtype) {
  return dtype == ORACLE_F32 ? 4 : dtype == ORACLE_BF16 ? 2 : 1;
}

int CheckIsolation(const std::vector<Request>& reqs, char* err,
                   int32_t errlen) {
  std::vector<Range> outputs, inputs;
  for (size_t i = 0; i < reqs.size(); ++i) {
    const oracle_request& r = *reqs[i].raw;
    const int32_t idx = static_cast<int32_t>(i);
    AddRange(r.out, reqs[i].num_bags * r.dim, sizeof(float), idx, "output",
             &outputs);
    AddRange(r.ids, r.num_ids, sizeof(int64_t), idx, "embedding-ID", &inputs);
    AddRange(r.offsets, r.num_offsets, r.offsets_i64 ? 8 : 4, idx,
             "row-pointer", &inputs);
    AddRange(r.weights, r.num_weights, sizeof(float), idx, "weight", &inputs);
    AddRange(r.table, r.vocab * r.dim, TableElementBytes(r.dtype), idx,
             "embedding-table", &inputs);
  }
  std::sort(outputs.begin(), outputs.end(),
            [](const Range& a, const Range& b) { return a.begin < b.begin; });
  for (size_t i = 1; i < outputs.size(); ++i) {
    if (Overlaps(outputs[i - 1], outputs[i])) {
      return Fail(ORACLE_INVALID_ARGUMENT, err, errlen,
                  "FP32 embedding-bag request outputs %d and %d overlap.",
                  outputs[i - 1].request, outputs[i].request);
    }
  }
  for (const Range& o : outputs) {
    for (const Range& in : inputs) {
      if (Overlaps(o, in)) {
        return Fail(ORACLE_INVALID_ARGUMENT, err, errlen,
                    "FP32 embedding-bag request %d output overlaps request %d "
                    "%s storage.",
                    o.request, in.request, in.kind);
      }
    }
  }
  return ORACLE_OK;
}

// BuildTasks (embedding_bag.cc:359-413): cost (ids + bags) * dim; target
// total / (threads * 4); a task never splits a bag.
struct Task {
  int32_t request;
  int64_t bag_begin, bag_end;
};

uint64_t TaskCost(const oracle_request& r, int64_t b0, int64_t b1) {
  const uint64_t ids = static_cast<uint64_t>(Offset(r, b1) - Offset(r, b0));
  return (ids + static_cast<uint64_t>(b1 - b0)) * static_cast<uint64_t>(r.dim);
}

std::vector<Task> BuildTasks(const std::vector<Request>& reqs, int threads) {
  constexpr uint64_t kTasksPerThread = 4;
  uint64_t total = 0;
  for (const Request& q : reqs) total += TaskCost(*q.raw, 0, q.num_bags);
  const uint64_t count = static_cast<uint64_t>(threads) * kTasksPerThread;
  const uint64_t target =
      std::max<uint64_t>(1, total / count + (total % count != 0));
  std::vector<Task> tasks;
  for (size_t i = 0; i < reqs.size(); ++i) {
    const oracle_request& r = *reqs[i].raw;
    int64_t tile_begin = 0;
    uint64_t tile_cost = 0;
    for (int64_t bag = 0; bag < reqs[i].num_bags; ++bag) {
      if (bag != tile_begin && tile_cost >= target) {
        tasks.push_back({static_cast<int32_t>(i), tile_begin, bag});
        tile_begin = bag;
        tile_cost = 0;
      }
      tile_cost += TaskCost(r, bag, bag + 1);
    }
    tasks.push_back({static_cast<int32_t>(i), tile_begin, reqs[i].num_bags});
  }
  return tasks;
}

// A persistent worker pool (the reference keeps an Eigen::ThreadPool alive
// in the engine, cpu_embedding_engine.cc:51-56), so that timing does not pay
// thread creation per call.
class WorkerPool {
 public:
  explicit WorkerPool(int n) {
    for (int i = 0; i < n; ++i) workers_.emplace_back([this] { Loop(); });
  }
  ~WorkerPool() {
    {
      std::lock_guard<std::mutex> lock(mu_);
      stop_ = true;
    }
    cv_.notify_all();
    for (auto& t : workers_) t.join();
  }
  int size() const { return static_cast<int>(workers_.size()); }

  // Runs job(worker) on `count` workers and waits for all of them.
  void Run(int count, const std::function<void()>& job) {
    std::unique_lock<std::mutex> lock(mu_);
    job_ = &job;
    pending_ = count;
    to_start_ = count;
    ++generation_;
    cv_.notify_all();
    done_cv_.wait(lock, [this] { return pending_ == 0; });
    job_ = nullptr;
  }

 private:
  void Loop() {
    uint64_t seen = 0;
    for (;;) {
      const std::function<void()>* job;
      {
        std::unique_lock<std::mutex> lock(mu_);
        cv_.wait(lock, [&] {
          return stop_ || (generation_ != seen && to_start_ > 0);
        });
        if (stop_) return;
        seen = generation_;
        --to_start_;
        job = job_;
      }
      (*job)();
      {
        std::lock_guard<std::mutex> lock(mu_);
        if (--pending_ == 0) done_cv_.notify_all();
      }
    }
  }

  std::mutex mu_;
  std::condition_variable cv_, done_cv_;
  std::vector<std::thread> workers_;
  const std::function<void()>* job_ = nullptr;
  int pending_ = 0, to_start_ = 0;
  uint64_t generation_ = 0;
  bool stop_ = false;
};

WorkerPool* PoolFor(int threads) {
  static std::mutex mu;
  static std::unique_ptr<WorkerPool> pool;
  std::lock_guard<std::mutex> lock(mu);
  if (!pool || pool->size() != threads) {
    pool.reset();
    pool = std::make_unique<WorkerPool>(threads);
  }
  return pool.get();
}

// ---------------------------------------------------------------------------
// Counter-based generator (independent restatement of the device generator).
uint64_t Mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

uint64_t Bits64(uint64_t seed, uint64_t stream, uint64_t index) {
  const uint64_t key =
      Mix64(seed * 0x9E3779B97F4A7C15ull + stream * 0xD1B54A32D192ED03ull);
  return Mix64(key + index * 0x9E3779B97F4A7C15ull);
}

// 24-bit uniform in [0,1), exactly representable as fp32.
float Uniform24(uint64_t seed, uint64_t stream, uint64_t index) {
  const uint32_t u = static_cast<uint32_t>(Bits64(seed, stream, index) >> 40);
  return static_cast<float>(u) * (1.0f / 16777216.0f);
}

// Generator streams: one block of 16 per table.
enum Stream : uint64_t {
  kValues = 0,
  kLengths = 1,
  kIds = 2,
  kWeights = 3,
  kScale = 5,
  kBias = 6,
};

uint64_t StreamOf(uint64_t table, Stream s) { return table * 16 + s; }

float TableValue(uint64_t seed, uint64_t table, int64_t row, int64_t dim,
                 int64_t c) {
  const float u = Uniform24(seed, StreamOf(table, kValues),
                            static_cast<uint64_t>(row * dim + c));
  const float scaled = 0.1f * u;
  return -0.05f + scaled;
}

// Rejection-inversion sampling of a bounded Zipf distribution
// (W. Hormann and G. Derflinger, "Rejection-inversion to generate variates
// from monotone discrete distributions", ACM TOMACS 6(3), 1996), written from
// the paper's construction: H is an antiderivative of h(x) = x^-alpha, a
// continuous variate is drawn by inverting H, rounded, and accepted when it
// falls under the hat.
struct Zipf {
  double alpha, n;
  double h_lo, h_hi, squeeze;

  static double Log1pOverX(double x) {
    return std::fabs(x) > 1e-8 ? std::log1p(x) / x
                               : 1.0 - x * (0.5 - x * (1.0 / 3.0 - 0.25 * x));
  }
  static double Expm1OverX(double x) {
    return std::fabs(x) > 1e-8
               ? std::expm1(x) / x
               : 1.0 + x * 0.5 * (1.0 + x * (1.0 / 3.0) * (1.0 + 0.25 * x));
  }
  double Hat(double x) const { return std::exp(-alpha * std::log(x)); }
  double H(double x) const {
    const double lx = std::log(x);
    return Expm1OverX((1.0 - alpha) * lx) * lx;
  }
  double HInverse(double y) const {
    double t = y * (1.0 - alpha);
    if (t < -1.0) t = -1.0;
    return std::exp(Log1pOverX(t) * y);
  }
  Zipf(int64_t count, double a) : alpha(a), n(static_cast<double>(count)) {
    h_lo = H(1.5) - 1.0;
    h_hi = H(n + 0.5);
    squeeze = 2.0 - HInverse(H(2.5) - Hat(2.0));
  }
  // u in [0,1): one draw; returns 0 when the draw is rejected.
  int64_t Try(double u) const {
    const double y = h_hi + u * (h_lo - h_hi);
    const double x = HInverse(y);
    double k = std::floor(x + 0.5);
    if (k < 1.0) k = 1.0;
    if (k > n) k = n;
    if (k - x <= squeeze || y >= H(k + 0.5) - Hat(k)) {
      return static_cast<int64_t>(k);
    }
    return 0;
  }
};

}  // namespace

extern "C" {

int oracle_embedding_bag_batch(const oracle_request* reqs, int32_t n,
                               int32_t num_threads, int64_t inline_threshold,
                               char* err, int32_t errlen) {
  // ExecuteEmbeddingBagBatch (embedding_bag.cc:477-535).
  if (n <= 0 || reqs == nullptr) {
    return Fail(ORACLE_INVALID_ARGUMENT, err, errlen,
                "Embedding-bag batch requires at least one request.");
  }
  std::vector<Request> prepared;
  prepared.reserve(static_cast<size_t>(n));
  for (int32_t i = 0; i < n; ++i) {
    char inner[512] = {0};
    const int code = ValidateRequest(reqs[i], inner, sizeof(inner));
    if (code != ORACLE_OK) {
      // RequestError (embedding_bag.cc:229-233).
      return Fail(code, err, errlen, "FP32 embedding-bag request %d: %s", i,
                  inner);
    }
    if (reqs[i].out == nullptr) {
      return Fail(ORACLE_INVALID_ARGUMENT, err, errlen,
                  "FP32 embedding-bag request %d requires an output allocator.",
                  i);
    }
    prepared.push_back({&reqs[i], reqs[i].num_offsets - 1});
  }
  const int code = CheckIsolation(prepared, err, errlen);
  if (code != ORACLE_OK) return code;

  int64_t total_output = 0;
  for (const Request& q : prepared) total_output += q.num_bags * q.raw->dim;
  if (num_threads <= 1 || total_output <= inline_threshold) {
    for (const Request& q : prepared) ReduceBags(*q.raw, 0, q.num_bags);
    return ORACLE_OK;
  }
  const std::vector<Task> tasks = BuildTasks(prepared, num_threads);
  const int workers = static_cast<int>(
      std::min<size_t>(static_cast<size_t>(num_threads), tasks.size()));
  std::atomic<size_t> next{0};
  std::function<void()> job = [&] {
    for (;;) {
      const size_t t = next.fetch_add(1, std::memory_order_relaxed);
      if (t >= tasks.size()) break;
      ReduceBags(*prepared[tasks[t].request].raw, tasks[t].bag_begin,
                 tasks[t].bag_end);
    }
  };
  PoolFor(num_threads)->Run(workers, job);
  return ORACLE_OK;
}

int oracle_assemble_bf16_accumulate(const uint16_t* table, int64_t vocab,
                                    int64_t dim, int32_t combine,
                                    const int64_t* ids, int64_t num_ids,
                                    const int32_t* row_pointers,
                                    int64_t num_row_pointers,
                                    const float* weights, uint16_t* out,
                                    char* err, int32_t errlen) {
  // AssembleCombinedEmbeddings<Eigen::bfloat16> (compute_activations.cc:
  // 36-154). Every bf16 operation computes in fp32 and rounds to bf16.
  (void)num_ids;
  const int64_t samples = num_row_pointers - 1;
  std::vector<uint16_t> acc(static_cast<size_t>(dim));
  for (int64_t s = 0; s < samples; ++s) {
    const int64_t start = row_pointers[s];
    const int64_t size = row_pointers[s + 1] - row_pointers[s];
    uint16_t* act = out + s * dim;
    if (size == 0) {
      std::fill(act, act + dim, static_cast<uint16_t>(0));
      continue;
    }
    for (int64_t k = 0; k < size; ++k) {
      const int64_t id = ids[start + k];
      if (id < 0 || id >= vocab) {
        return Fail(ORACLE_INVALID_ARGUMENT, err, errlen,
                    "Embedding ID (%" PRId64 ") at index %" PRId64
                    " is out of bounds [0, %" PRId64 ") for table table.",
                    id, start + k, vocab);
      }
    }
    std::fill(acc.begin(), acc.end(), static_cast<uint16_t>(0));
    float scale = 1.0f;
    if (weights == nullptr) {
      for (int64_t k = 0; k < size; ++k) {
        const uint16_t* row = table + ids[start + k] * dim;
        for (int64_t c = 0; c < dim; ++c) {
          acc[c] = FloatToBf16(Bf16ToFloat(acc[c]) + Bf16ToFloat(row[c]));
        }
      }
      if (combine == ORACLE_MEAN) scale = 1.0f / static_cast<float>(size);
      if (combine == ORACLE_SQRTN) {
        scale = 1.0f / std::sqrt(static_cast<float>(size));
      }
    } else {
      float sum_weights = 0.0f;
      for (int64_t k = 0; k < size; ++k) {
        const uint16_t* row = table + ids[start + k] * dim;
        const float w = weights[start + k];
        const float wb = Bf16ToFloat(FloatToBf16(w));
        for (int64_t c = 0; c < dim; ++c) {
          const uint16_t prod = FloatToBf16(wb * Bf16ToFloat(row[c]));
          acc[c] = FloatToBf16(Bf16ToFloat(acc[c]) + Bf16ToFloat(prod));
        }
        if (combine == ORACLE_MEAN) sum_weights += w;
        if (combine == ORACLE_SQRTN) sum_weights += w * w;
      }
      if (combine == ORACLE_MEAN) scale = 1.0f / sum_weights;
      if (combine == ORACLE_SQRTN) scale = 1.0f / std::sqrt(sum_weights);
    }
    if (scale != 1.0f) {
      const float sb = Bf16ToFloat(FloatToBf16(scale));
      for (int64_t c = 0; c < dim; ++c) {
        acc[c] = FloatToBf16(Bf16ToFloat(acc[c]) * sb);
      }
    }
    std::copy(acc.begin(), acc.end(), act);
  }
  return ORACLE_OK;
}

int oracle_sequence_gather(const void* table, int32_t dtype, int64_t vocab,
                           int64_t dim, const int64_t* ids,
                           const int32_t* row_pointers,
                           int64_t num_row_pointers, int64_t max_seq,
                           void* out, char* err, int32_t errlen) {
  // AssembleSequenceEmbeddings (compute_activations.cc:187-224).
  const size_t elem = dtype == ORACLE_F32 ? 4 : 2;
  const int64_t samples = num_row_pointers - 1;
  for (int64_t s = 0; s < samples; ++s) {
    const int64_t start = row_pointers[s];
    const int64_t len = row_pointers[s + 1] - start;
    const int64_t n = std::min(len, max_seq);
    for (int64_t k = 0; k < n; ++k) {
      const int64_t id = ids[start + k];
      if (id < 0 || id >= vocab) {
        return Fail(ORACLE_INVALID_ARGUMENT, err, errlen,
                    "Embedding ID (%" PRId64 ") at index %" PRId64
                    " is out of bounds [0, %" PRId64 ") for table table.",
                    id, k, vocab);
      }
    }
    char* dst = static_cast<char*>(out) + s * max_seq * dim * elem;
    for (int64_t k = 0; k < n; ++k) {
      std::memcpy(dst + k * dim * elem,
                  static_cast<const char*>(table) + ids[start + k] * dim * elem,
                  dim * elem);
    }
  }
  return ORACLE_OK;
}

int oracle_dense_to_csr(const void* dense, int32_t dense_i64, int64_t batch,
                        int64_t seq, int64_t pad_value, int64_t* ids,
                        int32_t* row_pointers, int64_t* num_ids, char* err,
                        int32_t errlen) {
  // DenseCpuEmbeddingLookupTransform::operator() (dense_cpu_embedding_lookup_
  // transform.cc:186-225): keep non-pad ids; an all-pad row keeps one pad id;
  // int32 row pointers with an overflow check.
  const int64_t elements = batch * seq;
  if (elements > std::numeric_limits<int32_t>::max()) {
    return Fail(ORACLE_INVALID_ARGUMENT, err, errlen,
                "dense_ids exceeds INT32_MAX elements: %" PRId64, elements);
  }
  int64_t count = 0;
  row_pointers[0] = 0;
  for (int64_t b = 0; b < batch; ++b) {
    int32_t active = 0;
    for (int64_t j = 0; j < seq; ++j) {
      const int64_t id =
          dense_i64 ? static_cast<const int64_t*>(dense)[b * seq + j]
                    : static_cast<const int32_t*>(dense)[b * seq + j];
      if (id != pad_value) {
        ids[count++] = id;
        ++active;
      }
    }
    if (active == 0) {
      ids[count++] = pad_value;
      active = 1;
    }
    const int64_t next = static_cast<int64_t>(row_pointers[b]) + active;
    if (next > std::numeric_limits<int32_t>::max()) {
      return Fail(ORACLE_INVALID_ARGUMENT, err, errlen,
                  "Row pointer offset overflowed int32_t.");
    }
    row_pointers[b + 1] = static_cast<int32_t>(next);
  }
  *num_ids = count;
  return ORACLE_OK;
}

int oracle_dense_lookup_row_pointers(int64_t batch, int64_t valency,
                                     int32_t* row_pointers, char* err,
                                     int32_t errlen) {
  // cpu_embedding_lookup_transform.cc:297-316.
  if (batch < 0 || valency < 0) {
    return Fail(ORACLE_INVALID_ARGUMENT, err, errlen,
                "Dense embedding IDs dimensions must be non-negative.");
  }
  if (batch >= std::numeric_limits<int32_t>::max()) {
    return Fail(ORACLE_INVALID_ARGUMENT, err, errlen,
                "Batch size exceeds INT32_MAX bounds.");
  }
  if (batch > 0 && valency > std::numeric_limits<int32_t>::max() / batch) {
    return Fail(ORACLE_INVALID_ARGUMENT, err, errlen,
                "Batch volume (batch_size * valency) exceeds INT32_MAX "
                "bounds.");
  }
  if (row_pointers != nullptr) {
    for (int64_t b = 0; b <= batch; ++b) {
      row_pointers[b] = static_cast<int32_t>(b * valency);
    }
  }
  return ORACLE_OK;
}

void oracle_dot_interaction(const float* dense, const float* pooled,
                            int64_t batch, int32_t num_tables, int32_t dim,
                            float* out) {
  // DLRM dot interaction: no counterpart in the reference (its DLRM uses
  // DCN-v2, examples/dlrm/model_jce.py:141-164). Row 0 of Z is the dense
  // vector; pairs (i, j) with i < j are emitted in row-major order after the
  // dense vector.
  const int32_t rows = num_tables + 1;
  const int64_t pairs = static_cast<int64_t>(rows) * (rows - 1) / 2;
  const int64_t width = dim + pairs;
  for (int64_t b = 0; b < batch; ++b) {
    auto row = [&](int32_t i) -> const float* {
      return i == 0 ? dense + b * dim
                    : pooled + (b * num_tables + (i - 1)) * dim;
    };
    float* o = out + b * width;
    for (int32_t c = 0; c < dim; ++c) o[c] = dense[b * dim + c];
    int64_t k = dim;
    for (int32_t i = 0; i < rows; ++i) {
      for (int32_t j = i + 1; j < rows; ++j) {
        const float* zi = row(i);
        const float* zj = row(j);
        double acc = 0.0;
        for (int32_t c = 0; c < dim; ++c) {
          acc += static_cast<double>(zi[c]) * static_cast<double>(zj[c]);
        }
        o[k++] = static_cast<float>(acc);
      }
    }
  }
}

double oracle_uniform(uint64_t seed, uint64_t stream, uint64_t index) {
  return static_cast<double>(Uniform24(seed, stream, index));
}

void oracle_synth_rows_f32(uint64_t seed, uint64_t table, int64_t row0,
                           int64_t nrows, int64_t dim, float* out) {
  for (int64_t r = 0; r < nrows; ++r) {
    for (int64_t c = 0; c < dim; ++c) {
      out[r * dim + c] = TableValue(seed, table, row0 + r, dim, c);
    }
  }
}

void oracle_synth_rows_bf16(uint64_t seed, uint64_t table, int64_t row0,
                            int64_t nrows, int64_t dim, uint16_t* out) {
  for (int64_t r = 0; r < nrows; ++r) {
    for (int64_t c = 0; c < dim; ++c) {
      out[r * dim + c] = FloatToBf16(TableValue(seed, table, row0 + r, dim, c));
    }
  }
}

void oracle_synth_rows_i8(uint64_t seed, uint64_t table, int64_t row0,
                          int64_t nrows, int64_t dim, int8_t* q, float* scale,
                          float* bias) {
  for (int64_t r = 0; r < nrows; ++r) {
    const int64_t row = row0 + r;
    for (int64_t c = 0; c < dim; ++c) {
      const uint64_t bits = Bits64(seed, StreamOf(table, kValues),
                                   static_cast<uint64_t>(row * dim + c));
      const uint64_t u24 = bits >> 40;
      q[r * dim + c] = static_cast<int8_t>(-127 + static_cast<int>((u24 * 255) >> 24));
    }
    const float us = Uniform24(seed, StreamOf(table, kScale), row);
    const float ub = Uniform24(seed, StreamOf(table, kBias), row);
    const float s_scaled = 9e-3f * us;
    const float b_scaled = 0.2f * ub;
    scale[r] = 1e-3f + s_scaled;
    bias[r] = -0.1f + b_scaled;
  }
}

void oracle_synth_rows_at(int32_t dtype, uint64_t seed, uint64_t table,
                          const int64_t* rows, int64_t n, int64_t dim,
                          void* out, float* scale, float* bias) {
  // Row by row through the contiguous generators: the value of (row, c)
  // depends only on the row index, so any subset of rows can be rebuilt.
  for (int64_t i = 0; i < n; ++i) {
    if (dtype == ORACLE_F32) {
      oracle_synth_rows_f32(seed, table, rows[i], 1, dim,
                            static_cast<float*>(out) + i * dim);
    } else if (dtype == ORACLE_BF16) {
      oracle_synth_rows_bf16(seed, table, rows[i], 1, dim,
                             static_cast<uint16_t*>(out) + i * dim);
    } else {
      oracle_synth_rows_i8(seed, table, rows[i], 1, dim,
                           static_cast<int8_t*>(out) + i * dim, scale + i,
                           bias + i);
    }
  }
}

void oracle_synth_lengths(int64_t n, int32_t lo, int32_t hi, uint64_t seed,
                          uint64_t table, int64_t* out) {
  // u24 scaled to the span by a 24-bit fixed-point multiply.
  const uint64_t span = static_cast<uint64_t>(hi - lo + 1);
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t u24 =
        Bits64(seed, StreamOf(table, kLengths), static_cast<uint64_t>(i)) >> 40;
    out[i] = lo + static_cast<int64_t>((u24 * span) >> 24);
  }
}

void oracle_synth_weights(int64_t n, uint64_t seed, uint64_t table,
                          int64_t index0, float* out) {
  for (int64_t i = 0; i < n; ++i) {
    out[i] = Uniform24(seed, StreamOf(table, kWeights),
                       static_cast<uint64_t>(index0 + i));
  }
}

void oracle_synth_ids(int64_t n, int64_t vocab, double alpha,
                      uint64_t perm_mul, uint64_t perm_add, uint64_t seed,
                      uint64_t table, int64_t index0, int64_t* out) {
  const uint64_t uv = static_cast<uint64_t>(vocab);
  const uint64_t stream = StreamOf(table, kIds);
  for (int64_t i = 0; i < n; ++i) {
    const uint64_t index = static_cast<uint64_t>(index0 + i);
    if (alpha <= 0.0) {
      // Uniform: the high 64 bits of bits * vocab.
      const unsigned __int128 wide =
          static_cast<unsigned __int128>(Bits64(seed, stream, index)) * uv;
      out[i] = static_cast<int64_t>(wide >> 64);
    } else {
      const int64_t k = oracle_zipf_rank(seed, stream, index, vocab, alpha);
      out[i] = static_cast<int64_t>(
          (static_cast<uint64_t>(k - 1) * perm_mul + perm_add) % uv);
    }
  }
}

int64_t oracle_zipf_rank(uint64_t seed, uint64_t stream, uint64_t index,
                         int64_t n, double alpha) {
  const Zipf zipf(n, alpha);
  int64_t k = 0;
  for (uint64_t attempt = 0; attempt < 64 && k == 0; ++attempt) {
    const uint64_t bits = Bits64(seed, stream, index * 64 + attempt);
    const double u = static_cast<double>(bits >> 11) * (1.0 / 9007199254740992.0);
    k = zipf.Try(u);
  }
  return k == 0 ? 1 : k;
}

int32_t oracle_host_cores(void) {
  cpu_set_t set;
  CPU_ZERO(&set);
  if (sched_getaffinity(0, sizeof(set), &set) == 0) return CPU_COUNT(&set);
  const unsigned n = std::thread::hardware_concurrency();
  return n == 0 ? 1 : static_cast<int32_t>(n);
}

}  // extern "C"
