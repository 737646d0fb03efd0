// Internal declarations shared by the CUDA sources of the engine.
#ifndef XSE_INTERNAL_H_
#define XSE_INTERNAL_H_

#include <cuda_runtime.h>
#include <nvtx3/nvToolsExt.h>
#include <stdint.h>

namespace xse {

// An NVTX range over one entry point's host work (the reference traces
// each graph node's execution with a tsl TraceMe span,
// data/processor/cc/core/graph/graph_executor.cc:62,111). Header-only NVTX:
// without a profiler attached a push or pop is one indirect call.
class TraceRange {
 public:
  explicit TraceRange(const char* name) { nvtxRangePushA(name); }
  ~TraceRange() { nvtxRangePop(); }
  TraceRange(const TraceRange&) = delete;
  TraceRange& operator=(const TraceRange&) = delete;
};

// Descriptors passed by value in one launch (kernel parameter space holds up
// to 32 KB on sm_70+ with CUDA 12.1+).
constexpr int kMaxDescsPerLaunch = 64;
// Sample blocks of one descriptor written to separate places (a sharded
// step's destinations); see BagDesc::block_bags.
constexpr int kMaxOutBlocks = 8;

// One pooling request as the kernels see it.
struct BagDesc {
  const void* rows;           // table rows of the shard window, row-major
  const float2* scale_bias;   // int8 rows: (scale, bias) per window row
  const void* ids;            // int32 or int64
  const void* offsets;        // int32 or int64, num_bags + 1 entries
  const float* weights;       // nullptr when unweighted
  float* out;                 // bag b at out + b * out_stride
  int64_t out_stride;
  // > 0: blocked output instead -- bag b at PoolParams::block_base[j] +
  // out_offset + (b - j * block_bags) * out_stride, j = b / block_bags.
  int64_t block_bags;
  int64_t out_offset;
  int64_t vocab;              // global rows; valid ids are [0, vocab)
  int64_t row_begin;          // shard window [row_begin, row_end)
  int64_t row_end;
  int64_t num_ids;
  int64_t num_weights;
  int64_t num_bags;
  int64_t task_begin;         // first pooling task of this descriptor
  int64_t work_begin;         // first validation work item of this descriptor
  int32_t dim;
  int32_t slot;               // request index into the status block
  int8_t combine;             // 1 sum, 2 mean, 3 sqrtn
  int8_t ids64;
  int8_t offs64;
  int8_t vec_out;             // output rows 16-byte aligned
};

// Per-request error record written by the device.
enum : unsigned int {
  kErrBadOffsets = 1u,         // first offset negative or offsets decreasing
  kErrLastExceedsIds = 2u,     // final offset > number of ids
  kErrLastExceedsWeights = 4u, // final offset > number of weights
  kErrBadId = 8u,              // some id outside [0, vocab)
  kErrDeviceWait = 128u,       // a bounded device-side wait ran out
};

struct DevRequestStatus {
  unsigned int flags;
  unsigned int reserved;
  // Bitwise complement of the smallest failing id position (0 = none), so
  // that a zeroed block starts empty and atomicMax keeps the minimum.
  unsigned long long inv_min_bad_index;
};

struct DevStatus {
  unsigned int group_error;  // nonzero once any request failed validation
  unsigned int work_counter;  // samples handed out by the fused interaction
  unsigned int reserved[2];
  DevRequestStatus req[1];   // capacity set at allocation
};

inline size_t DevStatusBytes(int capacity) {
  return sizeof(DevStatus) + sizeof(DevRequestStatus) * (capacity - 1);
}

struct PoolParams {
  int32_t n;
  int32_t fused_checks;   // 1: record errors here; 0: a validation pass ran
  int64_t total_tasks;
  int32_t bags_per_task;  // consecutive bags one lane group pools per task
  int32_t reserved;
  DevStatus* status;
  // Vector kernels: descriptors sorted by weighting mode; cumulative task
  // and block ends of modes 0, 1, 2 (set by the launcher).
  int64_t mode_tasks[3];
  int32_t mode_blocks[3];
  // Host-side kernel choice for 16-byte-vector rows (kernels ignore it):
  // kPoolAuto, kPoolStreaming (PoolVecKernel) or kPoolStaged
  // (PoolStagedKernel).
  int32_t kernel_choice;
  float* block_base[kMaxOutBlocks];  // blocked outputs (BagDesc::block_bags)
  BagDesc d[kMaxDescsPerLaunch];
};

enum : int32_t { kPoolAuto = 0, kPoolStreaming = 1, kPoolStaged = 2 };

// Row layout class of a launch: G lanes per row, V 16-byte vectors per lane.
// V == 0 selects the element-wise kernel (dims that are not whole vectors).
// A launch serves every weighting mode of its layout.
struct Layout {
  int dtype;
  int g;
  int v;
  bool exact;  // rows are exactly g*v vectors: no per-lane bounds checks
  int wmode;   // unused by the launcher (kept for callers that group by it)
  // Lanes own v contiguous vectors (one 256-bit load each) instead of
  // vectors gl + k g: int8 rows of 256, 512 or 1024 bytes, 32-byte aligned.
  bool wide = false;
};

// Weighting mode of a request (kernels are compiled per mode).
inline int WeightModeOf(const BagDesc& d) {
  if (d.weights == nullptr) return 0;
  return d.combine == 1 ? 1 : 2;
}

Layout ChooseLayout(int dtype, int dim, const void* rows);
// Pooling tasks (work units of one lane group) for num_bags bags.
int64_t TasksFor(const Layout& layout, int64_t num_bags);
// Validation work items of one request.
int64_t ValidationWork(int64_t num_bags, int64_t num_ids);

cudaError_t LaunchValidate(const PoolParams& p, int64_t total_work,
                           cudaStream_t stream);
// True when both PoolVecKernel and PoolStagedKernel serve a launch of this
// layout and size and neither is the fixed choice: the launch is larger than
// one wave of the staged kernel (small launches always take it).
bool PoolKernelTunable(const Layout& layout, int64_t total_tasks);

cudaError_t LaunchPool(const Layout& layout, const PoolParams& p,
                       cudaStream_t stream, int* launches);
cudaError_t LaunchInterleaveScaleBias(const float* scale, const float* bias,
                                      float2* out, int64_t n,
                                      cudaStream_t stream);
// Sets the calling thread's message returned by xse_last_error().
void SetLastErrorMessage(const char* message);

// Table loading (csrc/xse_capi.cu): the host upload's staging chunk (<= 0:
// one pageable copy) and fill threads; the fill reads file `fd` at
// file_offset when fd >= 0, else copies from src.
constexpr int64_t kDefaultUploadChunk = 32ll << 20;
constexpr int kDefaultUploadThreads = 8;
cudaError_t UploadFromHost(void* dst, const void* src, size_t bytes,
                           int64_t chunk, int threads, int fd,
                           int64_t file_offset);

// Fused pooling + dot interaction (PoolInteractKernel, csrc/xse_bag.cu).
struct InteractArgs {
  const float* dense;        // [batch] rows of dim floats, 16-byte aligned
  int64_t dense_stride;      // floats, multiple of 4
  float* out;                // [batch] rows of out_stride floats
  // Non-null: out receives each value's TF32 part (round to nearest, ties
  // away) and out_lo the exact remainder, the split operands of the next
  // layer's three-pass TF32 GEMM (rows of out_stride floats).
  float* out_lo;
  int64_t out_stride;        // >= dim + (T+1)T/2
  int64_t batch;
  int32_t samples_per_tile;  // shared-memory sample slots (set by the launcher)
  int32_t row_stride;        // set by the launcher
};

// Launches the fused kernel over p's descriptors (request order; each is one
// table with a.batch bags). Returns cudaErrorNotSupported, launching
// nothing, when no fused kernel serves this layout, weighting or size.
cudaError_t LaunchPoolInteract(const Layout& layout, const PoolParams& p,
                               const InteractArgs& a, cudaStream_t stream);

cudaError_t LaunchDotInteraction(const float* dense, int64_t dense_stride,
                                 const float* pooled, int64_t pooled_stride,
                                 int64_t batch, int num_tables, int dim,
                                 float* out, int64_t out_stride,
                                 cudaStream_t stream);

// Legacy per-feature path (csrc/xse_legacy.cu): FeatureBatchCsrInput checks,
// pooling in the table's type, sequence gather.
enum : unsigned int {
  kLegacySizeMismatch = 16u,  // first offset != 0 or last != number of ids
  kLegacyNotSorted = 32u,     // offsets decrease
  kLegacyWeights = 64u,       // weights neither empty nor one per id
  kLegacyBadId = kErrBadId,   // an id read by the feature is out of range
};
enum : int8_t { kLegacyPoolF32 = 0, kLegacyPoolBf16 = 1, kLegacySequence = 2 };

struct LegacyDesc {
  const void* rows;      // [vocab, dim] fp32 or bf16
  const void* ids;
  const void* offsets;   // num_bags + 1 entries
  const float* weights;  // nullptr or num_weights entries
  void* out;             // [num_bags, dim] or [num_bags, max_seq, dim]
  int64_t vocab;
  int64_t num_ids;
  int64_t num_weights;
  int64_t num_bags;
  int64_t task_begin;
  int64_t max_seq;       // sequence features only
  int32_t dim;
  int32_t slot;
  int8_t combine;
  int8_t ids64;
  int8_t offs64;
  int8_t dtype;          // 0 fp32, 1 bf16
  int8_t kind;           // kLegacy*
};

struct LegacyParams {
  int32_t n;
  int32_t reserved;
  int64_t total_tasks;   // samples of all requests
  DevStatus* status;
  LegacyDesc d[kMaxDescsPerLaunch];
};

cudaError_t LaunchLegacy(const LegacyParams& p, cudaStream_t stream);

// Dense ids -> CSR on the device (csrc/xse_dense_csr.cu): scratch bytes for
// `batch` rows, the conversion (rp: batch + 1 int32, ids: capacity
// batch * max(seq, 1) int64), and dense_lookup row pointers b * valency.
size_t DenseCsrScratchBytes(int64_t batch);
cudaError_t LaunchDenseToCsr(const void* dense, int is64, int64_t batch,
                             int64_t seq, int64_t pad, int32_t* rp,
                             int64_t* ids, void* scratch,
                             size_t scratch_bytes, cudaStream_t stream);
cudaError_t LaunchRowPointers(int32_t* rp, int64_t batch, int64_t valency,
                              cudaStream_t stream);

// Sets what xse_last_launch_count() reports for this thread.
void SetLastLaunchCount(int32_t launches);

}  // namespace xse

#include "../../include/xse_emb.h"

namespace xse {

// Slices of whole requests: part j pools a contiguous range of the bags of
// whole request owner[j] (its offsets point into the whole request's row
// pointers; ids, weights and feature are the whole request's) into its own
// output. The sharded executor sends each destination's sample block to a
// different place this way.
struct PartSet {
  const xse_bag_request* reqs;
  const int32_t* owner;
  int32_t n;
  bool validate;  // run the validation pass over the whole requests
  // Blocked form (blocks > 0; the parts must describe the same outputs and
  // are then only used for the isolation check): every whole request k is
  // cut into `blocks` sample blocks of block_bags, block j written at
  // block_base[j] + block_offset[k] with rows block_stride floats apart.
  // The kernels then see one descriptor per whole request.
  int32_t blocks = 0;
  int64_t block_bags = 0;
  float* const* block_base = nullptr;
  const int64_t* block_offset = nullptr;
  int64_t block_stride = 0;
};

// ExecuteBatch over `whole` (the status block's requests: its errors name
// whole requests) that pools `parts` instead of the whole requests. The
// validation pass, when it runs, reads every whole request once, not once
// per part.
int ExecuteParts(xse_engine* engine, const xse_bag_request* whole, int32_t n,
                 const PartSet& parts, cudaStream_t stream, int32_t flags,
                 xse_status* status);

}  // namespace xse

#endif  // XSE_INTERNAL_H_
