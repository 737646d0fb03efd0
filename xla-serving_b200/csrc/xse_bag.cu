// Pooled embedding-bag kernels for sm_100a.
//
// Replaces the reference's CPU hot loop ReducePortable / BagScale
// (data/cpu_embedding/cc/embedding_bag.cc:146-194) and its group validation
// (embedding_bag.cc:89-144).
//
// Design: a group of G lanes owns one bag (G = 4..32, so a warp pools 32/G
// bags at once). Each lane owns V 16-byte column vectors of a row, so a row
// gather is G*V independent 16-byte loads. The ids (and weights) of a bag are
// loaded G at a time, one per lane, and broadcast through the group with
// shuffles; U rows are loaded before any of them is added, which keeps U*V
// loads in flight per lane while the adds still run in CSR order.
//
// Random 256-byte row gathers reach the HBM copy bandwidth only with about 32
// resident warps per SM and several rows in flight per lane, and the pooling
// work around each gathered vector must stay small enough that instruction
// issue does not become the limit. So the per-row state held across a batch
// is only the loaded data, the kernels are bounded to four 256-thread blocks
// per SM, layouts whose rows are exactly G*V vectors drop per-lane bounds
// checks at compile time, and the fp32 arithmetic runs on packed pairs
// (sm_100 add/mul.rn.f32x2: two independently rounded IEEE operations in one
// instruction). That is PoolVecKernel. PoolStagedKernel instead copies a
// whole round of up to 32 rows of a bag into shared memory with cp.async,
// for launches too small to fill the GPU and for id streams whose rows
// mostly hit the caches; the engine times both on large launches and keeps
// the faster (the results are bit-identical).
//
// Every element is accumulated in fp32 in exactly the reference's order
// (out = 0; out += row or out += w*row, one separately rounded multiply and
// add), so fp32 results are bit-identical to the reference semantics; mean
// and sqrt-n scales are applied as one multiply by a correctly rounded
// reciprocal.
//
// HBM traffic per id: one row (dim * elem bytes) + the id (4/8 B) + the weight
// if any; per bag: one offset and the fp32 output row.

#include <cuda_runtime.h>

#include <utility>
#include <stdint.h>

#include "xse_internal.h"

namespace xse {
namespace {

constexpr int kThreads = 256;
using u64 = unsigned long long;

template <int DT>
struct ElemsPerVec;
template <>
struct ElemsPerVec<0> {
  static constexpr int value = 4;  // fp32
};
template <>
struct ElemsPerVec<1> {
  static constexpr int value = 8;  // bf16
};
template <>
struct ElemsPerVec<2> {
  static constexpr int value = 16;  // int8
};

// Tuning: rows in flight per lane for fp32/bf16 rows (int8 rows, whose
// dequantized vectors need four times the registers, use half), and the
// resident 256-thread blocks per SM the register budget is sized for.
#ifndef XSE_POOL_ROWS
#define XSE_POOL_ROWS 4
#endif
#ifndef XSE_POOL_MIN_BLOCKS
#define XSE_POOL_MIN_BLOCKS 3
#endif
// Row prefetch. Chunk prefetch (XSE_POOL_CHUNK_PREFETCH, fp32/bf16 rows in
// the throughput pooling kernel): when a chunk's ids are staged, each lane
// prefetches the whole row of its id into L1 (the kernel's row loads
// allocate in L1), so all of a chunk's rows are requested at once and the
// batches that gather them find them on chip or already in flight. Batch
// prefetch (XSE_POOL_PREFETCH, everywhere else): the rows of a chunk's next
// batch go to L2 while the current batch is in flight. Measured on one B200
// against batch prefetch: Zipf(1.1) table-wise slice 1.22-1.30 -> 1.04-1.07
// ms per step, multi-table 70.6 -> 69.7 us; int8 rows (3.06 -> 3.51 ms) and
// the deep small-launch variant were slower with it, so they keep batch
// prefetch; both kinds at once was slower than either.
#ifndef XSE_POOL_PREFETCH
#define XSE_POOL_PREFETCH 1
#endif
#ifndef XSE_POOL_CHUNK_PREFETCH
#define XSE_POOL_CHUNK_PREFETCH 1
#endif
// Chunk prefetch of int8 rows: 0 off, 1 into L2, 2 into L1.
#ifndef XSE_POOL_I8_CHUNK_PREFETCH
#define XSE_POOL_I8_CHUNK_PREFETCH 0
#endif
// Next-batch L2 prefetch of int8 rows: off. With the wide int8 lanes it cost
// more issue slots than it saved latency (int8 row-wise workload, pooling
// per step: 2.60 ms with it, 2.40 ms without; the chunk prefetch into L2:
// 3.37 ms).
#ifndef XSE_POOL_I8_PREFETCH
#define XSE_POOL_I8_PREFETCH 0
#endif

#ifndef XSE_POOL_I8_ROWS
#define XSE_POOL_I8_ROWS 2
#endif
#ifndef XSE_POOL_I8_MIN_BLOCKS
#define XSE_POOL_I8_MIN_BLOCKS 3
#endif

// 1: int8 rows of 256, 512 or 1024 bytes take the wide layout (32-byte
// lanes); 0: 16-byte lanes like every other row type.
#ifndef XSE_POOL_I8_WIDE
#define XSE_POOL_I8_WIDE 1
#endif
#ifndef XSE_POOL_BF16_WIDE
#define XSE_POOL_BF16_WIDE 1
#endif

// PoolStagedKernel: 0 never, 1 for launches small enough for one wave of
// it, 2 for every launch whose rows it serves.
#ifndef XSE_POOL_STAGED
#define XSE_POOL_STAGED 1
#endif

// 1: validation and pooling kernels use programmatic dependent launch.
#ifndef XSE_PDL
#define XSE_PDL 1
#endif

// Wide int8 layouts (32-byte lanes): rows in flight per lane and resident
// 256-thread blocks per SM. Measured on the int8 row-wise workload (26
// tables 10M x 256, Zipf(1.05)), pooling per step: 2 rows at 3 blocks/SM
// 2.86 ms (80 registers, some spilled), 2 at 2 blocks 2.91 ms, 3 at 3
// blocks 3.44 ms; 16-byte lanes 3.07 ms.
#ifndef XSE_POOL_I8W_ROWS
#define XSE_POOL_I8W_ROWS 2
#endif
#ifndef XSE_POOL_I8W_MIN_BLOCKS
#define XSE_POOL_I8W_MIN_BLOCKS 3
#endif
// Wide bf16 layouts: rows in flight per lane and resident blocks per SM.
// Measured on the multi-table workload (8 bf16 tables 500k x 128, uniform
// ids), pooling per step: 4 rows at 2 blocks/SM 65.2 us (128 registers, no
// spills); 2 at 3 blocks 75.1 us, 3 at 3 blocks 77.0 us (both spill);
// 16-byte lanes 70.3 us.
#ifndef XSE_POOL_BF16W_ROWS
#define XSE_POOL_BF16W_ROWS 4
#endif
#ifndef XSE_POOL_BF16W_MIN_BLOCKS
#define XSE_POOL_BF16W_MIN_BLOCKS 2
#endif

// Rows gathered per batch (in flight per lane, times V vectors each; a wide
// lane's V vectors are one load).
template <int DT, int V, bool WIDE = false>
struct RowsInFlight {
  static constexpr int base = DT == 2 ? XSE_POOL_I8_ROWS : XSE_POOL_ROWS;
  static constexpr int value =
      WIDE ? (DT == 2 ? XSE_POOL_I8W_ROWS : XSE_POOL_BF16W_ROWS)
           : (V >= base ? 1 : base / V);
};

// Resident blocks per SM each variant's register budget is sized for.
template <int DT, int V, bool WIDE = false>
struct MinBlocks {
  static constexpr int value =
      WIDE ? (DT == 2 ? XSE_POOL_I8W_MIN_BLOCKS : XSE_POOL_BF16W_MIN_BLOCKS)
      : ElemsPerVec<DT>::value * V <= 16 &&
              RowsInFlight<DT, V>::value * V <= 8
          ? (DT == 2 ? XSE_POOL_I8_MIN_BLOCKS : XSE_POOL_MIN_BLOCKS)
          : 2;
};

// ---- packed fp32 pairs (low word = first element) ------------------------
__device__ __forceinline__ u64 PackBits(uint32_t lo, uint32_t hi) {
  u64 r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "r"(lo), "r"(hi));
  return r;
}
__device__ __forceinline__ u64 PackF(float lo, float hi) {
  return PackBits(__float_as_uint(lo), __float_as_uint(hi));
}
__device__ __forceinline__ float LoF(u64 v) {
  return __uint_as_float(static_cast<uint32_t>(v));
}
__device__ __forceinline__ float HiF(u64 v) {
  return __uint_as_float(static_cast<uint32_t>(v >> 32));
}
__device__ __forceinline__ u64 Add2(u64 a, u64 b) {
  u64 r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ u64 Mul2(u64 a, u64 b) {
  u64 r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
__device__ __forceinline__ u64 Fma2(u64 a, u64 b, u64 c) {
  u64 r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}

__device__ __forceinline__ int64_t LoadIndex(const void* base, int is64,
                                             int64_t i) {
  return is64 ? __ldg(static_cast<const long long*>(base) + i)
              : static_cast<int64_t>(__ldg(static_cast<const int*>(base) + i));
}

// Read-only 16-byte row load. L1 selects its L1 policy: false does not
// allocate in L1 (reuse of rows comes from L2 only), true caches in L1 (hot
// rows of skewed id streams are then served by the SM that reads them).
// XSE_POOL_L1 is the policy of the pooling kernel (which uses no shared
// memory, so L1 has the SM's whole data cache): caching took the Zipf(1.1)
// table-wise slice from 1.226 to 1.137 ms per step and the uniform
// multi-table step from 71.6 to 70.7 us. XSE_INTERACT_L1 is the fused
// interaction kernel's: its shared-memory slots leave L1 small, and caching
// cost it 1.5 %.
#ifndef XSE_POOL_L1
#define XSE_POOL_L1 1
#endif
#ifndef XSE_INTERACT_L1
#define XSE_INTERACT_L1 0
#endif
// Chunk prefetch in the fused interaction kernel: 0 off (batch prefetch),
// 1 into L2, 2 into L1.
#ifndef XSE_INTERACT_CHUNK_PREFETCH
#define XSE_INTERACT_CHUNK_PREFETCH 0
#endif
template <bool L1>
__device__ __forceinline__ uint4 LoadRowVec(const uint4* p) {
  uint4 r;
  if constexpr (L1) {
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
  } else {
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
  }
  return r;
}

// Read-only 32-byte row load (sm_100 256-bit ld.global) into two vectors:
// the part of a row one lane owns in the wide int8 layouts (p 32-byte
// aligned).
template <bool L1>
__device__ __forceinline__ void LoadRowVec32(const uint4* p, uint4* a,
                                             uint4* b) {
  if constexpr (L1) {
    asm volatile(
        "ld.global.nc.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
        : "=r"(a->x), "=r"(a->y), "=r"(a->z), "=r"(a->w), "=r"(b->x),
          "=r"(b->y), "=r"(b->z), "=r"(b->w)
        : "l"(p));
  } else {
    asm volatile(
        "ld.global.nc.L1::no_allocate.v8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, "
        "[%8];"
        : "=r"(a->x), "=r"(a->y), "=r"(a->z), "=r"(a->w), "=r"(b->x),
          "=r"(b->y), "=r"(b->z), "=r"(b->w)
        : "l"(p));
  }
}

// Vector v of a lane's part of a row, relative to the lane's first vector:
// lanes own vectors gl + v G, or (WIDE) V contiguous vectors gl V + v.
template <int G, bool WIDE>
__device__ __forceinline__ int LaneVec(int v) {
  return WIDE ? v : v * G;
}

// Loads a lane's V vectors of one row (`src` = the row's first vector for
// this lane); vectors past a non-exact row's end read as zeros.
template <int G, int V, bool EXACT, bool WIDE, bool L1>
__device__ __forceinline__ void LoadLaneRow(const uint4* src, int gl,
                                            int row_vecs, uint4 (&raw)[V]) {
  if constexpr (WIDE) {
    static_assert(V == 2 && EXACT, "wide layouts are exact 32-byte lanes");
    LoadRowVec32<L1>(src, &raw[0], &raw[1]);
  } else {
#pragma unroll
    for (int v = 0; v < V; ++v) {
      if (EXACT || gl + v * G < row_vecs) {
        raw[v] = LoadRowVec<L1>(src + v * G);
      } else {
        raw[v] = make_uint4(0, 0, 0, 0);
      }
    }
  }
}

__device__ __forceinline__ void PrefetchRowVec(const uint4* p) {
  asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
}

// Prefetches the 128-byte lines of one row of `bytes` bytes at `row` (every
// line holds a byte of the row, so every address is mapped).
template <bool L1>
__device__ __forceinline__ void PrefetchRow(const void* row, int bytes) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(row);
  const int lines = static_cast<int>(((a & 127u) + bytes + 127) >> 7);
  const char* line = reinterpret_cast<const char*>(a & ~uintptr_t{127});
  for (int k = 0; k < lines; ++k) {
    if constexpr (L1) {
      asm volatile("prefetch.global.L1 [%0];" ::"l"(line + 128 * k));
    } else {
      asm volatile("prefetch.global.L2 [%0];" ::"l"(line + 128 * k));
    }
  }
}

// Products are scalar mul.rn.f32, which PTX never contracts into an FMA; a
// packed mul.rn.f32x2 feeding a packed add can be fused by the assembler,
// which would round once instead of twice and break bit parity.
__device__ __forceinline__ u64 MulPair(float a, float lo, float hi) {
  return PackF(__fmul_rn(a, lo), __fmul_rn(a, hi));
}

// One 16-byte row vector as fp32 pairs; int8 rows give their quantized
// values float(q) (exact), which AddRow scales. A byte b becomes float(b)
// exactly by placing b + 128 (b ^ 0x80) in the low mantissa bits of 2^23
// (one byte permute) and subtracting 2^23 + 128.
template <int DT>
__device__ __forceinline__ void UnpackPairs(
    const uint4& r, u64 (&x)[ElemsPerVec<DT>::value / 2]) {
  const uint32_t w[4] = {r.x, r.y, r.z, r.w};
  if constexpr (DT == 0) {
    x[0] = PackBits(w[0], w[1]);
    x[1] = PackBits(w[2], w[3]);
  } else if constexpr (DT == 1) {
#pragma unroll
    for (int k = 0; k < 4; ++k) x[k] = PackBits(w[k] << 16, w[k] & 0xffff0000u);
  } else {
    constexpr uint32_t kTwo23 = 0x4B000000u;         // 2^23
    const u64 neg_magic = PackF(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const uint32_t t = w[k] ^ 0x80808080u;
      const u64 lo = PackBits(__byte_perm(t, kTwo23, 0x7440),
                              __byte_perm(t, kTwo23, 0x7441));
      const u64 hi = PackBits(__byte_perm(t, kTwo23, 0x7442),
                              __byte_perm(t, kTwo23, 0x7443));
      x[2 * k] = Add2(lo, neg_magic);
      x[2 * k + 1] = Add2(hi, neg_magic);
    }
  }
}

// acc += row (or acc += w*row), element by element in fp32.
//
// Int8 row-wise rows: w * (q * scale + bias) summed over a bag's rows is
// accumulated as acc = fma(q, w * scale, acc) per element plus, once per
// row, bsum += w * bias (the bias is the same for every element of a row);
// FinishBag adds bsum to every element. That is one packed fma per pair of
// elements instead of a dequantizing fma and an add. The result equals
// dequantize-then-pool up to fp32 rounding: each step rounds once, so the
// difference stays within a few units of 2^-24 times
// sum |w| (|q| scale + |bias|) per element.
template <int DT, int V>
__device__ __forceinline__ void AddRow(
    u64 (&acc)[V][ElemsPerVec<DT>::value / 2], const uint4 (&raw)[V],
    float scale, float bias, bool weighted, float w, float* bsum) {
  constexpr int PPV = ElemsPerVec<DT>::value / 2;
  if constexpr (DT == 2) {
    const float ws = weighted ? __fmul_rn(w, scale) : scale;
    const u64 s2 = PackF(ws, ws);
#pragma unroll
    for (int v = 0; v < V; ++v) {
      u64 x[PPV];
      UnpackPairs<DT>(raw[v], x);
#pragma unroll
      for (int k = 0; k < PPV; ++k) acc[v][k] = Fma2(x[k], s2, acc[v][k]);
    }
    *bsum = weighted ? __fmaf_rn(w, bias, *bsum) : __fadd_rn(*bsum, bias);
  } else {
    (void)scale;
    (void)bias;
    (void)bsum;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      u64 x[PPV];
      UnpackPairs<DT>(raw[v], x);
#pragma unroll
      for (int k = 0; k < PPV; ++k) {
        acc[v][k] = weighted
                        ? Add2(acc[v][k], MulPair(w, LoF(x[k]), HiF(x[k])))
                        : Add2(acc[v][k], x[k]);
      }
    }
  }
}

__device__ __forceinline__ void RecordError(DevStatus* st, int slot,
                                            unsigned int flag) {
  atomicOr(&st->req[slot].flags, flag);
  atomicOr(&st->group_error, 1u);
}

__device__ __forceinline__ void RecordBadId(DevStatus* st, int slot,
                                            int64_t index) {
  atomicMax(&st->req[slot].inv_min_bad_index,
            ~static_cast<unsigned long long>(index));
  RecordError(st, slot, kErrBadId);
}

// Bag scale (embedding_bag.cc:146-167), computed once per bag.
__device__ __forceinline__ float BagScale(int combine, bool weighted,
                                          int64_t n, float wsum) {
  const float denom = weighted ? wsum : __ll2float_rn(n);
  return combine == 2 ? __fdiv_rn(1.0f, denom)
                      : __fdiv_rn(1.0f, __fsqrt_rn(denom));
}

// Output row of bag `bag` of descriptor d (blocked outputs: see
// BagDesc::block_bags; block indexes fit 32 bits).
__device__ __forceinline__ float* BagOut(const PoolParams& p, const BagDesc& d,
                                         int64_t bag) {
  if (d.block_bags <= 0) return d.out + bag * d.out_stride;
  const uint32_t j = static_cast<uint32_t>(bag) /
                     static_cast<uint32_t>(d.block_bags);
  return p.block_base[j] + d.out_offset +
         (bag - static_cast<int64_t>(j) * d.block_bags) * d.out_stride;
}

// Locates the descriptor of `task`; descriptors are ordered by task_begin and
// every group walks its tasks in increasing order, so the search only moves
// forward.
__device__ __forceinline__ int AdvanceDesc(const PoolParams& p, int t,
                                           int64_t task) {
  while (t + 1 < p.n && task >= p.d[t + 1].task_begin) ++t;
  return t;
}

// Same for validation work items, ordered by work_begin.
__device__ __forceinline__ int AdvanceWork(const PoolParams& p, int t,
                                           int64_t w) {
  while (t + 1 < p.n && w >= p.d[t + 1].work_begin) ++t;
  return t;
}

// Offsets of bag `bag`, checked. Returns false when the bag must be skipped.
__device__ __forceinline__ bool BagRange(const PoolParams& p,
                                         const BagDesc& d, int64_t bag,
                                         int64_t* begin, int64_t* end) {
  *begin = LoadIndex(d.offsets, d.offs64, bag);
  *end = LoadIndex(d.offsets, d.offs64, bag + 1);
  const bool weights_short = d.weights != nullptr && *end > d.num_weights;
  const bool bad = *begin < 0 || *end < *begin || *end > d.num_ids ||
                   weights_short;
  if (bad && p.fused_checks) {
    unsigned int f = 0;
    if (*begin < 0 || *end < *begin) f |= kErrBadOffsets;
    if (*end > d.num_ids) f |= kErrLastExceedsIds;
    if (weights_short) f |= kErrLastExceedsWeights;
    RecordError(p.status, d.slot, f);
  }
  return !bad;
}

// Stages one chunk of ids: lane gl takes position pos (if below end) and
// returns its row within the shard window, or -1 when the id contributes
// nothing (invalid -- an error -- or another shard's row).
__device__ __forceinline__ int StageRow(const PoolParams& p, const BagDesc& d,
                                        int64_t id, int64_t pos, bool live) {
  if (!live) return -1;
  if (id < 0 || id >= d.vocab) {
    if (p.fused_checks) RecordBadId(p.status, d.slot, pos);
    return -1;
  }
  if (id < d.row_begin || id >= d.row_end) return -1;
  return static_cast<int>(id - d.row_begin);
}

// How a bag's weights enter the pool; fixed per bag so the row loops carry no
// weighting branches. Only weighted means and sqrt-n need the weight sum.
// Each kernel is compiled for one mode: a kernel that branches between modes
// per bag keeps the union of their registers live and spills.
enum WeightMode : int {
  kUnweighted = 0,
  kWeightedSum = 1,   // weighted sum: no weight total needed
  kWeightedNorm = 2,  // weighted mean (sum of w) or sqrt-n (sum of w*w)
};

template <int WM>
__device__ __forceinline__ void AddWeight(float* wsum, float w, int combine) {
  if constexpr (WM == kWeightedNorm) {
    *wsum = __fadd_rn(*wsum, combine == 3 ? __fmul_rn(w, w) : w);
  }
}

// Adds raw row u to acc (int8 rows with their scale/bias, see AddRow).
template <int DT, int V, int WM>
__device__ __forceinline__ void AddGathered(
    u64 (&acc)[V][ElemsPerVec<DT>::value / 2], const uint4 (&raw)[V],
    float2 sb, float w, float* bsum) {
  AddRow<DT, V>(acc, raw, sb.x, sb.y, WM != kUnweighted, w, bsum);
}

// Full batch of U rows of a chunk whose ids all contribute: no per-row
// checks. Lanes past the end of a non-exact row add zeros to accumulator
// lanes that are never stored. PF: prefetch the chunk's next batch of rows
// into L2 while this one is in flight.
template <int DT, int G, int V, bool EXACT, bool WIDE, int WM, int U,
          bool L1, bool PF, typename Hook>
__device__ __forceinline__ void FullBatch(
    const BagDesc& d, const uint4* rows, int row_vecs, int gl, unsigned gmask,
    int my_row, float my_w, int j0, int cnt,
    u64 (&acc)[V][ElemsPerVec<DT>::value / 2], float* wsum, float* bsum,
    Hook&& hook) {
  const int stride = EXACT ? G * V : row_vecs;
  uint4 raw[U][V];
  float2 sb[U];
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int r = __shfl_sync(gmask, my_row, j0 + u, G);
    if constexpr (DT == 2) sb[u] = __ldg(d.scale_bias + r);
    LoadLaneRow<G, V, EXACT, WIDE, L1>(
        rows + static_cast<int64_t>(r) * stride, gl, row_vecs, raw[u]);
  }
  if constexpr (PF) {
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = j0 + U + u;
      if (j < cnt) {
        const int r = __shfl_sync(gmask, my_row, j, G);
        const uint4* src = rows + static_cast<int64_t>(r) * stride;
        if constexpr (WIDE) {
          PrefetchRowVec(src);  // the lane's 32 bytes share one line
        } else {
#pragma unroll
          for (int v = 0; v < V; ++v) {
            if (EXACT || gl + v * G < row_vecs) PrefetchRowVec(src + v * G);
          }
        }
      }
    }
  } else {
    (void)cnt;
  }
  hook();  // runs while this batch's rows are in flight
#pragma unroll
  for (int u = 0; u < U; ++u) {
    float w = 1.0f;
    if constexpr (WM != kUnweighted) {
      w = __shfl_sync(gmask, my_w, j0 + u, G);
      AddWeight<WM>(wsum, w, d.combine);
    }
    AddGathered<DT, V, WM>(acc, raw[u], DT == 2 ? sb[u] : make_float2(0, 0),
                           w, bsum);
  }
}

// General batch: up to U rows (positions j0..j0+n-1 of the chunk), skipping
// ids that contribute nothing.
template <int DT, int G, int V, bool EXACT, bool WIDE, int WM, int U,
          bool L1, typename Hook>
__device__ __forceinline__ void GatherBatch(
    const BagDesc& d, const uint4* rows, int row_vecs, int gl, unsigned gmask,
    int my_row, float my_w, int j0, int n,
    u64 (&acc)[V][ElemsPerVec<DT>::value / 2], float* wsum, float* bsum,
    Hook&& hook) {
  const int stride = EXACT ? G * V : row_vecs;
  uint4 raw[U][V];
  float2 sb[U];
  unsigned int present = 0;
#pragma unroll
  for (int u = 0; u < U; ++u) {
    const int j = u < n ? j0 + u : j0;
    const int r = __shfl_sync(gmask, my_row, j, G);
    const bool use = u < n && r >= 0;
    present |= use ? (1u << u) : 0u;
    if constexpr (DT == 2) {
      sb[u] = use ? __ldg(d.scale_bias + r) : make_float2(0.0f, 0.0f);
    }
    if (use) {
      LoadLaneRow<G, V, EXACT, WIDE, L1>(
          rows + static_cast<int64_t>(r) * stride, gl, row_vecs, raw[u]);
    }
  }
  hook();  // runs while this batch's rows are in flight
#pragma unroll
  for (int u = 0; u < U; ++u) {
    if (u < n) {
      float w = 1.0f;
      if constexpr (WM != kUnweighted) {
        w = __shfl_sync(gmask, my_w, j0 + u, G);
        AddWeight<WM>(wsum, w, d.combine);
      }
      if (present & (1u << u)) {
        AddGathered<DT, V, WM>(acc, raw[u],
                               DT == 2 ? sb[u] : make_float2(0, 0), w, bsum);
      }
    }
  }
}

// A chunk in which some ids contribute nothing (another row-wise shard's
// rows, or invalid ids under fused checks): the contributing positions are
// found with one ballot and gathered U at a time, so a chunk costs one
// memory round trip per U contributing rows rather than per U positions
// (on a row-wise shard of W ranks only about 1/W of the ids are local).
// Adds stay in CSR order; weight sums still count every position.
template <int DT, int G, int V, bool EXACT, bool WIDE, int WM, int U, bool L1,
          typename Hook>
__device__ __forceinline__ void SparseChunk(
    const BagDesc& d, const uint4* rows, int row_vecs, int gl, unsigned gmask,
    int my_row, float my_w, int cnt,
    u64 (&acc)[V][ElemsPerVec<DT>::value / 2], float* wsum, float* bsum,
    Hook&& hook) {
  const int stride = EXACT ? G * V : row_vecs;
  const int lane = threadIdx.x & 31;
  unsigned m = __ballot_sync(gmask, gl < cnt && my_row >= 0);
  m = (m >> (lane - gl)) & (G == 32 ? 0xffffffffu : ((1u << G) - 1u));
  if constexpr (WM == kWeightedNorm) {
    for (int j = 0; j < cnt; ++j) {
      AddWeight<WM>(wsum, __shfl_sync(gmask, my_w, j, G), d.combine);
    }
  }
  bool hooked = false;
  while (m != 0) {
    uint4 raw[U][V];
    float2 sb[U];
    int pos[U];
    int n = 0;
#pragma unroll
    for (int u = 0; u < U; ++u) {
      pos[u] = m != 0 ? __ffs(m) - 1 : 0;
      if (m != 0) {
        m &= m - 1;
        n = u + 1;
      }
      const int r = __shfl_sync(gmask, my_row, pos[u], G);
      if (u < n) {
        if constexpr (DT == 2) sb[u] = __ldg(d.scale_bias + r);
        LoadLaneRow<G, V, EXACT, WIDE, L1>(
            rows + static_cast<int64_t>(r) * stride, gl, row_vecs, raw[u]);
      }
    }
    if (!hooked) {
      hook();  // runs while the first batch's rows are in flight
      hooked = true;
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      float w = 1.0f;
      if constexpr (WM != kUnweighted) {
        w = __shfl_sync(gmask, my_w, pos[u], G);
      }
      if (u < n) {
        AddGathered<DT, V, WM>(acc, raw[u],
                               DT == 2 ? sb[u] : make_float2(0, 0), w, bsum);
      }
    }
  }
  if (!hooked) hook();
}

// 1: lanes holding 8 or 16 output floats store them with 32-byte stores.
#ifndef XSE_POOL_WIDE_STORES
#define XSE_POOL_WIDE_STORES 1
#endif

// One 32-byte store (sm_100 256-bit st.global): a lane's 8 output floats in
// one instruction, so a lane group writes its whole output row at once
// instead of two half-filled passes over the row's 32-byte sectors (which
// matters most when the row is a peer's memory, reached over NVLink).
__device__ __forceinline__ void Store32B(float* p, u64 a, u64 b, u64 c,
                                         u64 d) {
  asm volatile("st.global.v4.b64 [%0], {%1,%2,%3,%4};" ::"l"(p), "l"(a),
               "l"(b), "l"(c), "l"(d)
               : "memory");
}

// Scales (mean / sqrt-n) and stores one finished bag, then clears the
// accumulator for the next one. GLOBAL_OUT: `out` is global memory (this
// device's or a peer's), so 32-byte st.global stores may be used; the fused
// interaction kernel passes rows in shared memory and sets it false (a
// st.global to a shared address faults).
template <int DT, int G, int V, bool EXACT, bool GLOBAL_OUT, bool WIDE = false>
__device__ __forceinline__ void FinishBag(
    const BagDesc& d, float* out, bool vec_out, int64_t n, bool weighted,
    u64 (&acc)[V][ElemsPerVec<DT>::value / 2], float* wsum, int gl,
    int row_vecs, float* bsum) {
  constexpr int PPV = ElemsPerVec<DT>::value / 2;
  if constexpr (DT == 2) {
    // The rows' biases (see AddRow), once per element.
    const u64 b2 = PackF(*bsum, *bsum);
#pragma unroll
    for (int v = 0; v < V; ++v)
#pragma unroll
      for (int k = 0; k < PPV; ++k) acc[v][k] = Add2(acc[v][k], b2);
    *bsum = 0.0f;
  } else {
    (void)bsum;
  }
  if (n > 0 && d.combine != 1) {
    const float s = BagScale(d.combine, weighted, n, *wsum);
    const u64 s2 = PackF(s, s);
#pragma unroll
    for (int v = 0; v < V; ++v)
#pragma unroll
      for (int k = 0; k < PPV; ++k) acc[v][k] = Mul2(acc[v][k], s2);
  }
  // Lanes holding 8 or 16 floats store 32-byte pieces when the row is
  // 32-byte aligned (each lane's part then is too).
  const bool wide = XSE_POOL_WIDE_STORES && GLOBAL_OUT && PPV % 4 == 0 &&
                    vec_out && (reinterpret_cast<uintptr_t>(out) & 31u) == 0;
  if constexpr (WIDE && DT == 1 && PPV == 4 && V == 2) {
    // A wide bf16 lane holds two consecutive 32-byte pieces of the row
    // (pieces 2gl and 2gl+1); storing them as they lie leaves every store
    // instruction of the group half-filling each 64-byte span, which costs
    // twice the transactions when the row is a peer's memory over NVLink.
    // So the pieces are exchanged first: store s writes piece s*G + gl,
    // taken from lane (s*G + gl) / 2, and each store covers G contiguous
    // pieces.
    if (wide) {
      const int lane = threadIdx.x & 31;
      const unsigned gmask =
          G == 32 ? 0xffffffffu : (((1u << G) - 1u) << (lane - gl));
#pragma unroll
      for (int st = 0; st < 2; ++st) {
        const int q = st * G + gl;
        const int src = q >> 1;
        const bool odd = (q & 1) != 0;
        u64 piece[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const uint32_t a_lo = __shfl_sync(
              gmask, static_cast<uint32_t>(acc[0][e]), src, G);
          const uint32_t a_hi = __shfl_sync(
              gmask, static_cast<uint32_t>(acc[0][e] >> 32), src, G);
          const uint32_t b_lo = __shfl_sync(
              gmask, static_cast<uint32_t>(acc[1][e]), src, G);
          const uint32_t b_hi = __shfl_sync(
              gmask, static_cast<uint32_t>(acc[1][e] >> 32), src, G);
          piece[e] = odd ? PackBits(b_lo, b_hi) : PackBits(a_lo, a_hi);
        }
        Store32B(out + q * 8, piece[0], piece[1], piece[2], piece[3]);
      }
#pragma unroll
      for (int v = 0; v < V; ++v)
#pragma unroll
        for (int e = 0; e < PPV; ++e) acc[v][e] = 0;
      *wsum = 0.0f;
      return;
    }
  }
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int k = WIDE ? gl * V + v : gl + v * G;
    if (EXACT || k < row_vecs) {
      float* o = out + k * (2 * PPV);
      if (wide) {
#pragma unroll
        for (int e = 0; e + 3 < PPV; e += 4) {
          Store32B(o + 2 * e, acc[v][e], acc[v][e + 1], acc[v][e + 2],
                   acc[v][e + 3]);
        }
      } else if (vec_out) {
#pragma unroll
        for (int e = 0; e < PPV; e += 2) {
          *reinterpret_cast<ulonglong2*>(o + 2 * e) =
              make_ulonglong2(acc[v][e], acc[v][e + 1]);
        }
      } else {
#pragma unroll
        for (int e = 0; e < PPV; ++e) {
          o[2 * e] = LoF(acc[v][e]);
          o[2 * e + 1] = HiF(acc[v][e]);
        }
      }
    }
#pragma unroll
    for (int e = 0; e < PPV; ++e) acc[v][e] = 0;
  }
  *wsum = 0.0f;
}

// Checks a bag's offsets; returns false (recording the error in fused mode)
// when the bag must be skipped.
__device__ __forceinline__ bool CheckBag(const PoolParams& p, const BagDesc& d,
                                         int64_t begin, int64_t end) {
  const bool weights_short = d.weights != nullptr && end > d.num_weights;
  const bool bad = begin < 0 || end < begin || end > d.num_ids || weights_short;
  if (bad && p.fused_checks) {
    unsigned int f = 0;
    if (begin < 0 || end < begin) f |= kErrBadOffsets;
    if (end > d.num_ids) f |= kErrLastExceedsIds;
    if (weights_short) f |= kErrLastExceedsWeights;
    RecordError(p.status, d.slot, f);
  }
  return !bad;
}

__device__ __forceinline__ bool SafeBag(const BagDesc& d, int64_t begin,
                                        int64_t end) {
  return begin >= 0 && end >= begin && end <= d.num_ids &&
         (d.weights == nullptr || end <= d.num_weights);
}

// Loads the id (and weight) at position pos + gl of a bag ending at end.
template <int WM>
__device__ __forceinline__ void LoadChunk(const BagDesc& d, int64_t pos,
                                          int64_t end, int gl, int64_t* id,
                                          float* w) {
  if (pos + gl < end) {
    *id = LoadIndex(d.ids, d.ids64, pos + gl);
    if constexpr (WM != kUnweighted) *w = __ldg(d.weights + pos + gl);
  }
}

// One bag per lane-group task. Every descriptor of a launch has weighting
// mode WM (the launcher groups requests by mode). A group pools its bags in
// grid-stride order with one bag of lookahead: the next bag's offsets are
// loaded when the current bag starts, and the next id chunk -- of this bag,
// or the first of the next bag -- is loaded while the current chunk's first
// rows are in flight, so a bag's dependent loads (offsets, then ids, then
// rows) overlap the previous bag's row gathers.
//
// UR selects the rows in flight per batch: 0 takes the throughput setting
// (RowsInFlight, sized for MinBlocks resident blocks); a deep setting (a
// whole id chunk) serves launches too small to fill the GPU, where each
// group pools one or two bags and every batch is a full memory round trip.
//
// One launch serves every weighting mode of a layout group: descriptors are
// sorted by mode, and each mode's tasks [task_lo, task_hi) are pooled by its
// own range of blocks with a body compiled for that mode (a block never
// switches mode, so the bodies do not share registers).
template <int DT, int G, int V, bool EXACT, bool WIDE, int WM, int UR>
__device__ __forceinline__ void PoolBody(const PoolParams& p, int64_t task_lo,
                                         int64_t task_hi, int64_t block,
                                         int64_t blocks) {
  constexpr int PPV = ElemsPerVec<DT>::value / 2;
  constexpr int U = UR == 0 ? RowsInFlight<DT, V, WIDE>::value : UR;
  constexpr int kGroupsPerBlock = kThreads / G;
  constexpr bool kL1 = XSE_POOL_L1 != 0;
  constexpr int kChunkPrefetchTo =  // 0 none, 1 L2, 2 L1
      UR != 0 ? 0
      : DT == 2 ? XSE_POOL_I8_CHUNK_PREFETCH
                : (XSE_POOL_CHUNK_PREFETCH != 0 ? (kL1 ? 2 : 1) : 0);
  constexpr bool kChunkPrefetch = kChunkPrefetchTo != 0;
  constexpr bool kBatchPrefetch =
      (DT == 2 ? XSE_POOL_I8_PREFETCH : XSE_POOL_PREFETCH) != 0 &&
      !kChunkPrefetch;

  const int lane = threadIdx.x & 31;
  const int gl = lane % G;
  const unsigned gmask =
      G == 32 ? 0xffffffffu : (((1u << G) - 1u) << (lane - gl));
  const int64_t stride = blocks * kGroupsPerBlock;
  int64_t task = task_lo + block * kGroupsPerBlock + threadIdx.x / G;
  if (task >= task_hi) return;
  int t = AdvanceDesc(p, 0, task);
  int64_t begin, end;
  {
    const BagDesc& d = p.d[t];
    begin = LoadIndex(d.offsets, d.offs64, task - d.task_begin);
    end = LoadIndex(d.offsets, d.offs64, task - d.task_begin + 1);
  }
  bool have_chunk = false;  // cid/cw hold the current bag's first chunk
  int64_t cid = 0;
  float cw = 1.0f;
  for (;;) {
    const BagDesc& d = p.d[t];
    const int64_t bag = task - d.task_begin;
    // Lookahead: the next task's offsets, consumed one bag later.
    const int64_t ntask = task + stride;
    const bool has_next = ntask < task_hi;
    int nt = t;
    int64_t nbegin = 0, nend = 0;
    if (has_next) {
      nt = AdvanceDesc(p, t, ntask);
      const BagDesc& nd = p.d[nt];
      nbegin = LoadIndex(nd.offsets, nd.offs64, ntask - nd.task_begin);
      nend = LoadIndex(nd.offsets, nd.offs64, ntask - nd.task_begin + 1);
    }
    bool next_chunk = false;
    if (CheckBag(p, d, begin, end)) {
      const int row_vecs = EXACT ? G * V : d.dim / ElemsPerVec<DT>::value;
      const uint4* rows = static_cast<const uint4*>(d.rows) + gl * (WIDE ? V : 1);
      u64 acc[V][PPV];
#pragma unroll
      for (int v = 0; v < V; ++v)
#pragma unroll
        for (int k = 0; k < PPV; ++k) acc[v][k] = 0;
      float wsum = 0.0f;
      float bsum = 0.0f;
      if (!have_chunk) LoadChunk<WM>(d, begin, end, gl, &cid, &cw);
      for (int64_t base = begin; base < end; base += G) {
        const int cnt = static_cast<int>(end - base < G ? end - base : G);
        const int64_t id = cid;
        const float my_w = cw;
        const bool last = base + G >= end;
        // Issued after the chunk's first batch of rows: the next chunk of
        // this bag, or the next bag's first chunk.
        bool pending = true;
        auto prefetch = [&]() {
          if (!pending) return;
          pending = false;
          if (!last) {
            LoadChunk<WM>(d, base + G, end, gl, &cid, &cw);
          } else if (has_next) {
            const BagDesc& nd = p.d[nt];
            if (SafeBag(nd, nbegin, nend)) {
              LoadChunk<WM>(nd, nbegin, nend, gl, &cid, &cw);
              next_chunk = true;
            }
          }
        };
        const int my_row = StageRow(p, d, id, base + gl, gl < cnt);
        if constexpr (kChunkPrefetch) {
          if (my_row >= 0) {
            const int row_bytes = row_vecs * 16;
            PrefetchRow<kChunkPrefetchTo == 2>(
                static_cast<const char*>(d.rows) +
                    static_cast<int64_t>(my_row) * row_bytes,
                row_bytes);
          }
        }
        int j0 = 0;
        if (__all_sync(gmask, gl >= cnt || my_row >= 0)) {
          for (; j0 + U <= cnt; j0 += U) {
            FullBatch<DT, G, V, EXACT, WIDE, WM, U, kL1, kBatchPrefetch>(
                d, rows, row_vecs, gl, gmask, my_row, my_w, j0, cnt, acc,
                &wsum, &bsum, prefetch);
          }
          for (; j0 < cnt; j0 += U) {
            const int n = cnt - j0 < U ? cnt - j0 : U;
            GatherBatch<DT, G, V, EXACT, WIDE, WM, U, kL1>(
                d, rows, row_vecs, gl, gmask, my_row, my_w, j0, n, acc,
                &wsum, &bsum, prefetch);
          }
        } else {
          SparseChunk<DT, G, V, EXACT, WIDE, WM, 1, kL1>(
              d, rows, row_vecs, gl, gmask, my_row, my_w, cnt, acc, &wsum,
              &bsum, prefetch);
        }
      }
      FinishBag<DT, G, V, EXACT, true, WIDE>(d, BagOut(p, d, bag),
                                             d.vec_out, end - begin,
                                             WM != kUnweighted, acc, &wsum,
                                             gl, row_vecs, &bsum);
    }
    if (!has_next) break;
    task = ntask;
    t = nt;
    begin = nbegin;
    end = nend;
    have_chunk = next_chunk;
  }
}

// Programmatic dependent launch. The validation and pooling kernels are
// launched so that the next kernel of the stream may be scheduled before they
// finish: each of them lets its dependents launch on entry and, before its
// first global-memory access, waits until the kernel before it has completed
// and its writes are visible (griddepcontrol.wait returns at once when the
// launch had no programmatic dependency). The overlap hides the launch and
// block-scheduling latency between consecutive kernels of a step and
// between steps; no data is read early.
__device__ __forceinline__ void EnterDependent() {
#if XSE_PDL
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
#endif
}

template <int DT, int G, int V, bool EXACT, int UR, bool WIDE = false>
__global__ void __launch_bounds__(kThreads,
                                  UR == 0 ? MinBlocks<DT, V, WIDE>::value : 2)
    PoolVecKernel(const __grid_constant__ PoolParams p) {
  EnterDependent();
  if (!p.fused_checks && p.status->group_error != 0) return;
  const int64_t b = blockIdx.x;
  const int64_t b0 = p.mode_blocks[0], b1 = p.mode_blocks[1];
  if (b < b0) {
    PoolBody<DT, G, V, EXACT, WIDE, kUnweighted, UR>(p, 0, p.mode_tasks[0], b,
                                                     b0);
  } else if (b < b1) {
    PoolBody<DT, G, V, EXACT, WIDE, kWeightedSum, UR>(p, p.mode_tasks[0],
                                                      p.mode_tasks[1], b - b0,
                                                      b1 - b0);
  } else {
    PoolBody<DT, G, V, EXACT, WIDE, kWeightedNorm, UR>(p, p.mode_tasks[1],
                                                       p.mode_tasks[2],
                                                       b - b1, gridDim.x - b1);
  }
}

// ---- staged kernel ---------------------------------------------------------
//
// PoolVecKernel holds the rows of a batch in registers, U per lane, so a bag
// of n ids takes about n/U row round trips; with few bags per group (small
// launches) or with rows that mostly hit the caches (skewed ids) those round
// trips, not bandwidth, set the time. Here each lane copies its 16-byte
// column of up to kStageRows rows of the bag straight into its own
// shared-memory slots with cp.async (LDGSTS, no registers held while in
// flight), so a whole round of rows is requested at once, and then adds them
// from shared memory in CSR order with the same arithmetic as PoolVecKernel.
// A lane reads back only the slots it filled itself, so lanes never wait for
// one another's copies. Rows of exactly G 16-byte vectors (G = 4..32), one
// lane per vector; int8 rows take their (scale, bias) from the lane that
// holds the row's id. Small launches always use it; for larger ones the
// engine's tuner times both kernels and keeps the faster.
constexpr int kStageRows = 32;       // rows per round of a lane group
constexpr int kStageThreads = 448;   // 14 warps: 448 * 32 * 16 B = 224 KB
constexpr size_t kStageSmem =
    static_cast<size_t>(kStageThreads) * kStageRows * sizeof(uint4);

__device__ __forceinline__ void CopyAsync16(void* smem_dst,
                                            const void* global_src) {
  const uint32_t dst =
      static_cast<uint32_t>(__cvta_generic_to_shared(smem_dst));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 16;" ::"r"(dst),
               "l"(global_src)
               : "memory");
}

__device__ __forceinline__ void CopyAsyncWaitAll() {
  asm volatile("cp.async.commit_group;" ::: "memory");
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

// Ids (and weights) of one round of a bag: position k*G + gl of the round
// starting at `base` on this lane, for k < K (zero past the bag's end).
template <int WM, int G, int K>
__device__ __forceinline__ void LoadRound(const BagDesc& d, int64_t base,
                                          int64_t end, int gl,
                                          int64_t (&id)[K], float (&w)[K]) {
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int64_t pos = base + k * G + gl;
    id[k] = 0;
    w[k] = 1.0f;
    if (pos < end) {
      id[k] = LoadIndex(d.ids, d.ids64, pos);
      if constexpr (WM != kUnweighted) w[k] = __ldg(d.weights + pos);
    }
  }
}

// A group pools its bags (grid-stride tasks) as a software pipeline: while a
// bag's first round of rows is in flight it loads the next bag's first-round
// ids (whose offsets it loaded one bag earlier) and the offsets of the bag
// after that, so consecutive bags cost about one row round trip each.
// Further rounds of a long bag load their ids when they start.
template <int DT, int G, int WM>
__device__ __forceinline__ void StagedBody(const PoolParams& p,
                                           int64_t task_lo, int64_t task_hi,
                                           int64_t block, int64_t blocks,
                                           uint4* smem) {
  constexpr int PPV = ElemsPerVec<DT>::value / 2;
  constexpr int kGroups = kStageThreads / G;
  constexpr int K = kStageRows / G;  // ids per lane per round
  const int lane = threadIdx.x & 31;
  const int gl = lane % G;
  const unsigned gmask =
      G == 32 ? 0xffffffffu : (((1u << G) - 1u) << (lane - gl));
  const int group = threadIdx.x / G;
  // Slot of row u for this lane: mine[u * G].
  uint4* const mine = smem + group * (kStageRows * G) + gl;
  const int64_t stride = blocks * kGroups;
  int64_t task = task_lo + block * kGroups + group;
  if (task >= task_hi) return;
  int t = AdvanceDesc(p, 0, task);
  int64_t begin, end;
  {
    const BagDesc& d = p.d[t];
    begin = LoadIndex(d.offsets, d.offs64, task - d.task_begin);
    end = LoadIndex(d.offsets, d.offs64, task - d.task_begin + 1);
  }
  int64_t cid[K];
  float cw[K];
  if (SafeBag(p.d[t], begin, end)) {
    LoadRound<WM, G, K>(p.d[t], begin, end, gl, cid, cw);
  } else {
#pragma unroll
    for (int k = 0; k < K; ++k) {
      cid[k] = 0;
      cw[k] = 1.0f;
    }
  }
  int64_t ntask = task + stride;
  int nt = t;
  int64_t nbegin = 0, nend = 0;
  if (ntask < task_hi) {
    nt = AdvanceDesc(p, t, ntask);
    const BagDesc& nd = p.d[nt];
    nbegin = LoadIndex(nd.offsets, nd.offs64, ntask - nd.task_begin);
    nend = LoadIndex(nd.offsets, nd.offs64, ntask - nd.task_begin + 1);
  }
  for (;;) {
    const BagDesc& d = p.d[t];
    const int64_t bag = task - d.task_begin;
    const bool has_next = ntask < task_hi;
    const int64_t n2task = ntask + stride;
    int n2t = nt;
    int64_t n2begin = 0, n2end = 0;
    int64_t xid[K];
    float xw[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      xid[k] = 0;
      xw[k] = 1.0f;
    }
    bool prefetched = false;
    // The next bag's first-round ids and the offsets after it.
    auto prefetch = [&]() {
      prefetched = true;
      if (has_next && SafeBag(p.d[nt], nbegin, nend)) {
        LoadRound<WM, G, K>(p.d[nt], nbegin, nend, gl, xid, xw);
      }
      if (n2task < task_hi) {
        n2t = AdvanceDesc(p, nt, n2task);
        const BagDesc& n2d = p.d[n2t];
        n2begin = LoadIndex(n2d.offsets, n2d.offs64, n2task - n2d.task_begin);
        n2end =
            LoadIndex(n2d.offsets, n2d.offs64, n2task - n2d.task_begin + 1);
      }
    };
    if (CheckBag(p, d, begin, end)) {
      const uint4* rows = static_cast<const uint4*>(d.rows) + gl;
      u64 acc[1][PPV];
#pragma unroll
      for (int k = 0; k < PPV; ++k) acc[0][k] = 0;
      float wsum = 0.0f;
      float bsum = 0.0f;
      for (int64_t base = begin; base < end; base += kStageRows) {
        const int cnt = static_cast<int>(
            end - base < kStageRows ? end - base : kStageRows);
        if (base != begin) LoadRound<WM, G, K>(d, base, end, gl, cid, cw);
        int my_row[K];
        float2 my_sb[K];  // int8 rows: (scale, bias) of this lane's id
#pragma unroll
        for (int k = 0; k < K; ++k) {
          const int j = k * G + gl;
          my_row[k] = StageRow(p, d, cid[k], base + j, j < cnt);
          if constexpr (DT == 2) {
            my_sb[k] = my_row[k] >= 0 ? __ldg(d.scale_bias + my_row[k])
                                      : make_float2(0.0f, 0.0f);
          }
        }
        // Every contributing row of the round in flight at once.
        unsigned int present = 0;
#pragma unroll
        for (int k = 0; k < K; ++k) {
          if (k * G < cnt) {
#pragma unroll
            for (int jj = 0; jj < G; ++jj) {
              const int u = k * G + jj;
              const int r = __shfl_sync(gmask, my_row[k], jj, G);
              if (u < cnt && r >= 0) {
                CopyAsync16(mine + u * G, rows + static_cast<int64_t>(r) * G);
                present |= 1u << u;
              }
            }
          }
        }
        if (!prefetched) prefetch();
        CopyAsyncWaitAll();
        // Adds in CSR order.
#pragma unroll
        for (int k = 0; k < K; ++k) {
          if (k * G < cnt) {
#pragma unroll
            for (int jj = 0; jj < G; ++jj) {
              const int u = k * G + jj;
              float w = 1.0f;
              if constexpr (WM != kUnweighted) {
                w = __shfl_sync(gmask, cw[k], jj, G);
              }
              if (u < cnt) {
                if constexpr (WM != kUnweighted) {
                  AddWeight<WM>(&wsum, w, d.combine);
                }
                float2 sb = make_float2(0.0f, 0.0f);
                if constexpr (DT == 2) {
                  sb.x = __shfl_sync(gmask, my_sb[k].x, jj, G);
                  sb.y = __shfl_sync(gmask, my_sb[k].y, jj, G);
                }
                if ((present >> u) & 1u) {
                  const uint4 raw[1] = {mine[u * G]};
                  AddGathered<DT, 1, WM>(acc, raw, sb, w, &bsum);
                }
              }
            }
          }
        }
      }
      FinishBag<DT, G, 1, true, true>(d, BagOut(p, d, bag),
                                      d.vec_out, end - begin,
                                      WM != kUnweighted, acc, &wsum, gl, G,
                                      &bsum);
    }
    if (!prefetched) prefetch();
    if (!has_next) break;
    task = ntask;
    t = nt;
    begin = nbegin;
    end = nend;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      cid[k] = xid[k];
      cw[k] = xw[k];
    }
    ntask = n2task;
    nt = n2t;
    nbegin = n2begin;
    nend = n2end;
  }
}

template <int DT, int G>
__global__ void __launch_bounds__(kStageThreads, 1)
    PoolStagedKernel(const __grid_constant__ PoolParams p) {
  EnterDependent();
  if (!p.fused_checks && p.status->group_error != 0) return;
  extern __shared__ uint4 stage_smem[];
  const int64_t b = blockIdx.x;
  const int64_t b0 = p.mode_blocks[0], b1 = p.mode_blocks[1];
  if (b < b0) {
    StagedBody<DT, G, kUnweighted>(p, 0, p.mode_tasks[0], b, b0, stage_smem);
  } else if (b < b1) {
    StagedBody<DT, G, kWeightedSum>(p, p.mode_tasks[0], p.mode_tasks[1],
                                    b - b0, b1 - b0, stage_smem);
  } else {
    StagedBody<DT, G, kWeightedNorm>(p, p.mode_tasks[1], p.mode_tasks[2],
                                     b - b1, gridDim.x - b1, stage_smem);
  }
}

// ---- fused pooling + dot interaction --------------------------------------
//
// Blocks take samples one at a time from a counter in the status block (a
// block's local sample ls is the ls-th it took), so that all blocks finish
// together; a block's items are (local sample, request) pairs in
// sample-major order, taken one at a time by its warps from a shared counter
// (request t's bag b is table t of sample b). The warp that takes a sample's
// first item fetches the sample. A warp pools its
// bag with the same per-bag code (CSR order, the same roundings) as
// PoolVecKernel and stores the row into the sample's slot of shared memory,
// Z[slot] = [dense; pooled_0; ...; pooled_{T-1}] (row stride RS floats; NS
// slots in a ring). The warp that stores a sample's last row computes its
// interaction row -- [dense, Z[i].Z[j] for 0 <= i < j <= T (row-major),
// zeros to out_stride] -- and frees the slot; the other warps keep pooling
// meanwhile, so no block-wide barrier stalls the gathers. The pooled
// [B, T, D] tensor never reaches HBM. The Gram Z Z^T (R = T + 1 <= 32 rows)
// runs on the tensor cores as split-TF32 mma.sync tiles (three MMAs per tile,
// fp32 accumulation: fp32-level accuracy). A warp that needs a slot still
// held by the sample NS before waits for it with a bounded spin.

// x = hi + lo: hi is x with the 13 low mantissa bits cleared (exact in
// TF32), lo = x - hi (exact in fp32, |lo| < 2^-10 |x|); the MMA reads lo's
// top TF32 bits, so lo*hi' + hi*lo' + hi*hi' carries x*y to about 2^-20
// relative, the dropped lo*lo' being below that. A mask and a subtraction:
// the conversion instructions' throughput would bound the Gram.
__device__ __forceinline__ void SplitTf32(float x, uint32_t* hi,
                                          uint32_t* lo) {
  const uint32_t h = __float_as_uint(x) & 0xffffe000u;
  *hi = h;
  *lo = __float_as_uint(x - __uint_as_float(h));
}

// Stores interaction value v at o[i], or -- when the caller asked for the
// next layer's split operands (olo non-null) -- its TF32 part rounded to
// nearest (ties away, as xse_tf32_split) at o[i] and the exact remainder
// at olo[i].
__device__ __forceinline__ void StoreInteraction(float* o, float* olo,
                                                 int64_t i, float v) {
  if (olo == nullptr) {
    o[i] = v;
    return;
  }
  uint32_t h;
  asm("cvt.rna.tf32.f32 %0, %1;" : "=r"(h) : "f"(v));
  const float vh = __uint_as_float(h);
  o[i] = vh;
  olo[i] = __fsub_rn(v, vh);
}

// acc += A (16x8, row-major fragment a) * B (8x8, column-major fragment b).
__device__ __forceinline__ void MmaTf32(float (&acc)[4], const uint32_t (&a)[4],
                                        uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k8.row.col.f32.tf32.tf32.f32 "
      "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
      : "+f"(acc[0]), "+f"(acc[1]), "+f"(acc[2]), "+f"(acc[3])
      : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}

// Gram of one sample's rows Z[0..R) (R <= 32, row stride RS floats, D
// columns) on the tensor cores, half `half` of the six 16x8 output tiles
// that hold the pairs i < j: half 0 (rows 0-15) x (cols 0-7, 8-15, 16-23),
// half 1 (rows 0-15) x (cols 24-31) and (rows 16-31) x (cols 16-23, 24-31).
// Each product is split into TF32 hi/lo parts (three MMAs), accumulated in
// fp32. Rows past R read row R-1; their outputs are not stored. Writes pair
// (i, j) to o[i (2R - i - 1) / 2 + j - i - 1].
template <int D, int HALF>
__device__ __forceinline__ void GramHalfTf32x3(const float* zs, int R, int RS,
                                               float* o, float* olo) {
  const int lane = threadIdx.x & 31;
  const int g = lane >> 2, tig = lane & 3;
  const float* rp[4];
#pragma unroll
  for (int k = 0; k < 4; ++k) {
    const int r = 8 * k + g;
    rp[k] = zs + (r < R ? r : R - 1) * RS + tig;
  }
  float acc[3][4];
#pragma unroll
  for (int t = 0; t < 3; ++t)
#pragma unroll
    for (int e = 0; e < 4; ++e) acc[t][e] = 0.0f;
#pragma unroll 1
  for (int k0 = 0; k0 < D; k0 += 8) {
    // v[2k] = Z[8k+g][k0+tig], v[2k+1] = Z[8k+g][k0+tig+4].
    uint32_t hi[8], lo[8];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      SplitTf32(rp[k][k0], &hi[2 * k], &lo[2 * k]);
      SplitTf32(rp[k][k0 + 4], &hi[2 * k + 1], &lo[2 * k + 1]);
    }
    // A fragments: row block 0 = rows 0-15, row block 1 = rows 16-31.
    const uint32_t a0h[4] = {hi[0], hi[2], hi[1], hi[3]};
    const uint32_t a0l[4] = {lo[0], lo[2], lo[1], lo[3]};
    const uint32_t a1h[4] = {hi[4], hi[6], hi[5], hi[7]};
    const uint32_t a1l[4] = {lo[4], lo[6], lo[5], lo[7]};
    // B fragment of column block c: (hi[2c], hi[2c+1]).
#pragma unroll
    for (int t = 0; t < 3; ++t) {
      const int cb = HALF == 0 ? t : (t == 0 ? 3 : t + 1);
      const bool rb1 = HALF == 1 && t > 0;
      const uint32_t(&ah)[4] = rb1 ? a1h : a0h;
      const uint32_t(&al)[4] = rb1 ? a1l : a0l;
      MmaTf32(acc[t], al, hi[2 * cb], hi[2 * cb + 1]);
      MmaTf32(acc[t], ah, lo[2 * cb], lo[2 * cb + 1]);
      MmaTf32(acc[t], ah, hi[2 * cb], hi[2 * cb + 1]);
    }
  }
#pragma unroll
  for (int t = 0; t < 3; ++t) {
    const int cb = HALF == 0 ? t : (t == 0 ? 3 : t + 1);
    const int i0 = (HALF == 1 && t > 0) ? 16 + g : g;
    const int j0 = 8 * cb + 2 * tig;
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int i = i0 + (e >= 2 ? 8 : 0);
      const int j = j0 + (e & 1);
      if (i < j && j < R) {
        StoreInteraction(o, olo, i * (2 * R - i - 1) / 2 + j - i - 1,
                         acc[t][e]);
      }
    }
  }
}

constexpr int kInteractSlots = 4;
constexpr int kSampleRing = 8;  // > kInteractSlots + 1 local samples in flight
constexpr int kSlotSpinLimit = 1 << 22;  // polls (~1 s with the back-off)

// Warp-wide: waits until *flag == want (shared memory); false if the wait
// ran out.
__device__ __forceinline__ bool WaitShared(const volatile long long* flag,
                                           long long want) {
  for (int it = 0; it < kSlotSpinLimit; ++it) {
    if (*flag == want) return true;
    __nanosleep(64);
  }
  return false;
}

template <int DT, int WM>
__global__ void __launch_bounds__(kThreads, MinBlocks<DT, 1>::value)
    PoolInteractKernel(const __grid_constant__ PoolParams p,
                       const InteractArgs a) {
  constexpr int G = 32, V = 1;
  constexpr bool EXACT = true;
  constexpr int PPV = ElemsPerVec<DT>::value / 2;
  constexpr int U = RowsInFlight<DT, V>::value;
  constexpr int D = G * ElemsPerVec<DT>::value;
  constexpr int kNs = kInteractSlots;
  constexpr bool kL1 = XSE_INTERACT_L1 != 0;
  constexpr bool kChunkPrefetch = XSE_INTERACT_CHUNK_PREFETCH != 0;
  constexpr bool kBatchPrefetch =
      (DT == 2 ? XSE_POOL_I8_PREFETCH : XSE_POOL_PREFETCH) != 0 &&
      !kChunkPrefetch;
  EnterDependent();
  if (!p.fused_checks && p.status->group_error != 0) return;
  extern __shared__ float4 smem_vec[];
  __shared__ long long owner[kNs];  // local sample allowed in each slot
  __shared__ int filled[kNs];       // rows stored for that sample
  __shared__ long long next_item;
  __shared__ long long sample_of[kSampleRing];   // global sample of ls
  __shared__ long long sample_tag[kSampleRing];  // the ls stored there
  const int T = p.n, R = T + 1, RS = a.row_stride;
  const int P = R * (R - 1) / 2;
  const int64_t width = D + P;
  float* z = reinterpret_cast<float*>(smem_vec);
  const int lane = threadIdx.x & 31;
  const int gl = lane;
  const unsigned gmask = 0xffffffffu;
  if (threadIdx.x < kNs) {
    owner[threadIdx.x] = threadIdx.x;
    filled[threadIdx.x] = 0;
  }
  if (threadIdx.x < kSampleRing) sample_tag[threadIdx.x] = -1;
  if (threadIdx.x == 0) next_item = kThreads / 32;
  __syncthreads();

  // Item u -> (local sample, request, global sample); false once the
  // samples are used up (or a wait ran out). Fetches are not in local
  // order, so a sample past the end can precede valid ones: the warp that
  // fetched it passes its slot on (FreeSlot) once it holds no other item.
  auto resolve = [&](int64_t item, int64_t* ls, int* t, int64_t* gs,
                     bool* fetched) {
    *ls = item / T;
    *t = static_cast<int>(item % T);
    *fetched = *t == 0;
    const int k = static_cast<int>(*ls % kSampleRing);
    volatile long long* vs = &sample_of[k];
    long long g = 0;
    if (*t == 0) {
      if (lane == 0) {
        g = atomicAdd(&p.status->work_counter, 1u);
        *vs = g;
        __threadfence_block();
        *reinterpret_cast<volatile long long*>(&sample_tag[k]) = *ls;
      }
      g = __shfl_sync(0xffffffffu, g, 0);
    } else {
      if (!WaitShared(&sample_tag[k], *ls)) {
        if (lane == 0) RecordError(p.status, 0, kErrDeviceWait);
        *fetched = false;
        return false;
      }
      g = *vs;
    }
    *gs = g;
    return g < a.batch;
  };
  // Passes the slot of local sample ls (past the end: no rows, no
  // interaction) on to ls + kNs once ls may hold it.
  auto free_slot = [&](int64_t lsv) {
    const int sl = static_cast<int>(lsv % kNs);
    if (!WaitShared(&owner[sl], lsv)) {
      if (lane == 0) RecordError(p.status, 0, kErrDeviceWait);
      return;
    }
    __syncwarp();
    if (lane == 0) {
      *reinterpret_cast<volatile long long*>(&owner[sl]) = lsv + kNs;
    }
  };
  int64_t u = threadIdx.x / 32;
  int t;
  int64_t ls, bag, begin, end;
  bool fetched;
  if (!resolve(u, &ls, &t, &bag, &fetched)) {
    if (fetched) free_slot(ls);
    return;
  }
  {
    const BagDesc& d = p.d[t];
    begin = LoadIndex(d.offsets, d.offs64, bag);
    end = LoadIndex(d.offsets, d.offs64, bag + 1);
  }
  bool have_chunk = false;
  int64_t cid = 0;
  float cw = 1.0f;
  for (;;) {
    const BagDesc& d = p.d[t];
    // Lookahead: take the next item now and load its offsets.
    long long nu = 0;
    if (lane == 0) {
      nu = atomicAdd(reinterpret_cast<unsigned long long*>(&next_item), 1ull);
    }
    nu = __shfl_sync(0xffffffffu, nu, 0);
    int nt = t;
    int64_t nls = 0, nbag = 0, nbegin = 0, nend = 0;
    bool nfetched;
    const bool has_next = resolve(nu, &nls, &nt, &nbag, &nfetched);
    if (has_next) {
      const BagDesc& nd = p.d[nt];
      nbegin = LoadIndex(nd.offsets, nd.offs64, nbag);
      nend = LoadIndex(nd.offsets, nd.offs64, nbag + 1);
    }
    bool next_chunk = false;
    const int slot = static_cast<int>(ls % kNs);
    float* zs = z + static_cast<size_t>(slot) * R * RS;
    const bool ok = CheckBag(p, d, begin, end);
    u64 acc[V][PPV];
#pragma unroll
    for (int k = 0; k < PPV; ++k) acc[0][k] = 0;
    float wsum = 0.0f;
    float bsum = 0.0f;  // int8 rows only; the fused kernel serves fp32/bf16
    if (ok) {
      const int row_vecs = G * V;
      const uint4* rows = static_cast<const uint4*>(d.rows) + gl;
      if (!have_chunk) LoadChunk<WM>(d, begin, end, gl, &cid, &cw);
      for (int64_t base = begin; base < end; base += G) {
        const int cnt = static_cast<int>(end - base < G ? end - base : G);
        const int64_t id = cid;
        const float my_w = cw;
        const bool last = base + G >= end;
        bool pending = true;
        auto prefetch = [&]() {
          if (!pending) return;
          pending = false;
          if (!last) {
            LoadChunk<WM>(d, base + G, end, gl, &cid, &cw);
          } else if (has_next) {
            const BagDesc& nd = p.d[nt];
            if (SafeBag(nd, nbegin, nend)) {
              LoadChunk<WM>(nd, nbegin, nend, gl, &cid, &cw);
              next_chunk = true;
            }
          }
        };
        const int my_row = StageRow(p, d, id, base + gl, gl < cnt);
        if constexpr (kChunkPrefetch) {
          if (my_row >= 0) {
            PrefetchRow<XSE_INTERACT_CHUNK_PREFETCH == 2>(
                static_cast<const char*>(d.rows) +
                    static_cast<int64_t>(my_row) * (row_vecs * 16),
                row_vecs * 16);
          }
        }
        int j0 = 0;
        if (__all_sync(gmask, gl >= cnt || my_row >= 0)) {
          for (; j0 + U <= cnt; j0 += U) {
            FullBatch<DT, G, V, EXACT, false, WM, U, kL1, kBatchPrefetch>(
                d, rows, row_vecs, gl, gmask, my_row, my_w, j0, cnt, acc,
                &wsum, &bsum, prefetch);
          }
        }
        for (; j0 < cnt; j0 += U) {
          const int n = cnt - j0 < U ? cnt - j0 : U;
          GatherBatch<DT, G, V, EXACT, false, WM, U, kL1>(
              d, rows, row_vecs, gl, gmask, my_row, my_w, j0, n, acc, &wsum,
              &bsum, prefetch);
        }
      }
    }
    // The slot may still hold local sample ls - kNs until its interaction
    // row is out.
    if (!WaitShared(&owner[slot], ls)) {
      if (lane == 0) RecordError(p.status, 0, kErrDeviceWait);
      return;
    }
    if (ok) {
      FinishBag<DT, G, V, EXACT, false>(d, zs + (1 + t) * RS, true,
                                        end - begin, WM != kUnweighted, acc,
                                        &wsum, gl, G * V, &bsum);
    }
    __syncwarp();
    __threadfence_block();
    int done = 0;
    if (lane == 0) done = atomicAdd(&filled[slot], 1) + 1;
    done = __shfl_sync(0xffffffffu, done, 0);
    if (done == T) {
      // Last row of this sample: its interaction row, then free the slot.
      __threadfence_block();
      const float* dense = a.dense + bag * a.dense_stride;
      float* o = a.out + bag * a.out_stride;
      float* olo = a.out_lo != nullptr ? a.out_lo + bag * a.out_stride
                                       : nullptr;
      for (int c = lane * 4; c < D; c += 128) {
        *reinterpret_cast<float4*>(zs + c) =
            __ldg(reinterpret_cast<const float4*>(dense + c));
      }
      __syncwarp();
      for (int c = lane; c < D; c += 32) {
        StoreInteraction(o, olo, c, zs[c]);  // any out alignment
      }
      for (int64_t c = width + lane; c < a.out_stride; c += 32) {
        StoreInteraction(o, olo, c, 0.0f);
      }
      GramHalfTf32x3<D, 0>(zs, R, RS, o + D, olo ? olo + D : nullptr);
      GramHalfTf32x3<D, 1>(zs, R, RS, o + D, olo ? olo + D : nullptr);
      __syncwarp();
      if (lane == 0) {
        filled[slot] = 0;
        __threadfence_block();
        *reinterpret_cast<volatile long long*>(&owner[slot]) = ls + kNs;
      }
    }
    if (!has_next) {
      if (nfetched) free_slot(nls);
      break;
    }
    u = nu;
    ls = nls;
    t = nt;
    bag = nbag;
    begin = nbegin;
    end = nend;
    have_chunk = next_chunk;
  }
}

// Element-wise variant for rows that are not whole 16-byte vectors (odd
// dims or unaligned tables). A warp owns a bag; lanes own columns
// c = lane + 32*k, in column chunks of 32*kCols.
template <int DT>
__global__ void __launch_bounds__(kThreads)
    PoolScalarKernel(const __grid_constant__ PoolParams p) {
  constexpr int kCols = 4;
  EnterDependent();
  if (!p.fused_checks && p.status->group_error != 0) return;
  const int lane = threadIdx.x & 31;
  const int64_t warps_per_block = kThreads / 32;
  const int64_t stride = static_cast<int64_t>(gridDim.x) * warps_per_block;
  int t = 0;
  for (int64_t task = blockIdx.x * warps_per_block + threadIdx.x / 32;
       task < p.total_tasks; task += stride) {
    t = AdvanceDesc(p, t, task);
    const BagDesc& d = p.d[t];
    const int64_t bag = task - d.task_begin;
    int64_t begin, end;
    if (!BagRange(p, d, bag, &begin, &end)) continue;
    const bool weighted = d.weights != nullptr;
    const int64_t n = end - begin;
    for (int c0 = 0; c0 < d.dim; c0 += 32 * kCols) {
      float acc[kCols];
#pragma unroll
      for (int k = 0; k < kCols; ++k) acc[k] = 0.0f;
      float wsum = 0.0f;
      for (int64_t pidx = begin; pidx < end; ++pidx) {
        const int64_t id = LoadIndex(d.ids, d.ids64, pidx);
        const float w = weighted ? __ldg(d.weights + pidx) : 1.0f;
        if (weighted) {
          wsum = __fadd_rn(wsum, d.combine == 3 ? __fmul_rn(w, w) : w);
        }
        if (id < 0 || id >= d.vocab) {
          if (p.fused_checks && lane == 0 && c0 == 0) {
            RecordBadId(p.status, d.slot, pidx);
          }
          continue;
        }
        if (id < d.row_begin || id >= d.row_end) continue;
        const int64_t r = id - d.row_begin;
#pragma unroll
        for (int k = 0; k < kCols; ++k) {
          const int c = c0 + lane + 32 * k;
          if (c < d.dim) {
            float x;
            const int64_t at = r * d.dim + c;
            if constexpr (DT == 0) {
              x = __ldg(static_cast<const float*>(d.rows) + at);
            } else if constexpr (DT == 1) {
              const unsigned short b =
                  __ldg(static_cast<const unsigned short*>(d.rows) + at);
              x = __uint_as_float(static_cast<uint32_t>(b) << 16);
            } else {
              const float2 sb = __ldg(d.scale_bias + r);
              const float q = __int2float_rn(
                  __ldg(static_cast<const signed char*>(d.rows) + at));
              x = __fmaf_rn(q, sb.x, sb.y);
            }
            acc[k] = weighted ? __fadd_rn(acc[k], __fmul_rn(w, x))
                              : __fadd_rn(acc[k], x);
          }
        }
      }
      float s = 1.0f;
      if (n > 0 && d.combine != 1) s = BagScale(d.combine, weighted, n, wsum);
#pragma unroll
      for (int k = 0; k < kCols; ++k) {
        const int c = c0 + lane + 32 * k;
        if (c < d.dim) {
          BagOut(p, d, bag)[c] =
              (n > 0 && d.combine != 1) ? __fmul_rn(acc[k], s) : acc[k];
        }
      }
    }
  }
}

// Group validation (ValidateEmbeddingBagInput, embedding_bag.cc:99-133).
// Offsets must start >= 0 and never decrease; the final offset must not
// exceed the ids (or weights); every id in [first, last) must be in
// [0, vocab). A request's offsets followed by its id positions are cut into
// chunks of kValidateChunk elements; a warp checks one chunk, lane l taking
// elements l, l+32, ... (coalesced), and looks up the chunk's request once.
// Every load of a chunk (its offsets, or its ids -- all in [0, num_ids), so
// in bounds -- and the request's first and last offsets) is issued before
// any is checked, so a chunk costs one memory round trip; checking as the
// loads returned made each id load wait for the previous one's verdict.
constexpr int kValidateChunk = 256;

__global__ void __launch_bounds__(kThreads)
    ValidateKernel(const __grid_constant__ PoolParams p, int64_t total_work) {
  EnterDependent();
  constexpr int K = kValidateChunk / 32;
  const int lane = threadIdx.x & 31;
  const int64_t warps = static_cast<int64_t>(gridDim.x) * (kThreads / 32);
  int t = 0;
  for (int64_t c = static_cast<int64_t>(blockIdx.x) * (kThreads / 32) +
                   threadIdx.x / 32;
       c < total_work; c += warps) {
    t = AdvanceWork(p, t, c);
    const BagDesc& d = p.d[t];
    const int64_t num_offsets = d.num_bags + 1;
    const int64_t elems = num_offsets + d.num_ids;
    const int64_t i0 = (c - d.work_begin) * kValidateChunk;
    const int64_t first = LoadIndex(d.offsets, d.offs64, 0);
    const int64_t last = LoadIndex(d.offsets, d.offs64, d.num_bags);
    int64_t cur[K], prev[K];
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int64_t i = i0 + k * 32 + lane;
      cur[k] = 0;
      prev[k] = 0;
      if (i < num_offsets) {
        cur[k] = LoadIndex(d.offsets, d.offs64, i);
        if (i > 0) prev[k] = LoadIndex(d.offsets, d.offs64, i - 1);
      } else if (i < elems && d.ids != nullptr) {
        cur[k] = LoadIndex(d.ids, d.ids64, i - num_offsets);
      }
    }
    unsigned int flags = 0;
    int64_t bad_pos = -1;
#pragma unroll
    for (int k = 0; k < K; ++k) {
      const int64_t i = i0 + k * 32 + lane;
      if (i < num_offsets) {
        if (i == 0 ? cur[k] < 0 : prev[k] > cur[k]) flags |= kErrBadOffsets;
        if (i == num_offsets - 1) {
          if (cur[k] > d.num_ids) flags |= kErrLastExceedsIds;
          if (d.weights != nullptr && cur[k] > d.num_weights) {
            flags |= kErrLastExceedsWeights;
          }
        }
      } else if (i < elems && d.ids != nullptr) {
        // Positions grow with k: the first bad one is this lane's smallest.
        const int64_t pos = i - num_offsets;
        if (bad_pos < 0 && pos >= first && pos < last &&
            (cur[k] < 0 || cur[k] >= d.vocab)) {
          bad_pos = pos;
        }
      }
    }
    if (flags != 0) RecordError(p.status, d.slot, flags);
    if (bad_pos >= 0) RecordBadId(p.status, d.slot, bad_pos);
  }
}

__global__ void InterleaveKernel(const float* scale, const float* bias,
                                 float2* out, int64_t n) {
  const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
       i < n; i += stride) {
    out[i] = make_float2(scale[i], bias[i]);
  }
}

int SmCount() {
  static int sms = [] {
    int dev = 0, n = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
    return n > 0 ? n : 148;
  }();
  return sms;
}

template <typename Kernel>
int BlocksPerSm(Kernel kernel) {
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads, 0);
  return per_sm > 0 ? per_sm : 1;
}

// Launches `kernel` on `grid` blocks of `threads` with a programmatic
// dependency on the previous kernel of the stream (see EnterDependent).
template <typename... Params, typename... Args>
cudaError_t LaunchDependentBlock(void (*kernel)(Params...), int grid,
                                 int threads, size_t smem,
                                 cudaStream_t stream, Args&&... args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = dim3(static_cast<unsigned>(grid));
  cfg.blockDim = dim3(static_cast<unsigned>(threads));
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = XSE_PDL;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

// Same with blocks of kThreads.
template <typename... Params, typename... Args>
cudaError_t LaunchDependentSmem(void (*kernel)(Params...), int grid,
                                size_t smem, cudaStream_t stream,
                                Args&&... args) {
  return LaunchDependentBlock(kernel, grid, kThreads, smem, stream,
                              std::forward<Args>(args)...);
}

template <typename... Params, typename... Args>
cudaError_t LaunchDependent(void (*kernel)(Params...), int grid,
                            cudaStream_t stream, Args&&... args) {
  return LaunchDependentSmem(kernel, grid, 0, stream,
                             std::forward<Args>(args)...);
}

template <typename Kernel>
int GridFor(Kernel kernel, int64_t groups_needed, int groups_per_block) {
  const int64_t max_grid =
      static_cast<int64_t>(SmCount()) * BlocksPerSm(kernel);
  const int64_t want = (groups_needed + groups_per_block - 1) / groups_per_block;
  return static_cast<int>(want < 1 ? 1 : (want < max_grid ? want : max_grid));
}

// Numbers the tasks of every descriptor for runs of `runs` bags.
void AssignTasks(PoolParams* p, int runs) {
  int64_t tasks = 0;
  for (int k = 0; k < p->n; ++k) {
    p->d[k].task_begin = tasks;
    tasks += (p->d[k].num_bags + runs - 1) / runs;
  }
  p->bags_per_task = runs;
  p->total_tasks = tasks;
}

// Rows in flight of the latency-bound variant (register-limited to 2
// resident blocks per SM): up to XSE_POOL_DEEP_ROWS, at most one id chunk.
#ifndef XSE_POOL_DEEP_ROWS
#define XSE_POOL_DEEP_ROWS 8
#endif
template <int DT, int G, int V>
constexpr int DeepRows() {
  return (DT == 2 || V != 1) ? 0
                             : (G < XSE_POOL_DEEP_ROWS ? G : XSE_POOL_DEEP_ROWS);
}

// Splits `grid` blocks over the weighting modes in proportion to their tasks
// (every mode with tasks gets at least one block) and records the cumulative
// task and block ends in p.
void SplitModes(PoolParams* p, int64_t max_grid, int groups_per_block) {
  int64_t tasks[3] = {0, 0, 0};
  for (int k = 0; k < p->n; ++k) tasks[WeightModeOf(p->d[k])] += p->d[k].num_bags;
  int64_t need[3], total_need = 0;
  for (int m = 0; m < 3; ++m) {
    need[m] = (tasks[m] + groups_per_block - 1) / groups_per_block;
    total_need += need[m];
  }
  int64_t blocks[3] = {0, 0, 0};
  if (total_need <= max_grid) {
    for (int m = 0; m < 3; ++m) blocks[m] = need[m];
  } else {
    const int64_t total = p->total_tasks > 0 ? p->total_tasks : 1;
    for (int m = 0; m < 3; ++m) {
      if (tasks[m] == 0) continue;
      const int64_t share = max_grid * tasks[m] / total;
      blocks[m] = share < 1 ? 1 : share;  // grid-stride covers the rest
    }
  }
  int64_t task_end = 0, block_end = 0;
  for (int m = 0; m < 3; ++m) {
    task_end += tasks[m];
    block_end += blocks[m];
    p->mode_tasks[m] = task_end;
    p->mode_blocks[m] = static_cast<int32_t>(block_end);
  }
}

template <int DT, int G, int V, bool EXACT, bool WIDE = false>
cudaError_t LaunchVec(const PoolParams& in, cudaStream_t stream) {
  PoolParams p = in;
  // Descriptors by weighting mode (stable: request order within a mode). An
  // in-place insertion sort over at most kMaxDescsPerLaunch entries: unlike
  // std::stable_sort it never takes a heap buffer, so launches stay
  // allocation-free.
  for (int k = 1; k < p.n; ++k) {
    const BagDesc moving = p.d[k];
    const int mode = WeightModeOf(moving);
    int j = k;
    while (j > 0 && WeightModeOf(p.d[j - 1]) > mode) {
      p.d[j] = p.d[j - 1];
      --j;
    }
    p.d[j] = moving;
  }
  AssignTasks(&p, 1);
  auto kernel = PoolVecKernel<DT, G, V, EXACT, 0, WIDE>;
  int64_t max_grid = static_cast<int64_t>(SmCount()) * BlocksPerSm(kernel);
#if XSE_POOL_STAGED
  if constexpr ((V == 1 || (WIDE && G * V <= 32)) && EXACT) {
    // At most one wave of the staged kernel's groups (one block per SM):
    // whole rounds of rows in flight per bag (see PoolStagedKernel). Larger
    // launches take it when the caller chose it (kPoolStaged). A wide
    // layout's rows are G * V 16-byte vectors to the staged kernel.
    constexpr int kStagedG = WIDE ? G * V : G;
    constexpr int kGroups = kStageThreads / kStagedG;
    const bool small =
        p.total_tasks <= static_cast<int64_t>(SmCount()) * kGroups;
    if (p.kernel_choice == kPoolStaged ||
        (p.kernel_choice == kPoolAuto &&
         (XSE_POOL_STAGED == 2 || small))) {
      auto staged = PoolStagedKernel<DT, kStagedG>;
      // Set on every launch: the attribute belongs to the current device.
      cudaError_t e = cudaFuncSetAttribute(
          staged, cudaFuncAttributeMaxDynamicSharedMemorySize,
          static_cast<int>(kStageSmem));
      if (e != cudaSuccess) return e;
      SplitModes(&p, SmCount(), kGroups);
      return LaunchDependentBlock(staged, p.mode_blocks[2], kStageThreads,
                                  kStageSmem, stream, p);
    }
  }
#endif
  constexpr int kDeep = DeepRows<DT, G, V>();
  if constexpr (kDeep > 0) {
    // Fewer bags than one wave of the throughput kernel's groups: every
    // group pools about one bag, so latency (round trips per bag), not
    // bandwidth, sets the time; gather a whole chunk per round trip.
    if (p.total_tasks <= max_grid * (kThreads / G)) {
      auto deep = PoolVecKernel<DT, G, V, EXACT, kDeep>;
      SplitModes(&p, static_cast<int64_t>(SmCount()) * BlocksPerSm(deep),
                 kThreads / G);
      return LaunchDependent(deep, p.mode_blocks[2], stream, p);
    }
  }
  SplitModes(&p, max_grid, kThreads / G);
  return LaunchDependent(kernel, p.mode_blocks[2], stream, p);
}

template <int DT, int G, int V>
cudaError_t LaunchVecExact(const Layout& l, const PoolParams& p,
                           cudaStream_t stream) {
  return l.exact ? LaunchVec<DT, G, V, true>(p, stream)
                 : LaunchVec<DT, G, V, false>(p, stream);
}

// Int8 or bf16 rows of 16, 32 or 64 16-byte vectors, 32-byte aligned: each
// lane owns 32 contiguous bytes (one 256-bit load per row), G = vectors / 2.
template <int DT>
cudaError_t LaunchWide(const Layout& l, const PoolParams& p,
                       cudaStream_t stream) {
  if constexpr (DT != 0) {
    switch (l.g) {
      case 8: return LaunchVec<DT, 8, 2, true, true>(p, stream);
      case 16: return LaunchVec<DT, 16, 2, true, true>(p, stream);
      default: return LaunchVec<DT, 32, 2, true, true>(p, stream);
    }
  } else {
    (void)l;
    (void)p;
    (void)stream;
    return cudaErrorNotSupported;
  }
}

template <int DT>
cudaError_t LaunchForDtype(const Layout& l, const PoolParams& p,
                           cudaStream_t stream) {
  if (l.v == 0) {
    PoolParams q = p;
    AssignTasks(&q, 1);
    auto kernel = PoolScalarKernel<DT>;
    const int grid = GridFor(kernel, q.total_tasks, kThreads / 32);
    return LaunchDependent(kernel, grid, stream, q);
  }
  if (l.wide) return LaunchWide<DT>(l, p, stream);
  if (l.v == 1) {
    switch (l.g) {
      case 4: return LaunchVecExact<DT, 4, 1>(l, p, stream);
      case 8: return LaunchVecExact<DT, 8, 1>(l, p, stream);
      case 16: return LaunchVecExact<DT, 16, 1>(l, p, stream);
      default: return LaunchVecExact<DT, 32, 1>(l, p, stream);
    }
  }
  if (l.v == 2) return LaunchVecExact<DT, 32, 2>(l, p, stream);
  if constexpr (DT == 2) {
    return LaunchVecExact<DT, 32, 4>(l, p, stream);
  } else {
    if (l.v == 4) return LaunchVecExact<DT, 32, 4>(l, p, stream);
    return LaunchVecExact<DT, 32, 8>(l, p, stream);
  }
}

// Shared memory of the fused kernel: S samples of R rows (RS floats each).
size_t InteractSmem(int samples, int rows, int row_stride) {
  return static_cast<size_t>(samples) * rows * row_stride * sizeof(float);
}

template <int DT, int WM>
cudaError_t LaunchInteractFor(const PoolParams& p, InteractArgs a,
                              cudaStream_t stream) {
  auto kernel = PoolInteractKernel<DT, WM>;
  constexpr int D = 32 * ElemsPerVec<DT>::value;
  const int rows = p.n + 1;
  a.row_stride = D + 4;  // rows 16-byte aligned, 16-byte bank shift per row
  a.samples_per_tile = kInteractSlots;
  const size_t smem = InteractSmem(kInteractSlots, rows, a.row_stride);
  if (smem > 200 * 1024) return cudaErrorNotSupported;
  // Set on every launch: the attribute belongs to the current device.
  cudaError_t e = cudaFuncSetAttribute(
      kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
      static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  int per_sm = 0;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kernel, kThreads,
                                                smem);
  // Samples are handed out at run time; no more blocks than samples.
  int64_t grid = static_cast<int64_t>(SmCount()) * (per_sm > 0 ? per_sm : 1);
  if (grid > a.batch) grid = a.batch;
  if (grid < 1) grid = 1;
  return LaunchDependentSmem(kernel, static_cast<int>(grid), smem, stream, p,
                             a);
}

template <int DT>
cudaError_t LaunchInteractMode(int wm, const PoolParams& p,
                               const InteractArgs& a, cudaStream_t stream) {
  switch (wm) {
    case kUnweighted: return LaunchInteractFor<DT, kUnweighted>(p, a, stream);
    case kWeightedSum: return LaunchInteractFor<DT, kWeightedSum>(p, a, stream);
    default: return LaunchInteractFor<DT, kWeightedNorm>(p, a, stream);
  }
}

}  // namespace

bool PoolKernelTunable(const Layout& layout, int64_t total_tasks) {
#if XSE_POOL_STAGED
  const int staged_g = layout.wide ? layout.g * layout.v : layout.g;
  if (!layout.exact || (layout.v != 1 && !layout.wide) || staged_g > 32) {
    return false;
  }
  const int64_t groups = kStageThreads / staged_g;
  return total_tasks > static_cast<int64_t>(SmCount()) * groups;
#else
  (void)layout;
  (void)total_tasks;
  return false;
#endif
}

Layout ChooseLayout(int dtype, int dim, const void* rows) {
  const int elem = dtype == 0 ? 4 : dtype == 1 ? 2 : 1;
  const int64_t row_bytes = static_cast<int64_t>(dim) * elem;
  const bool aligned = (reinterpret_cast<uintptr_t>(rows) & 15u) == 0;
  if (!aligned || row_bytes % 16 != 0) return {dtype, 32, 0, false};
  const int64_t vecs = row_bytes / 16;
  // Int8 (and bf16) rows of 256, 512 or 1024 bytes: 32-byte lanes, so a
  // row takes half the lanes, shuffles, address computations and loop
  // steps, and a lane keeps twice the bytes in flight per row it holds.
  // (fp32 rows keep 16-byte lanes: the fused interaction kernel serves
  // that layout.)
  if (((dtype == 2 && XSE_POOL_I8_WIDE) ||
       (dtype == 1 && XSE_POOL_BF16_WIDE)) &&
      (vecs == 16 || vecs == 32 || vecs == 64) &&
      (reinterpret_cast<uintptr_t>(rows) & 31u) == 0) {
    return {dtype, static_cast<int>(vecs / 2), 2, true, 0, true};
  }
  if (vecs <= 32) {
    int g = 4;
    while (g < vecs) g *= 2;
    return {dtype, g, 1, g == vecs};
  }
  const int64_t per_lane = (vecs + 31) / 32;
  int v = 0;
  if (per_lane <= 2) {
    v = 2;
  } else if (per_lane <= 4) {
    v = 4;
  } else if (per_lane <= 8 && dtype != 2) {
    v = 8;
  } else {
    return {dtype, 32, 0, false};
  }
  return {dtype, 32, v, 32 * v == vecs};
}

int64_t TasksFor(const Layout& layout, int64_t num_bags) {
  (void)layout;  // the launcher renumbers tasks for its kernel
  return num_bags;
}

int64_t ValidationWork(int64_t num_bags, int64_t num_ids) {
  return (num_bags + 1 + num_ids + kValidateChunk - 1) / kValidateChunk;
}

cudaError_t LaunchPool(const Layout& layout, const PoolParams& p,
                       cudaStream_t stream, int* launches) {
  if (p.total_tasks <= 0) return cudaSuccess;
  ++*launches;
  switch (layout.dtype) {
    case 0: return LaunchForDtype<0>(layout, p, stream);
    case 1: return LaunchForDtype<1>(layout, p, stream);
    default: return LaunchForDtype<2>(layout, p, stream);
  }
}

cudaError_t LaunchPoolInteract(const Layout& layout, const PoolParams& p,
                               const InteractArgs& a, cudaStream_t stream) {
  if (p.n < 1 || p.n + 1 > 32 || layout.v != 1 || !layout.exact ||
      layout.dtype > 1 || layout.g != 32) {
    return cudaErrorNotSupported;
  }
  const int wm = WeightModeOf(p.d[0]);
  for (int k = 1; k < p.n; ++k) {
    if (WeightModeOf(p.d[k]) != wm) return cudaErrorNotSupported;
  }
  if (((reinterpret_cast<uintptr_t>(a.dense) & 15u) != 0) ||
      a.dense_stride % 4 != 0) {
    return cudaErrorNotSupported;
  }
  if (a.batch <= 0) return cudaSuccess;
  return layout.dtype == 0 ? LaunchInteractMode<0>(wm, p, a, stream)
                           : LaunchInteractMode<1>(wm, p, a, stream);
}

cudaError_t LaunchValidate(const PoolParams& p, int64_t total_work,
                           cudaStream_t stream) {
  if (total_work <= 0) return cudaSuccess;
  const int grid = GridFor(ValidateKernel, total_work, kThreads / 32);
  return LaunchDependent(ValidateKernel, grid, stream, p, total_work);
}

cudaError_t LaunchInterleaveScaleBias(const float* scale, const float* bias,
                                      float2* out, int64_t n,
                                      cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  const int64_t blocks = (n + kThreads - 1) / kThreads;
  const int grid = static_cast<int>(blocks < 4096 ? blocks : 4096);
  InterleaveKernel<<<grid, kThreads, 0, stream>>>(scale, bias, out, n);
  return cudaGetLastError();
}

}  // namespace xse
