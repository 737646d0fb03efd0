// Operator layer: host-buffer operators and the table resource (C ABI in
// include/xse_ops.h).
//
// Mirrors XSE's CpuEmbeddingLookupTransform, DenseCpuEmbeddingLookupTransform
// and CpuEmbeddingEngineResource (data/kernels/cpu_embedding/) with the same
// checks, in the same order, with the same messages. Each call stages the
// host inputs of all features into one pinned buffer, copies them to the GPU
// in one transfer, runs the engine's group execution (validation, then
// pooling) and copies all pooled outputs back in one transfer into pinned
// host buffers.

#include <cuda_runtime.h>
#include <fcntl.h>
#include <stdint.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <algorithm>
#include <cctype>
#include <cinttypes>
#include <climits>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <string>
#include <unordered_map>
#include <unordered_set>
#include <vector>

#include "../../include/xse_emb.h"
#include "../../include/xse_ops.h"
#include "xse_internal.h"

namespace {

// Messages go to the engine's thread-local channel (xse_last_error).
int Fail(int code, const char* fmt, ...) {
  char buf[1024];
  va_list args;
  va_start(args, fmt);
  vsnprintf(buf, sizeof(buf), fmt, args);
  va_end(args);
  xse::SetLastErrorMessage(buf);
  return code;
}

// The engine call that failed already set the message.
int FailFromEngine(int code) { return code; }

int CudaFail(cudaError_t e, const char* what) {
  return Fail(XSE_INTERNAL, "%s: %s", what, cudaGetErrorString(e));
}

// ---------------------------------------------------------------------------
// Pinned host memory. Blocks are pooled by size class so steady-state calls
// do not pay cudaHostAlloc; a block may back several output buffers, and
// returns to the pool when its last buffer is freed.
struct PinnedBlock {
  void* ptr = nullptr;
  size_t bytes = 0;
  int refs = 0;
};

class PinnedPool {
 public:
  static PinnedPool& Get() {
    static PinnedPool* pool = new PinnedPool();  // lives until exit
    return *pool;
  }

  // Returns a block of at least `bytes` with one reference.
  PinnedBlock* Acquire(size_t bytes) {
    const size_t cls = SizeClass(bytes);
    {
      std::lock_guard<std::mutex> lock(mu_);
      auto& free_list = free_[cls];
      if (!free_list.empty()) {
        PinnedBlock* b = free_list.back();
        free_list.pop_back();
        b->refs = 1;
        return b;
      }
    }
    // A new block is allocated outside the lock: cudaHostAlloc takes
    // milliseconds, and other callers' acquires and releases go on meanwhile.
    void* p = nullptr;
    if (cudaHostAlloc(&p, cls, cudaHostAllocDefault) != cudaSuccess) {
      return nullptr;
    }
    return new PinnedBlock{p, cls, 1};
  }

  void Retain(PinnedBlock* b, void* data) {
    std::lock_guard<std::mutex> lock(mu_);
    ++b->refs;
    owners_[data] = b;
  }
  void Register(PinnedBlock* b, void* data) {
    std::lock_guard<std::mutex> lock(mu_);
    owners_[data] = b;
  }

  // Drops one reference; false if `data` is not ours.
  bool ReleaseData(void* data) {
    std::lock_guard<std::mutex> lock(mu_);
    auto it = owners_.find(data);
    if (it == owners_.end()) return false;
    PinnedBlock* b = it->second;
    owners_.erase(it);
    DropLocked(b);
    return true;
  }

  void Release(PinnedBlock* b) {
    std::lock_guard<std::mutex> lock(mu_);
    DropLocked(b);
  }

 private:
  static size_t SizeClass(size_t bytes) {
    size_t c = 4096;
    while (c < bytes) c <<= 1;
    return c;
  }
  void DropLocked(PinnedBlock* b) {
    if (--b->refs == 0) free_[b->bytes].push_back(b);
  }

  std::mutex mu_;
  std::map<size_t, std::vector<PinnedBlock*>> free_;
  std::unordered_map<void*, PinnedBlock*> owners_;
};

size_t DtypeBytes(int32_t dtype) {
  switch (dtype) {
    case XSE_HB_S32:
    case XSE_HB_F32:
      return 4;
    case XSE_HB_S64:
      return 8;
    default:
      return 0;
  }
}

int64_t NumElements(const xse_host_buffer& b) {
  int64_t n = 1;
  for (int32_t i = 0; i < b.rank; ++i) n *= b.dims[i];
  return n;
}

bool Uninitialized(const xse_host_buffer& b) {
  return b.dtype == XSE_HB_INVALID;
}

size_t AlignUp(size_t x, size_t a) { return (x + a - 1) / a * a; }

// True for page-locked host memory (copied by DMA without staging).
bool IsPinned(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();  // clear the sticky-free error of the query
    return false;
  }
  return a.type == cudaMemoryTypeHost;
}

// A device arena that only grows (reused across calls of one operator).
struct DeviceArena {
  int device = 0;
  void* ptr = nullptr;
  size_t bytes = 0;
  ~DeviceArena() {
    if (ptr != nullptr) {
      int prev = 0;
      cudaGetDevice(&prev);
      cudaSetDevice(device);
      cudaFree(ptr);
      cudaSetDevice(prev);
    }
  }
  int Reserve(size_t need) {
    if (need <= bytes) return XSE_OK;
    if (ptr != nullptr) cudaFree(ptr);
    ptr = nullptr;
    bytes = 0;
    const size_t size = std::max(need, static_cast<size_t>(1) << 20);
    const cudaError_t e = cudaMalloc(&ptr, size);
    if (e != cudaSuccess) return CudaFail(e, "device staging allocation");
    bytes = size;
    return XSE_OK;
  }
};

class DeviceGuard {
 public:
  explicit DeviceGuard(int device) : device_(device) {
    cudaGetDevice(&prev_);
    if (prev_ != device_) cudaSetDevice(device_);
  }
  ~DeviceGuard() {
    if (prev_ != device_) cudaSetDevice(prev_);
  }

 private:
  int device_ = 0, prev_ = 0;
};

// ---------------------------------------------------------------------------
// CpuEmbeddingManifest text proto (data/kernels/cpu_embedding/
// cpu_embedding.proto:19-44), plus the optional per-table data_type.
struct ManifestTable {
  std::string name;
  int64_t vocab_size = 0;
  int64_t embedding_dim = 0;
  std::string combine_mode = "COMBINE_MODE_UNSPECIFIED";
  std::string data_type = "FLOAT32";
};

struct ManifestFeature {
  std::string name;
  std::string table;
  int64_t max_sequence_length = 0;
};

struct Manifest {
  std::vector<ManifestTable> tables;
  std::vector<ManifestFeature> features;
  int64_t max_cpu_slots = 0;
  int64_t block_size = 0;
};

// A small text-format reader: `field: value`, `message { ... }` (with an
// optional colon), '#' comments, quoted strings, integers and enum names.
class TextProtoReader {
 public:
  explicit TextProtoReader(const std::string& text) : s_(text) {}

  bool Parse(Manifest* m, std::string* error) {
    while (SkipSpace(), pos_ < s_.size()) {
      std::string field;
      if (!Ident(&field)) return Err(error, "expected a field name");
      if (field == "tables" || field == "feature_specs") {
        if (!OpenBrace()) return Err(error, "expected '{' after " + field);
        if (field == "tables") {
          ManifestTable t;
          if (!ParseTable(&t, error)) return false;
          m->tables.push_back(t);
        } else {
          ManifestFeature f;
          if (!ParseFeature(&f, error)) return false;
          m->features.push_back(f);
        }
      } else if (field == "max_cpu_slots" || field == "block_size") {
        std::string v;
        if (!Colon() || !Scalar(&v)) return Err(error, "bad value of " + field);
        (field == "max_cpu_slots" ? m->max_cpu_slots : m->block_size) =
            std::strtoll(v.c_str(), nullptr, 10);
      } else {
        return Err(error, "unknown field " + field);
      }
    }
    return true;
  }

 private:
  bool ParseTable(ManifestTable* t, std::string* error) {
    while (SkipSpace(), pos_ < s_.size() && s_[pos_] != '}') {
      std::string field, v;
      if (!Ident(&field) || !Colon() || !Scalar(&v)) {
        return Err(error, "malformed table entry");
      }
      if (field == "name") t->name = v;
      else if (field == "vocab_size") t->vocab_size = std::strtoll(v.c_str(), nullptr, 10);
      else if (field == "embedding_dim") t->embedding_dim = std::strtoll(v.c_str(), nullptr, 10);
      else if (field == "combine_mode") t->combine_mode = v;
      else if (field == "data_type") t->data_type = v;
      else return Err(error, "unknown table field " + field);
    }
    return CloseBrace() || Err(error, "unterminated table");
  }

  bool ParseFeature(ManifestFeature* f, std::string* error) {
    while (SkipSpace(), pos_ < s_.size() && s_[pos_] != '}') {
      std::string field, v;
      if (!Ident(&field) || !Colon() || !Scalar(&v)) {
        return Err(error, "malformed feature entry");
      }
      if (field == "name") f->name = v;
      else if (field == "table") f->table = v;
      else if (field == "max_sequence_length") f->max_sequence_length = std::strtoll(v.c_str(), nullptr, 10);
      else return Err(error, "unknown feature field " + field);
    }
    return CloseBrace() || Err(error, "unterminated feature spec");
  }

  void SkipSpace() {
    while (pos_ < s_.size()) {
      if (std::isspace(static_cast<unsigned char>(s_[pos_]))) {
        ++pos_;
      } else if (s_[pos_] == '#') {
        while (pos_ < s_.size() && s_[pos_] != '\n') ++pos_;
      } else {
        break;
      }
    }
  }
  bool Ident(std::string* out) {
    SkipSpace();
    const size_t b = pos_;
    while (pos_ < s_.size() &&
           (std::isalnum(static_cast<unsigned char>(s_[pos_])) ||
            s_[pos_] == '_')) {
      ++pos_;
    }
    *out = s_.substr(b, pos_ - b);
    return !out->empty();
  }
  bool Colon() {
    SkipSpace();
    if (pos_ < s_.size() && s_[pos_] == ':') {
      ++pos_;
      return true;
    }
    return false;
  }
  bool OpenBrace() {
    SkipSpace();
    if (pos_ < s_.size() && s_[pos_] == ':') ++pos_;
    SkipSpace();
    if (pos_ < s_.size() && s_[pos_] == '{') {
      ++pos_;
      return true;
    }
    return false;
  }
  bool CloseBrace() {
    SkipSpace();
    if (pos_ < s_.size() && s_[pos_] == '}') {
      ++pos_;
      return true;
    }
    return false;
  }
  bool Scalar(std::string* out) {
    SkipSpace();
    if (pos_ >= s_.size()) return false;
    const char q = s_[pos_];
    if (q == '"' || q == '\'') {
      ++pos_;
      std::string v;
      while (pos_ < s_.size() && s_[pos_] != q) {
        if (s_[pos_] == '\\' && pos_ + 1 < s_.size()) ++pos_;
        v.push_back(s_[pos_++]);
      }
      if (pos_ >= s_.size()) return false;
      ++pos_;
      *out = v;
      return true;
    }
    const size_t b = pos_;
    while (pos_ < s_.size() &&
           (std::isalnum(static_cast<unsigned char>(s_[pos_])) ||
            s_[pos_] == '_' || s_[pos_] == '-' || s_[pos_] == '+' ||
            s_[pos_] == '.')) {
      ++pos_;
    }
    *out = s_.substr(b, pos_ - b);
    return !out->empty();
  }
  static bool Err(std::string* error, const std::string& what) {
    *error = what;
    return false;
  }

  const std::string& s_;
  size_t pos_ = 0;
};

// A read-only memory map of an asset file; the descriptor stays open for
// pread uploads.
struct MappedFile {
  void* data = nullptr;
  size_t bytes = 0;
  int fd = -1;
  ~MappedFile() {
    if (data != nullptr && bytes > 0) munmap(data, bytes);
    if (fd >= 0) ::close(fd);
  }
  bool Open(const std::string& path, std::string* error) {
    const int fd = ::open(path.c_str(), O_RDONLY | O_CLOEXEC);
    if (fd < 0) {
      *error = std::string("could not open ") + path + ": " + strerror(errno);
      return false;
    }
    struct stat st;
    if (fstat(fd, &st) != 0) {
      *error = std::string("could not stat ") + path;
      ::close(fd);
      return false;
    }
    bytes = static_cast<size_t>(st.st_size);
    if (bytes > 0) {
      data = mmap(nullptr, bytes, PROT_READ, MAP_PRIVATE, fd, 0);
      if (data == MAP_FAILED) {
        data = nullptr;
        *error = std::string("could not map ") + path;
        ::close(fd);
        return false;
      }
    }
    this->fd = fd;
    return true;
  }
};

bool ReadFile(const std::string& path, std::string* out) {
  FILE* f = std::fopen(path.c_str(), "rb");
  if (f == nullptr) return false;
  char buf[65536];
  size_t n;
  out->clear();
  while ((n = std::fread(buf, 1, sizeof(buf), f)) > 0) out->append(buf, n);
  std::fclose(f);
  return true;
}

}  // namespace

namespace xse {
// xse_engine_add_table with upload options (csrc/xse_capi.cu); rows read
// from file `fd` at file_offset when fd >= 0.
int AddTable(xse_engine* engine, const xse_table_desc* desc,
             int64_t upload_chunk, int upload_threads, int fd,
             int64_t file_offset);
}  // namespace xse

// ---------------------------------------------------------------------------
struct xse_resource {
  int device = 0;
  xse_engine* engine = nullptr;
  std::mutex mu;
  std::unordered_map<std::string, int32_t> feature_to_embedding_dim;
  ~xse_resource() { xse_engine_destroy(engine); }
};

namespace {

int CombineFromManifest(const std::string& mode, const std::string& table,
                        int32_t* out) {
  if (mode == "COMBINE_MODE_UNSPECIFIED" || mode == "0") {
    return Fail(XSE_INVALID_ARGUMENT, "Unspecified combine mode for table: %s",
                table.c_str());
  }
  if (mode == "SUM" || mode == "1") *out = XSE_COMBINE_SUM;
  else if (mode == "MEAN" || mode == "2") *out = XSE_COMBINE_MEAN;
  else if (mode == "SQRT_N" || mode == "3") *out = XSE_COMBINE_SQRTN;
  else {
    return Fail(XSE_INVALID_ARGUMENT, "Unknown combine mode for table: %s",
                table.c_str());
  }
  return XSE_OK;
}

// LoadCpuEmbeddingEngine (cpu_embedding_resource.cc:97-225), with the
// placement and upload options of xse_load_options.
int LoadResource(xse_resource* res, const std::string& manifest_path,
                 const std::unordered_map<std::string, std::string>& tables,
                 const xse_load_options& opt) {
  std::string text;
  if (!ReadFile(manifest_path, &text)) {
    return Fail(XSE_NOT_FOUND, "Could not read manifest %s",
                manifest_path.c_str());
  }
  Manifest m;
  std::string perr;
  TextProtoReader reader(text);
  if (!reader.Parse(&m, &perr)) {
    return Fail(XSE_INVALID_ARGUMENT, "Could not parse manifest %s: %s",
                manifest_path.c_str(), perr.c_str());
  }
  std::unordered_map<std::string, int64_t> table_to_dim;
  std::unordered_map<std::string, bool> table_local;
  const bool sharded = opt.sharding != XSE_SHARD_NONE && opt.world > 1;
  int64_t table_index = -1;
  for (const ManifestTable& t : m.tables) {
    ++table_index;
    auto it = tables.find(t.name);
    if (it == tables.end()) {
      return Fail(XSE_NOT_FOUND, "Failed to find table asset: %s",
                  t.name.c_str());
    }
    if (t.vocab_size <= 0 || t.embedding_dim <= 0) {
      return Fail(XSE_INVALID_ARGUMENT,
                  "Table dimensions must be strictly positive. Got "
                  "vocab_size: %" PRId64 ", embedding_dim: %" PRId64,
                  t.vocab_size, t.embedding_dim);
    }
    table_to_dim[t.name] = t.embedding_dim;
    const bool local = !sharded || opt.sharding != XSE_SHARD_TABLEWISE ||
                       table_index % opt.world == opt.rank;
    table_local[t.name] = local;
    int32_t dtype = XSE_DT_F32;
    size_t elem = 4;
    if (t.data_type == "BFLOAT16") {
      dtype = XSE_DT_BF16;
      elem = 2;
    } else if (t.data_type == "INT8_ROWWISE") {
      dtype = XSE_DT_I8_ROWWISE;
      elem = 1;
    } else if (t.data_type != "FLOAT32") {
      return Fail(XSE_INVALID_ARGUMENT, "Unknown data type %s for table: %s",
                  t.data_type.c_str(), t.name.c_str());
    }
    const unsigned __int128 cells =
        static_cast<unsigned __int128>(t.vocab_size) * t.embedding_dim;
    if (cells > SIZE_MAX / 8) {
      return Fail(XSE_INVALID_ARGUMENT,
                  "Table dimensions too large, multiplication overflowed: "
                  "%" PRId64 " * %" PRId64,
                  t.vocab_size, t.embedding_dim);
    }
    size_t expected = static_cast<size_t>(cells) * elem;
    if (dtype == XSE_DT_I8_ROWWISE) expected += 8 * t.vocab_size;
    MappedFile file;
    std::string ferr;
    if (!file.Open(it->second, &ferr)) {
      return Fail(XSE_NOT_FOUND, "Failed to map table asset %s at %s: %s",
                  t.name.c_str(), it->second.c_str(), ferr.c_str());
    }
    if (file.bytes != expected) {
      return Fail(XSE_INVALID_ARGUMENT,
                  "Table asset size mismatch for %s. Expected %zu bytes, but "
                  "got %zu",
                  t.name.c_str(), expected, file.bytes);
    }
    int32_t combine = 0;
    int code = CombineFromManifest(t.combine_mode, t.name, &combine);
    if (code != XSE_OK) return code;
    if (!local) continue;  // another rank's table (table-wise)
    int64_t row_begin = 0, row_end = t.vocab_size;
    if (sharded && opt.sharding == XSE_SHARD_ROWWISE) {
      row_begin = t.vocab_size * opt.rank / opt.world;
      row_end = t.vocab_size * (opt.rank + 1) / opt.world;
    }
    xse_table_desc desc{};
    desc.name = t.name.c_str();
    desc.dtype = dtype;
    desc.combine = combine;
    desc.vocab = t.vocab_size;
    desc.dim = static_cast<int32_t>(t.embedding_dim);
    desc.placement = XSE_PLACE_COPY_FROM_HOST;
    desc.row_begin = row_begin;
    desc.row_end = row_end;
    const char* base = static_cast<const char*>(file.data);
    desc.rows = base + static_cast<size_t>(row_begin) * t.embedding_dim * elem;
    if (dtype == XSE_DT_I8_ROWWISE) {
      desc.scale = reinterpret_cast<const float*>(base + cells) + row_begin;
      desc.bias = reinterpret_cast<const float*>(base + cells +
                                                 4 * t.vocab_size) +
                  row_begin;
    }
    code = xse::AddTable(
        res->engine, &desc,
        opt.chunk_bytes == 0 ? xse::kDefaultUploadChunk : opt.chunk_bytes,
        opt.upload_threads > 0 ? opt.upload_threads
                               : xse::kDefaultUploadThreads,
        file.fd,
        static_cast<int64_t>(row_begin) * t.embedding_dim *
            static_cast<int64_t>(elem));
    if (code != XSE_OK) return FailFromEngine(code);
  }
  for (const ManifestFeature& f : m.features) {
    auto loc = table_local.find(f.table);
    if (loc == table_local.end() || loc->second) {
      int code = xse_engine_register_feature(
          res->engine, f.name.c_str(), f.table.c_str(),
          static_cast<int32_t>(f.max_sequence_length));
      if (code != XSE_OK) return FailFromEngine(code);
    }
    auto it = table_to_dim.find(f.table);
    if (it == table_to_dim.end()) {
      return Fail(XSE_NOT_FOUND, "Failed to find table %s for feature %s",
                  f.table.c_str(), f.name.c_str());
    }
    if (!res->feature_to_embedding_dim
             .emplace(f.name, static_cast<int32_t>(it->second))
             .second) {
      return Fail(XSE_ALREADY_EXISTS, "Duplicate feature name in manifest: %s",
                  f.name.c_str());
    }
  }
  return XSE_OK;
}

int EmbeddingDim(xse_resource* res, const std::string& feature, int32_t* dim) {
  std::lock_guard<std::mutex> lock(res->mu);
  auto it = res->feature_to_embedding_dim.find(feature);
  if (it == res->feature_to_embedding_dim.end()) {
    return Fail(XSE_NOT_FOUND, "Embedding dimension not found for feature: %s",
                feature.c_str());
  }
  *dim = it->second;
  return XSE_OK;
}

// One feature's lookup, prepared on the host.
struct Prepared {
  int64_t batch_size = 0;      // output rows
  const void* ids = nullptr;   // host
  int32_t ids_type = XSE_INDEX_I64;
  int64_t num_ids = 0;
  const int32_t* row_pointers = nullptr;  // host
  int64_t num_row_pointers = 0;
  const float* weights = nullptr;
  int64_t num_weights = 0;
  int32_t dim = 0;
  int64_t out_elems = 0;
  // Shape of the output host buffer (AllocateOutput,
  // cpu_embedding_lookup_transform.cc:61-70).
  int32_t out_rank = 2;
  int64_t out_dims[2] = {0, 0};
  // Dense [batch_size, dense_seq] ids (DenseCpuEmbeddingLookupTransform):
  // `ids` holds them as given; the CSR (pad filter, all-pad rule, row
  // pointers) is built on the device.
  bool device_csr = false;
  int64_t dense_seq = 0;
  int64_t pad_value = 0;
  // dense_lookup: row pointers b * valency are generated on the device.
  int64_t device_rp_valency = -1;
};

// Device buffers and the status block of one call in flight.
struct Staging {
  int device = 0;
  DeviceArena dev;
  xse_status* status = nullptr;
  int32_t status_capacity = 0;
  bool busy = false;
  ~Staging() {
    if (status != nullptr) xse_status_destroy(status);
  }
};

// The staging slots of one operator. Each call takes a free slot (the pool
// grows on demand), so calls from several threads on different streams run
// concurrently: one call's input copies overlap another's output copies.
struct StagingPool {
  int device = 0;
  std::mutex mu;
  std::vector<std::unique_ptr<Staging>> slots;

  Staging* Acquire() {
    std::lock_guard<std::mutex> lock(mu);
    for (auto& s : slots) {
      if (!s->busy) {
        s->busy = true;
        return s.get();
      }
    }
    slots.push_back(std::make_unique<Staging>());
    Staging* s = slots.back().get();
    s->device = device;
    s->dev.device = device;
    s->busy = true;
    return s;
  }
  void Release(Staging* s) {
    std::lock_guard<std::mutex> lock(mu);
    s->busy = false;
  }
};

class StagingLease {
 public:
  explicit StagingLease(StagingPool* pool) : pool_(pool), s_(pool->Acquire()) {}
  ~StagingLease() { pool_->Release(s_); }
  Staging* get() const { return s_; }

 private:
  StagingPool* pool_;
  Staging* s_;
};

// Stages every feature's inputs in one pinned buffer, copies them to the
// device in one transfer, runs the group and copies all outputs back in one
// transfer. On success fills `outputs`; on failure nothing is returned.
int RunGroup(xse_engine* engine, StagingPool* staging_pool,
             const std::vector<std::string>& features,
             std::vector<Prepared>& prep, xse_host_buffer* outputs,
             cudaStream_t stream) {
  const size_t n = prep.size();
  // Layout of the staged inputs, of the outputs and of device-only CSR
  // buffers (ids and scan scratch of dense features).
  std::vector<size_t> ids_at(n), rp_at(n), w_at(n), out_at(n), csr_at(n),
      scratch_at(n), scratch_bytes(n);
  size_t in_bytes = 0;
  for (size_t i = 0; i < n; ++i) {
    const Prepared& p = prep[i];
    ids_at[i] = in_bytes;
    in_bytes = AlignUp(in_bytes + p.num_ids * (p.ids_type == XSE_INDEX_I64 ? 8 : 4), 64);
    rp_at[i] = in_bytes;
    in_bytes = AlignUp(in_bytes + p.num_row_pointers * 4, 64);
    w_at[i] = in_bytes;
    in_bytes = AlignUp(in_bytes + p.num_weights * 4, 64);
  }
  size_t out_bytes = 0;
  for (size_t i = 0; i < n; ++i) {
    out_at[i] = out_bytes;
    out_bytes = AlignUp(out_bytes + prep[i].out_elems * 4, 256);
  }
  size_t csr_bytes = 0;
  for (size_t i = 0; i < n; ++i) {
    const Prepared& p = prep[i];
    if (!p.device_csr) continue;
    csr_at[i] = csr_bytes;
    csr_bytes = AlignUp(
        csr_bytes + p.batch_size * std::max<int64_t>(p.dense_seq, 1) * 8, 256);
    scratch_bytes[i] = xse::DenseCsrScratchBytes(p.batch_size);
    scratch_at[i] = csr_bytes;
    csr_bytes = AlignUp(csr_bytes + scratch_bytes[i], 256);
  }
  StagingLease lease(staging_pool);
  Staging* staging = lease.get();
  DeviceGuard guard(staging->device);
  int code = staging->dev.Reserve(AlignUp(in_bytes, 256) +
                                  AlignUp(out_bytes, 256) + csr_bytes + 64);
  if (code != XSE_OK) return code;
  if (staging->status_capacity < static_cast<int32_t>(n)) {
    if (staging->status != nullptr) xse_status_destroy(staging->status);
    staging->status = nullptr;
    staging->status_capacity = 0;
    code = xse_status_create(std::max<int32_t>(static_cast<int32_t>(n), 8),
                             &staging->status);
    if (code != XSE_OK) return FailFromEngine(code);
    staging->status_capacity = std::max<int32_t>(static_cast<int32_t>(n), 8);
  }
  PinnedPool& pool = PinnedPool::Get();
  PinnedBlock* in_block = pool.Acquire(std::max<size_t>(in_bytes, 64));
  PinnedBlock* out_block = pool.Acquire(std::max<size_t>(out_bytes, 64));
  if (in_block == nullptr || out_block == nullptr) {
    if (in_block) pool.Release(in_block);
    if (out_block) pool.Release(out_block);
    return Fail(XSE_RESOURCE_EXHAUSTED, "pinned staging allocation failed");
  }
  char* host_in = static_cast<char*>(in_block->ptr);
  char* dev_in = static_cast<char*>(staging->dev.ptr);
  char* dev_out = dev_in + AlignUp(in_bytes, 256);
  char* dev_csr = dev_out + AlignUp(out_bytes, 256);
  // Inputs already in pinned memory go straight to the device; the others
  // are gathered into the pinned staging block and sent in one transfer.
  // Small calls (a serving request of a few hundred examples) gather every
  // input, pinned or not, and get their dense_lookup row pointers written
  // by the host: one transfer instead of a DMA per buffer and a launch per
  // feature. That pays while the host copy (about 64 KiB per transfer or
  // launch saved, at a few microseconds each) costs less than what it
  // saves; a call of one or two large buffers sends them directly.
  constexpr size_t kGatherAllBytes = static_cast<size_t>(1) << 20;
  constexpr size_t kGatherBytesPerSaving = static_cast<size_t>(64) << 10;
  size_t savings = 0;
  for (size_t i = 0; i < n; ++i) {
    const Prepared& p = prep[i];
    savings += (p.num_ids > 0) + (p.num_weights > 0) +
               (p.row_pointers != nullptr ||
                (!p.device_csr && p.device_rp_valency >= 0));
  }
  const bool gather_all =
      in_bytes <= std::min(kGatherAllBytes,
                           kGatherBytesPerSaving * (savings > 0 ? savings - 1 : 0));
  cudaError_t e = cudaSuccess;
  size_t lo = SIZE_MAX, hi = 0;
  auto stage = [&](const void* src, size_t at, size_t bytes) {
    if (bytes == 0 || e != cudaSuccess) return;
    if (!gather_all && IsPinned(src)) {
      e = cudaMemcpyAsync(dev_in + at, src, bytes, cudaMemcpyHostToDevice,
                          stream);
    } else {
      std::memcpy(host_in + at, src, bytes);
      lo = std::min(lo, at);
      hi = std::max(hi, at + bytes);
    }
  };
  std::vector<bool> host_rp(n, false);
  for (size_t i = 0; i < n; ++i) {
    const Prepared& p = prep[i];
    stage(p.ids, ids_at[i], p.num_ids * (p.ids_type == XSE_INDEX_I64 ? 8 : 4));
    if (p.row_pointers != nullptr) {
      stage(p.row_pointers, rp_at[i], p.num_row_pointers * 4);
    } else if (gather_all && !p.device_csr && p.device_rp_valency >= 0) {
      // dense_lookup row pointers b * valency (int32 range checked when the
      // call was prepared).
      int32_t* rp = reinterpret_cast<int32_t*>(host_in + rp_at[i]);
      for (int64_t b = 0; b <= p.batch_size; ++b) {
        rp[b] = static_cast<int32_t>(b * p.device_rp_valency);
      }
      lo = std::min(lo, rp_at[i]);
      hi = std::max(hi, rp_at[i] + static_cast<size_t>(p.batch_size + 1) * 4);
      host_rp[i] = true;
    }
    stage(p.weights, w_at[i], p.num_weights * 4);
  }
  if (e == cudaSuccess && hi > lo) {
    e = cudaMemcpyAsync(dev_in + lo, host_in + lo, hi - lo,
                        cudaMemcpyHostToDevice, stream);
  }
  // Row pointers (and dense features' CSR ids) built on the device.
  for (size_t i = 0; i < n && e == cudaSuccess; ++i) {
    const Prepared& p = prep[i];
    int32_t* rp = reinterpret_cast<int32_t*>(dev_in + rp_at[i]);
    if (p.device_csr) {
      e = xse::LaunchDenseToCsr(
          dev_in + ids_at[i], p.ids_type == XSE_INDEX_I64 ? 1 : 0,
          p.batch_size, p.dense_seq, p.pad_value, rp,
          reinterpret_cast<int64_t*>(dev_csr + csr_at[i]),
          dev_csr + scratch_at[i], scratch_bytes[i], stream);
    } else if (p.device_rp_valency >= 0 && !host_rp[i]) {
      e = xse::LaunchRowPointers(rp, p.batch_size, p.device_rp_valency,
                                 stream);
    }
  }
  std::vector<xse_bag_request> reqs(n);
  for (size_t i = 0; i < n; ++i) {
    const Prepared& p = prep[i];
    xse_bag_request& r = reqs[i];
    r.feature_name = features[i].c_str();
    r.ids = dev_in + ids_at[i];
    r.ids_type = p.ids_type;
    r.offsets_type = XSE_INDEX_I32;
    r.num_ids = p.num_ids;
    if (p.device_csr) {
      r.ids = dev_csr + csr_at[i];
      r.ids_type = XSE_INDEX_I64;
      r.num_ids = p.batch_size * std::max<int64_t>(p.dense_seq, 1);
    }
    r.offsets = dev_in + rp_at[i];
    r.num_offsets = p.num_row_pointers;
    r.weights = p.num_weights > 0
                    ? reinterpret_cast<const float*>(dev_in + w_at[i])
                    : nullptr;
    r.num_weights = p.num_weights;
    r.output = reinterpret_cast<float*>(dev_out + out_at[i]);
    r.output_stride = 0;
  }
  if (e == cudaSuccess) {
    // Asynchronous group on this call's own status block: the output copy
    // is queued right behind the pooling, and the status read-back (which
    // waits for the stream) decides whether the outputs are returned.
    code = xse_engine_execute_batch(engine, reqs.data(),
                                    static_cast<int32_t>(n), stream,
                                    XSE_EXEC_STRICT | XSE_EXEC_ASYNC,
                                    staging->status);
    if (code != XSE_OK) {
      cudaStreamSynchronize(stream);
      pool.Release(in_block);
      pool.Release(out_block);
      return FailFromEngine(code);
    }
    e = cudaMemcpyAsync(out_block->ptr, dev_out, out_bytes,
                        cudaMemcpyDeviceToHost, stream);
    code = xse_status_wait(staging->status, stream);
    if (code != XSE_OK) {
      cudaStreamSynchronize(stream);
      pool.Release(in_block);
      pool.Release(out_block);
      return FailFromEngine(code);
    }
  }
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  pool.Release(in_block);
  if (e != cudaSuccess) {
    pool.Release(out_block);
    return CudaFail(e, "operator transfer");
  }
  // Every output is a view into the one pinned block.
  for (size_t i = 0; i < n; ++i) {
    xse_host_buffer& o = outputs[i];
    std::memset(&o, 0, sizeof(o));
    o.data = static_cast<char*>(out_block->ptr) + out_at[i];
    o.dtype = XSE_HB_F32;
    o.rank = prep[i].out_rank;
    o.dims[0] = prep[i].out_dims[0];
    o.dims[1] = prep[i].out_dims[1];
    if (i == 0) {
      pool.Register(out_block, o.data);
    } else {
      pool.Retain(out_block, o.data);
    }
  }
  if (n == 0) pool.Release(out_block);
  return XSE_OK;
}

}  // namespace

// ---------------------------------------------------------------------------
struct xse_lookup_transform {
  xse_resource* resource = nullptr;
  std::vector<std::string> feature_names;
  std::vector<std::string> output_feature_names;
  bool dense_lookup = false;
  int64_t embedding_dim = 128;
  StagingPool staging;
};

struct xse_dense_lookup_transform {
  xse_resource* resource = nullptr;
  std::vector<std::string> feature_names;
  int64_t pad_value = 0;
  std::vector<std::string> output_feature_names;
  StagingPool staging;
};

namespace {

// ValidateLookupInputs (cpu_embedding_lookup_transform.cc:159-242).
int ValidateLookupInputs(const xse_host_buffer& ids,
                         const xse_host_buffer& rp,
                         const xse_host_buffer& w) {
  if (rp.rank == 0 && !Uninitialized(rp)) {
    return Fail(XSE_INVALID_ARGUMENT,
                "row_pointers HostBuffer must be at least 1D (got scalar).");
  }
  if (Uninitialized(ids)) {
    return Fail(XSE_INVALID_ARGUMENT, "ids HostBuffer is uninitialized.");
  }
  if (Uninitialized(rp)) {
    return Fail(XSE_INVALID_ARGUMENT,
                "row_pointers HostBuffer is uninitialized.");
  }
  if (Uninitialized(w)) {
    return Fail(XSE_INVALID_ARGUMENT, "weights HostBuffer is uninitialized.");
  }
  if (ids.dtype != XSE_HB_S64 && ids.dtype != XSE_HB_S32) {
    return Fail(XSE_INVALID_ARGUMENT, "Embedding IDs must be int32 or int64.");
  }
  if (rp.dtype != XSE_HB_S32) {
    return Fail(XSE_INVALID_ARGUMENT, "Row pointers must be int32 (kS32).");
  }
  if (NumElements(w) > 0 && w.dtype != XSE_HB_F32) {
    return Fail(XSE_INVALID_ARGUMENT, "Weights must be float32 (kF32).");
  }
  if (NumElements(ids) > 0 && ids.data == nullptr) {
    return Fail(XSE_INVALID_ARGUMENT, "ids HostBuffer base pointer is null.");
  }
  if (NumElements(rp) > 0 && rp.data == nullptr) {
    return Fail(XSE_INVALID_ARGUMENT,
                "row_pointers HostBuffer base pointer is null.");
  }
  if (NumElements(w) > 0 && w.data == nullptr) {
    return Fail(XSE_INVALID_ARGUMENT,
                "weights HostBuffer base pointer is null.");
  }
  const int64_t rp_size = NumElements(rp);
  if (rp_size < 2) {
    return Fail(XSE_INVALID_ARGUMENT,
                "Row pointers must have at least 2 elements.");
  }
  const int32_t* rp_ptr = static_cast<const int32_t*>(rp.data);
  if (rp_ptr[0] != 0) {
    return Fail(XSE_INVALID_ARGUMENT,
                "First element of row pointers must be 0.");
  }
  const int64_t ids_size = NumElements(ids);
  if (rp_ptr[rp_size - 1] < 0) {
    return Fail(XSE_INVALID_ARGUMENT,
                "Last element of row pointers must be non-negative.");
  }
  if (static_cast<int64_t>(rp_ptr[rp_size - 1]) != ids_size) {
    return Fail(XSE_INVALID_ARGUMENT,
                "Embedding ids size (%" PRId64
                ") does not match last element of row pointers (%d)",
                ids_size, rp_ptr[rp_size - 1]);
  }
  if (NumElements(w) > 0 && NumElements(w) != ids_size) {
    return Fail(XSE_INVALID_ARGUMENT,
                "Weights size (%" PRId64 ") does not match expected size "
                "(%" PRId64 ")",
                NumElements(w), ids_size);
  }
  return XSE_OK;
}

void SetOutputShape(Prepared* p) {
  // AllocateOutput: [batch, size/batch] when batch divides size, else [size].
  const int64_t size = p->out_elems;
  if (p->batch_size > 0 && size % p->batch_size == 0) {
    p->out_rank = 2;
    p->out_dims[0] = p->batch_size;
    p->out_dims[1] = size / p->batch_size;
  } else {
    p->out_rank = 1;
    p->out_dims[0] = size;
  }
}

int TableDim(xse_engine* engine, const std::string& feature, int32_t* dim) {
  char table[512];
  int32_t seq = 0;
  int code = xse_engine_feature_table(engine, feature.c_str(), table,
                                      sizeof(table), &seq);
  if (code != XSE_OK) return FailFromEngine(code);
  xse_table_info info;
  code = xse_engine_table_info(engine, table, &info);
  if (code != XSE_OK) return FailFromEngine(code);
  *dim = info.dim;
  return XSE_OK;
}

}  // namespace

extern "C" {

int xse_host_buffer_alloc(int32_t dtype, int32_t rank, const int64_t* dims,
                          xse_host_buffer* out) {
  if (out == nullptr || rank < 0 || rank > XSE_HB_MAX_RANK ||
      DtypeBytes(dtype) == 0 || (rank > 0 && dims == nullptr)) {
    return Fail(XSE_INVALID_ARGUMENT, "invalid host buffer request");
  }
  std::memset(out, 0, sizeof(*out));
  out->dtype = dtype;
  out->rank = rank;
  int64_t elems = 1;
  for (int32_t i = 0; i < rank; ++i) {
    if (dims[i] < 0) return Fail(XSE_INVALID_ARGUMENT, "negative dimension");
    out->dims[i] = dims[i];
    elems *= dims[i];
  }
  PinnedBlock* b =
      PinnedPool::Get().Acquire(std::max<size_t>(elems * DtypeBytes(dtype), 64));
  if (b == nullptr) {
    return Fail(XSE_RESOURCE_EXHAUSTED, "pinned host allocation failed");
  }
  out->data = b->ptr;
  PinnedPool::Get().Register(b, b->ptr);
  return XSE_OK;
}

void xse_host_buffer_free(xse_host_buffer* buffer) {
  if (buffer == nullptr || buffer->data == nullptr) return;
  PinnedPool::Get().ReleaseData(buffer->data);
  buffer->data = nullptr;
}

int xse_resource_create(int32_t device, xse_resource** out) {
  if (out == nullptr) return Fail(XSE_INVALID_ARGUMENT, "out is null");
  auto res = std::make_unique<xse_resource>();
  res->device = device;
  xse_engine_options opts{device, 0};
  const int code = xse_engine_create(&opts, &res->engine);
  if (code != XSE_OK) return FailFromEngine(code);
  *out = res.release();
  return XSE_OK;
}

int xse_resource_load(const char* const* asset_names,
                      const char* const* asset_paths, int32_t num_assets,
                      int32_t device, xse_resource** out) {
  return xse_resource_load_sharded(asset_names, asset_paths, num_assets,
                                   device, nullptr, out);
}

int xse_resource_load_sharded(const char* const* asset_names,
                              const char* const* asset_paths,
                              int32_t num_assets, int32_t device,
                              const xse_load_options* options,
                              xse_resource** out) {
  xse::TraceRange trace("xse.resource_load");
  xse_load_options opt{1, 0, XSE_SHARD_NONE, 0, 0};
  if (options != nullptr) opt = *options;
  if (opt.sharding < XSE_SHARD_NONE || opt.sharding > XSE_SHARD_ROWWISE ||
      (opt.sharding != XSE_SHARD_NONE &&
       (opt.world < 1 || opt.rank < 0 || opt.rank >= opt.world))) {
    return Fail(XSE_INVALID_ARGUMENT,
                "Bad placement: sharding %d, rank %d of %d.", opt.sharding,
                opt.rank, opt.world);
  }
  if (out == nullptr || num_assets < 0 ||
      (num_assets > 0 && (asset_names == nullptr || asset_paths == nullptr))) {
    return Fail(XSE_INVALID_ARGUMENT, "invalid asset list");
  }
  // CpuEmbeddingEngineResource::LoadImpl (cpu_embedding_resource.cc:
  // 215-239).
  std::string manifest;
  bool have_manifest = false;
  std::unordered_map<std::string, std::string> tables;
  for (int32_t i = 0; i < num_assets; ++i) {
    const std::string name = asset_names[i] ? asset_names[i] : "";
    if (name == "__jce_manifest__") {
      manifest = asset_paths[i] ? asset_paths[i] : "";
      have_manifest = true;
    } else if (!tables.emplace(name, asset_paths[i] ? asset_paths[i] : "")
                    .second) {
      return Fail(XSE_INVALID_ARGUMENT, "Duplicate table asset found for %s",
                  name.c_str());
    }
  }
  if (!have_manifest) {
    return Fail(XSE_NOT_FOUND, "Failed to find manifest asset in JCE Resource.");
  }
  xse_resource* res = nullptr;
  int code = xse_resource_create(device, &res);
  if (code != XSE_OK) return code;
  code = LoadResource(res, manifest, tables, opt);
  if (code != XSE_OK) {
    const std::string keep = xse_last_error();
    delete res;
    xse::SetLastErrorMessage(keep.c_str());
    return code;
  }
  *out = res;
  return XSE_OK;
}

void xse_resource_destroy(xse_resource* resource) { delete resource; }

xse_engine* xse_resource_engine(xse_resource* resource) {
  return resource == nullptr ? nullptr : resource->engine;
}

int xse_resource_embedding_dim(xse_resource* resource, const char* feature,
                               int32_t* dim) {
  if (resource == nullptr || feature == nullptr || dim == nullptr) {
    return Fail(XSE_INVALID_ARGUMENT, "arguments must be non-null");
  }
  return EmbeddingDim(resource, feature, dim);
}

int xse_resource_register_embedding_dim(xse_resource* resource,
                                        const char* feature, int32_t dim) {
  if (resource == nullptr || feature == nullptr) {
    return Fail(XSE_INVALID_ARGUMENT, "arguments must be non-null");
  }
  std::lock_guard<std::mutex> lock(resource->mu);
  resource->feature_to_embedding_dim[feature] = dim;
  return XSE_OK;
}

int xse_lookup_transform_create(xse_resource* resource,
                                const char* const* feature_names,
                                int32_t num_features, int32_t dense_lookup,
                                const char* const* output_feature_names,
                                int32_t num_output_names,
                                int64_t embedding_dim,
                                xse_lookup_transform** out) {
  // CpuEmbeddingLookupTransform::Create (cpu_embedding_lookup_transform.cc:
  // 87-151).
  if (out == nullptr) return Fail(XSE_INVALID_ARGUMENT, "out is null");
  if (resource == nullptr) {
    return Fail(XSE_INVALID_ARGUMENT,
                "CpuEmbeddingLookupTransform requires a non-null resource.");
  }
  if (num_features <= 0) {
    return Fail(XSE_INVALID_ARGUMENT,
                "CpuEmbeddingLookupTransform requires at least one feature "
                "name.");
  }
  if (num_output_names != 0 && num_output_names != num_features) {
    return Fail(XSE_INVALID_ARGUMENT,
                "CpuEmbeddingLookupTransform output_feature_names size must "
                "match feature_names size if provided.");
  }
  auto t = std::make_unique<xse_lookup_transform>();
  std::unordered_set<std::string> seen;
  for (int32_t i = 0; i < num_features; ++i) {
    const std::string name = feature_names[i] ? feature_names[i] : "";
    if (name.empty()) {
      return Fail(XSE_INVALID_ARGUMENT,
                  "CpuEmbeddingLookupTransform requires non-empty feature "
                  "names.");
    }
    if (!seen.insert(name).second) {
      return Fail(XSE_INVALID_ARGUMENT, "Duplicate feature name found: %s",
                  name.c_str());
    }
    t->feature_names.push_back(name);
  }
  std::unordered_set<std::string> seen_out;
  for (int32_t i = 0; i < num_output_names; ++i) {
    const std::string name =
        output_feature_names[i] ? output_feature_names[i] : "";
    if (name.empty()) {
      return Fail(XSE_INVALID_ARGUMENT,
                  "CpuEmbeddingLookupTransform requires non-empty output "
                  "feature names.");
    }
    if (!seen_out.insert(name).second) {
      return Fail(XSE_INVALID_ARGUMENT,
                  "Duplicate output feature name found: %s", name.c_str());
    }
    t->output_feature_names.push_back(name);
  }
  t->resource = resource;
  t->dense_lookup = dense_lookup != 0;
  t->embedding_dim = embedding_dim;
  t->staging.device = resource->device;
  *out = t.release();
  return XSE_OK;
}

void xse_lookup_transform_destroy(xse_lookup_transform* transform) {
  delete transform;
}

int xse_lookup_transform_run(xse_lookup_transform* t,
                             const xse_host_buffer* ids, int32_t num_ids,
                             const xse_host_buffer* row_pointers,
                             int32_t num_row_pointers,
                             const xse_host_buffer* weights,
                             int32_t num_weights, xse_host_buffer* outputs,
                             void* stream) {
  xse::TraceRange trace("xse.lookup_transform");
  // CpuEmbeddingLookupTransform::operator() (cpu_embedding_lookup_
  // transform.cc:244-356).
  if (t == nullptr || outputs == nullptr) {
    return Fail(XSE_INVALID_ARGUMENT, "transform and outputs must be non-null");
  }
  const int32_t nf = static_cast<int32_t>(t->feature_names.size());
  if (num_ids != nf) {
    return Fail(XSE_INVALID_ARGUMENT,
                "CpuEmbeddingLookupTransform expected %d ids buffers, but got "
                "%d.",
                nf, num_ids);
  }
  if (!t->dense_lookup) {
    if (num_row_pointers != nf) {
      return Fail(XSE_INVALID_ARGUMENT,
                  "CpuEmbeddingLookupTransform expected %d row_pointers "
                  "buffers, but got %d.",
                  nf, num_row_pointers);
    }
    if (num_weights != nf) {
      return Fail(XSE_INVALID_ARGUMENT,
                  "CpuEmbeddingLookupTransform expected %d weights buffers, "
                  "but got %d.",
                  nf, num_weights);
    }
  }
  std::vector<Prepared> prep(static_cast<size_t>(nf));
  for (int32_t i = 0; i < nf; ++i) {
    const xse_host_buffer& hb = ids[i];
    Prepared& p = prep[i];
    if (Uninitialized(hb) || hb.data == nullptr) {
      return Fail(XSE_INVALID_ARGUMENT,
                  "ids HostBuffer is uninitialized or null.");
    }
    if (hb.dtype == XSE_HB_S32) {
      p.ids_type = XSE_INDEX_I32;  // the kernels read int32 ids directly
    } else if (hb.dtype == XSE_HB_S64) {
      p.ids_type = XSE_INDEX_I64;
    } else {
      return Fail(XSE_INVALID_ARGUMENT,
                  "Embedding IDs must be int32 or int64.");
    }
    p.ids = hb.data;
    p.num_ids = NumElements(hb);
    if (t->dense_lookup) {
      if (hb.rank != 2) {
        return Fail(XSE_INVALID_ARGUMENT,
                    "Dense embedding IDs must be a 2D HostBuffer [batch_size, "
                    "valency].");
      }
      p.batch_size = hb.dims[0];
      const int64_t valency = hb.dims[1];
      if (p.batch_size < 0 || valency < 0) {
        return Fail(XSE_INVALID_ARGUMENT,
                    "Dense embedding IDs dimensions must be non-negative.");
      }
      if (p.batch_size >= INT32_MAX) {
        return Fail(XSE_INVALID_ARGUMENT,
                    "Batch size exceeds INT32_MAX bounds.");
      }
      if (p.batch_size > 0 && valency > INT32_MAX / p.batch_size) {
        return Fail(XSE_INVALID_ARGUMENT,
                    "Batch volume (batch_size * valency) exceeds INT32_MAX "
                    "bounds.");
      }
      // Row pointers b * valency, generated on the device (by the host for
      // calls small enough to go in one transfer).
      p.device_rp_valency = valency;
      p.row_pointers = nullptr;
      p.num_row_pointers = p.batch_size + 1;
    } else {
      const int code =
          ValidateLookupInputs(hb, row_pointers[i], weights[i]);
      if (code != XSE_OK) return code;
      const xse_host_buffer& rp = row_pointers[i];
      p.batch_size = NumElements(rp) > 0 ? rp.dims[0] - 1 : 0;
      p.row_pointers = static_cast<const int32_t*>(rp.data);
      p.num_row_pointers = NumElements(rp);
      p.weights = static_cast<const float*>(weights[i].data);
      p.num_weights = NumElements(weights[i]);
    }
  }
  xse_engine* engine = t->resource->engine;
  for (int32_t i = 0; i < nf; ++i) {
    Prepared& p = prep[i];
    int32_t dim = 0;
    // ExecuteBatch resolves the features; an unknown one fails there.
    if (TableDim(engine, t->feature_names[i], &dim) != XSE_OK) {
      dim = 0;
    }
    p.dim = dim;
    p.out_elems = std::max<int64_t>(p.num_row_pointers - 1, 0) * dim;
    SetOutputShape(&p);
  }
  return RunGroup(engine, &t->staging, t->feature_names, prep, outputs,
                  static_cast<cudaStream_t>(stream));
}

int xse_dense_lookup_transform_create(xse_resource* resource,
                                      const char* const* feature_names,
                                      int32_t num_features, int64_t pad_value,
                                      const char* const* output_feature_names,
                                      int32_t num_output_names,
                                      xse_dense_lookup_transform** out) {
  // DenseCpuEmbeddingLookupTransform::Create (dense_cpu_embedding_lookup_
  // transform.cc:76-99).
  if (out == nullptr) return Fail(XSE_INVALID_ARGUMENT, "out is null");
  if (resource == nullptr) {
    return Fail(XSE_INVALID_ARGUMENT,
                "DenseCpuEmbeddingLookupTransform requires a non-null "
                "resource.");
  }
  if (num_features <= 0) {
    return Fail(XSE_INVALID_ARGUMENT,
                "DenseCpuEmbeddingLookupTransform requires at least one "
                "feature name.");
  }
  auto t = std::make_unique<xse_dense_lookup_transform>();
  for (int32_t i = 0; i < num_features; ++i) {
    const std::string name = feature_names[i] ? feature_names[i] : "";
    if (name.empty()) {
      return Fail(XSE_INVALID_ARGUMENT,
                  "DenseCpuEmbeddingLookupTransform requires non-empty "
                  "feature names.");
    }
    t->feature_names.push_back(name);
  }
  for (int32_t i = 0; i < num_output_names; ++i) {
    t->output_feature_names.push_back(
        output_feature_names[i] ? output_feature_names[i] : "");
  }
  t->resource = resource;
  t->pad_value = pad_value;
  t->staging.device = resource->device;
  *out = t.release();
  return XSE_OK;
}

void xse_dense_lookup_transform_destroy(xse_dense_lookup_transform* t) {
  delete t;
}

int xse_dense_lookup_transform_run(xse_dense_lookup_transform* t,
                                   const xse_host_buffer* dense_ids,
                                   int32_t num_inputs,
                                   xse_host_buffer* outputs, void* stream) {
  xse::TraceRange trace("xse.dense_lookup_transform");
  // DenseCpuEmbeddingLookupTransform::operator() (dense_cpu_embedding_
  // lookup_transform.cc:148-268).
  if (t == nullptr || outputs == nullptr) {
    return Fail(XSE_INVALID_ARGUMENT, "transform and outputs must be non-null");
  }
  const int32_t nf = static_cast<int32_t>(t->feature_names.size());
  if (num_inputs != nf) {
    return Fail(XSE_INVALID_ARGUMENT,
                "DenseCpuEmbeddingLookupTransform expected %d inputs, got %d",
                nf, num_inputs);
  }
  std::vector<Prepared> prep(static_cast<size_t>(nf));
  for (int32_t f = 0; f < nf; ++f) {
    const xse_host_buffer& d = dense_ids[f];
    const char* fname = t->feature_names[f].c_str();
    if (d.rank <= 0) {
      return Fail(XSE_INVALID_ARGUMENT,
                  "dense_ids for feature %s must have rank >= 1.", fname);
    }
    const int64_t num_elements = NumElements(d);
    if (num_elements > 0 && d.data == nullptr) {
      return Fail(XSE_INVALID_ARGUMENT,
                  "dense_ids base pointer for feature %s is null with "
                  "%" PRId64 " elements.",
                  fname, num_elements);
    }
    if (num_elements > INT32_MAX) {
      return Fail(XSE_INVALID_ARGUMENT,
                  "dense_ids for feature %s exceeds INT32_MAX elements: "
                  "%" PRId64,
                  fname, num_elements);
    }
    const int64_t batch = d.dims[0];
    if (batch > INT32_MAX) {
      return Fail(XSE_INVALID_ARGUMENT,
                  "batch_size for feature %s exceeds INT32_MAX: %" PRId64,
                  fname, batch);
    }
    const int64_t seq = batch > 0 ? num_elements / batch : 0;
    if (d.dtype != XSE_HB_S64 && d.dtype != XSE_HB_S32) {
      return Fail(XSE_INVALID_ARGUMENT,
                  "dense_ids for feature %s must be kS64 or kS32, got kind: "
                  "%d",
                  fname, d.dtype);
    }
    // Keep non-pad ids; an all-pad row keeps one pad id
    // (dense_cpu_embedding_lookup_transform.cc:197-212): built on the device
    // from the dense buffer as given. Each row keeps at most max(seq, 1) ids,
    // so the row pointers stay within the checked element count (the
    // reference's int32 overflow check cannot fire past the checks above).
    if (batch * std::max<int64_t>(seq, 1) > INT32_MAX) {
      return Fail(XSE_INVALID_ARGUMENT,
                  "Row pointer offset overflowed int32_t.");
    }
    Prepared& p = prep[f];
    p.ids = d.data;
    p.ids_type = d.dtype == XSE_HB_S64 ? XSE_INDEX_I64 : XSE_INDEX_I32;
    p.num_ids = batch * seq;
    p.row_pointers = nullptr;
    p.num_row_pointers = batch + 1;
    p.batch_size = batch;
    p.device_csr = true;
    p.dense_seq = seq;
    p.pad_value = t->pad_value;
  }
  for (int32_t f = 0; f < nf; ++f) {
    int32_t dim = 0;
    int code = EmbeddingDim(t->resource, t->feature_names[f], &dim);
    if (code != XSE_OK) return code;
    Prepared& p = prep[f];
    p.dim = dim;
    p.out_elems = p.batch_size * dim;
    p.out_rank = 2;
    p.out_dims[0] = p.batch_size;
    p.out_dims[1] = dim;
  }
  return RunGroup(t->resource->engine, &t->staging, t->feature_names, prep,
                  outputs, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
