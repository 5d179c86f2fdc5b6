// GGUF v2/v3 container reader (mmap, zero-copy) and writer.
//
// Parity: crates/hawking-core/src/gguf.rs:218 (GgufFile::open), :231-319 (header, KV table,
// tensor index, data alignment from general.alignment, default 32), :543-578 (metadata kinds).
// The reader keeps the file mapped and hands out byte ranges; nothing is copied.
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <variant>
#include <vector>

namespace hk {

enum class GgufKind : uint32_t {
  U8 = 0, I8 = 1, U16 = 2, I16 = 3, U32 = 4, I32 = 5, F32 = 6, BOOL = 7, STRING = 8,
  ARRAY = 9, U64 = 10, I64 = 11, F64 = 12,
};

struct GgufValue;
using GgufArray = std::vector<GgufValue>;
struct GgufValue {
  GgufKind kind = GgufKind::U32;
  // Scalars are widened: integers into i (u64 values above INT64_MAX keep their bit pattern),
  // floats into f, strings into s, arrays into arr (elements share arr_kind).
  int64_t i = 0;
  double f = 0;
  std::string s;
  GgufKind arr_kind = GgufKind::U8;
  std::shared_ptr<GgufArray> arr;
};

struct GgufTensorInfo {
  std::string name;
  std::vector<uint64_t> dims;  // ggml order: dims[0] is the contiguous (row) length
  uint32_t type = 0;
  uint64_t offset = 0;         // relative to the data section
  uint64_t nbytes = 0;
  uint64_t n_elements() const;
};

class GgufFile {
 public:
  // Map and parse. Throws std::runtime_error with a precise reason on any malformed input.
  static std::unique_ptr<GgufFile> open(const std::string& path);
  // Parse an in-memory image (the caller keeps it alive).
  static std::unique_ptr<GgufFile> from_memory(const uint8_t* data, size_t size);
  ~GgufFile();

  uint32_t version() const { return version_; }
  uint64_t alignment() const { return alignment_; }
  uint64_t data_offset() const { return data_offset_; }
  const std::map<std::string, GgufValue>& metadata() const { return kv_; }
  const std::vector<GgufTensorInfo>& tensors() const { return tensors_; }
  const GgufTensorInfo* find(const std::string& name) const;
  const uint8_t* tensor_data(const GgufTensorInfo& t) const { return base_ + data_offset_ + t.offset; }
  const uint8_t* base() const { return base_; }
  size_t size() const { return size_; }
  const std::string& path() const { return path_; }

 private:
  void parse();
  std::string path_;
  const uint8_t* base_ = nullptr;
  size_t size_ = 0;
  bool mapped_ = false;
  uint32_t version_ = 0;
  uint64_t alignment_ = 32;
  uint64_t data_offset_ = 0;
  std::map<std::string, GgufValue> kv_;
  std::vector<GgufTensorInfo> tensors_;
  std::map<std::string, size_t> index_;
};

// Streaming writer: metadata and tensor table first, then payloads, each aligned.
class GgufWriter {
 public:
  explicit GgufWriter(uint64_t alignment = 32) : alignment_(alignment) {}
  void set(const std::string& key, const GgufValue& v) { kv_.emplace_back(key, v); }
  // dims in ggml order; data must hold type_nbytes(type, prod(dims)) bytes.
  void add_tensor(const std::string& name, const std::vector<uint64_t>& dims, uint32_t type,
                  const uint8_t* data, size_t nbytes);
  // Writes atomically (tmp file + rename).
  void write(const std::string& path) const;

 private:
  uint64_t alignment_;
  std::vector<std::pair<std::string, GgufValue>> kv_;
  struct Pending { GgufTensorInfo info; std::vector<uint8_t> bytes; };
  std::vector<Pending> tensors_;
};

}  // namespace hk
