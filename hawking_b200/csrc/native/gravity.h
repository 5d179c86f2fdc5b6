// `.gravity` packed-artifact container: single shards and multi-shard directories.
//
// Shard layout (little endian): b"GRAVITY\0" | u32 format_version (<= 1) | u64 header_len |
// canonical-JSON header | body. The header holds schema "hawking.gravity.shard_header.v1",
// model / architecture / tokenizer / compression / shard / gguf_metadata objects,
// integrity {body_sha256, tensor_count} and tensors [{name, codec, offset, bytes, sha256, shape,
// elements}] with offsets relative to the body; payloads are concatenated with no gaps.
// A directory holds model.gravity.index.json ({weight_map, tensor_dtypes, shard_sha256,
// architecture, ...}) and model-*.gravity shards.
//
// Parity: crates/hawking-core/src/artifact.rs:114-446 (open, read_tensor, parse_prefix_header,
// plan_shard, commit_shard, verify), crates/hawking-core/src/gravity.rs:877-990 (index),
// crates/hawking-core/src/gguf.rs:479-492 (codec -> ggml type mapping).
#pragma once
#include <cstdint>
#include <map>
#include <memory>
#include <string>
#include <vector>

#include "json.h"

namespace hk {

struct GravityTensor {
  std::string name;
  std::string codec;
  uint64_t offset = 0;   // relative to the body
  uint64_t bytes = 0;
  std::string sha256;
  std::vector<uint64_t> shape;
  uint64_t elements = 0;
  Json extra;            // the full descriptor object (codec-specific fields included)
};

class GravityShard {
 public:
  static std::unique_ptr<GravityShard> open(const std::string& path);
  ~GravityShard();
  const Json& header() const { return header_; }
  uint32_t format_version() const { return version_; }
  uint64_t body_offset() const { return body_off_; }
  const std::vector<GravityTensor>& tensors() const { return tensors_; }
  const GravityTensor* find(const std::string& name) const;
  const uint8_t* data(const GravityTensor& t) const { return base_ + body_off_ + t.offset; }
  const std::string& path() const { return path_; }
  size_t size() const { return size_; }
  // Full integrity audit: contiguity (no gaps/overlaps/trailing bytes), per-tensor and body
  // sha256, claimed packed/complete bits-per-weight. Returns a JSON report with "ok".
  Json verify() const;
  // Verify one tensor's payload digest (admission check before first use).
  bool verify_tensor(const std::string& name) const;

 private:
  std::string path_;
  const uint8_t* base_ = nullptr;
  size_t size_ = 0;
  uint32_t version_ = 0;
  uint64_t body_off_ = 0;
  Json header_;
  std::vector<GravityTensor> tensors_;
  std::map<std::string, size_t> index_;
};

// Writer: collects payloads, then writes the shard atomically (tmp + rename).
class GravityWriter {
 public:
  // meta may carry model / architecture / tokenizer / compression / shard / gguf_metadata.
  explicit GravityWriter(Json meta = Json::object()) : meta_(std::move(meta)) {}
  // descriptor: a JSON object with at least "name" (codec / shape / elements / extra fields kept).
  void add(Json descriptor, const uint8_t* data, size_t nbytes);
  // Returns the header actually written.
  Json write(const std::string& path) const;

 private:
  Json meta_;
  std::vector<std::pair<Json, std::vector<uint8_t>>> items_;
};

// ggml type id for a gravity codec string ("native.f16" -> F16, "ggml.q4_k" -> Q4_K, ...), -1 if
// the codec is not a plain ggml block format.
int gravity_codec_to_ggml(const std::string& codec);

}  // namespace hk
