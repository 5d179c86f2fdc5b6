// SHA-256 (FIPS 180-4), used for `.gravity` payload and body integrity digests.
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>

namespace hk {

class Sha256 {
 public:
  Sha256();
  void update(const void* data, size_t n);
  void final(uint8_t out[32]);
  std::string hex();  // finalises
  static std::string hex_of(const void* data, size_t n);

 private:
  void block(const uint8_t* p);
  uint32_t h_[8];
  uint8_t buf_[64];
  size_t blen_ = 0;
  uint64_t total_ = 0;
};

}  // namespace hk
