// SHA-256 (FIPS 180-4), used for `.gravity` payload and body integrity digests.
#pragma once
#include <cstddef>
#include <cstdint>
#include <string>

namespace hk {

class Sha256 {
 public:
  Sha256();
  // portable = true: the plain C++ compression function even where the CPU has SHA extensions
  // (cross-check in the tests).
  explicit Sha256(bool portable) : Sha256() { portable_ = portable; }
  void update(const void* data, size_t n);
  void final(uint8_t out[32]);
  std::string hex();  // finalises
  static std::string hex_of(const void* data, size_t n);

 private:
  void block(const uint8_t* p);
  void blocks(const uint8_t* p, size_t n);
  bool portable_ = false;
  uint32_t h_[8];
  uint8_t buf_[64];
  size_t blen_ = 0;
  uint64_t total_ = 0;
};

}  // namespace hk
