// SHA-256 (FIPS 180-4) for the optimizer-state identity of
// src/train/trainer.rs:297-320.  Host code; streaming interface.
#pragma once

#include <cstddef>
#include <cstdint>

namespace slmopt {

class Sha256 {
 public:
  Sha256();
  void update(const void* data, size_t n);
  void final(uint8_t out[32]);
  static void hex(const uint8_t digest[32], char out[65]);

 private:
  void compress(const uint8_t* block, size_t blocks);
  uint32_t h_[8];
  uint64_t length_;
  uint8_t buf_[64];
  size_t used_;
  bool use_shani_;
};

}  // namespace slmopt
