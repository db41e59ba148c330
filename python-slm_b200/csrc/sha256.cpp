// SHA-256 (FIPS 180-4).  Portable compression function plus, where the host
// CPU reports the SHA extensions (CPUID leaf 7, EBX bit 29), the x86 SHA-NI
// instruction sequence from Intel's published "Intel SHA Extensions" white
// paper (2013), which hashes the ~1.9 GB optimizer state several times faster.
#include "sha256.h"

#include <cpuid.h>
#include <immintrin.h>

#include <cstring>

namespace slmopt {
namespace {

constexpr uint32_t kK[64] = {
    0x428a2f98u, 0x71374491u, 0xb5c0fbcfu, 0xe9b5dba5u, 0x3956c25bu, 0x59f111f1u, 0x923f82a4u,
    0xab1c5ed5u, 0xd807aa98u, 0x12835b01u, 0x243185beu, 0x550c7dc3u, 0x72be5d74u, 0x80deb1feu,
    0x9bdc06a7u, 0xc19bf174u, 0xe49b69c1u, 0xefbe4786u, 0x0fc19dc6u, 0x240ca1ccu, 0x2de92c6fu,
    0x4a7484aau, 0x5cb0a9dcu, 0x76f988dau, 0x983e5152u, 0xa831c66du, 0xb00327c8u, 0xbf597fc7u,
    0xc6e00bf3u, 0xd5a79147u, 0x06ca6351u, 0x14292967u, 0x27b70a85u, 0x2e1b2138u, 0x4d2c6dfcu,
    0x53380d13u, 0x650a7354u, 0x766a0abbu, 0x81c2c92eu, 0x92722c85u, 0xa2bfe8a1u, 0xa81a664bu,
    0xc24b8b70u, 0xc76c51a3u, 0xd192e819u, 0xd6990624u, 0xf40e3585u, 0x106aa070u, 0x19a4c116u,
    0x1e376c08u, 0x2748774cu, 0x34b0bcb5u, 0x391c0cb3u, 0x4ed8aa4au, 0x5b9cca4fu, 0x682e6ff3u,
    0x748f82eeu, 0x78a5636fu, 0x84c87814u, 0x8cc70208u, 0x90befffau, 0xa4506cebu, 0xbef9a3f7u,
    0xc67178f2u};

inline uint32_t rotr(uint32_t x, int n) { return (x >> n) | (x << (32 - n)); }

void compress_portable(uint32_t h[8], const uint8_t* p, size_t blocks) {
  for (; blocks; --blocks, p += 64) {
    uint32_t w[64];
    for (int i = 0; i < 16; ++i)
      w[i] = (uint32_t(p[4 * i]) << 24) | (uint32_t(p[4 * i + 1]) << 16) |
             (uint32_t(p[4 * i + 2]) << 8) | uint32_t(p[4 * i + 3]);
    for (int i = 16; i < 64; ++i) {
      const uint32_t s0 = rotr(w[i - 15], 7) ^ rotr(w[i - 15], 18) ^ (w[i - 15] >> 3);
      const uint32_t s1 = rotr(w[i - 2], 17) ^ rotr(w[i - 2], 19) ^ (w[i - 2] >> 10);
      w[i] = w[i - 16] + s0 + w[i - 7] + s1;
    }
    uint32_t a = h[0], b = h[1], c = h[2], d = h[3], e = h[4], f = h[5], g = h[6], k = h[7];
    for (int i = 0; i < 64; ++i) {
      const uint32_t t1 = k + (rotr(e, 6) ^ rotr(e, 11) ^ rotr(e, 25)) + ((e & f) ^ (~e & g)) +
                          kK[i] + w[i];
      const uint32_t t2 = (rotr(a, 2) ^ rotr(a, 13) ^ rotr(a, 22)) + ((a & b) ^ (a & c) ^ (b & c));
      k = g;
      g = f;
      f = e;
      e = d + t1;
      d = c;
      c = b;
      b = a;
      a = t1 + t2;
    }
    h[0] += a;
    h[1] += b;
    h[2] += c;
    h[3] += d;
    h[4] += e;
    h[5] += f;
    h[6] += g;
    h[7] += k;
  }
}

// Four rounds with the SHA-NI instructions: sha256rnds2 performs two rounds on
// the (ABEF, CDGH) state halves; the message-schedule words come from
// sha256msg1/sha256msg2 plus the alignr-based W[t-7] term.
__attribute__((target("sha,sse4.1"))) void compress_shani(uint32_t h[8], const uint8_t* p,
                                                          size_t blocks) {
  const __m128i byteswap = _mm_set_epi64x(0x0c0d0e0f08090a0bll, 0x0405060700010203ll);
  __m128i tmp = _mm_loadu_si128(reinterpret_cast<const __m128i*>(&h[0]));  // DCBA
  __m128i st1 = _mm_loadu_si128(reinterpret_cast<const __m128i*>(&h[4]));  // HGFE
  tmp = _mm_shuffle_epi32(tmp, 0xB1);                                       // CDAB
  st1 = _mm_shuffle_epi32(st1, 0x1B);                                       // EFGH
  __m128i st0 = _mm_alignr_epi8(tmp, st1, 8);                               // ABEF
  st1 = _mm_blend_epi16(st1, tmp, 0xF0);                                    // CDGH

  for (; blocks; --blocks, p += 64) {
    const __m128i save0 = st0, save1 = st1;
    __m128i msg[4];
    for (int i = 0; i < 4; ++i)
      msg[i] = _mm_shuffle_epi8(
          _mm_loadu_si128(reinterpret_cast<const __m128i*>(p + 16 * i)), byteswap);
    for (int r = 0; r < 16; ++r) {
      // Words 4r..4r+3 of the schedule are in msg[r % 4].
      __m128i wk = _mm_add_epi32(msg[r & 3],
                                 _mm_loadu_si128(reinterpret_cast<const __m128i*>(&kK[4 * r])));
      st1 = _mm_sha256rnds2_epu32(st1, st0, wk);
      wk = _mm_shuffle_epi32(wk, 0x0E);
      st0 = _mm_sha256rnds2_epu32(st0, st1, wk);
      if (r < 12) {
        // W[16+4r .. 19+4r] = sigma terms over the previous 16 words.
        __m128i next = _mm_sha256msg1_epu32(msg[r & 3], msg[(r + 1) & 3]);
        next = _mm_add_epi32(next, _mm_alignr_epi8(msg[(r + 3) & 3], msg[(r + 2) & 3], 4));
        msg[r & 3] = _mm_sha256msg2_epu32(next, msg[(r + 3) & 3]);
      }
    }
    st0 = _mm_add_epi32(st0, save0);
    st1 = _mm_add_epi32(st1, save1);
  }
  tmp = _mm_shuffle_epi32(st0, 0x1B);  // FEBA
  st1 = _mm_shuffle_epi32(st1, 0xB1);  // DCHG
  st0 = _mm_blend_epi16(tmp, st1, 0xF0);  // DCBA
  st1 = _mm_alignr_epi8(st1, tmp, 8);     // HGFE
  _mm_storeu_si128(reinterpret_cast<__m128i*>(&h[0]), st0);
  _mm_storeu_si128(reinterpret_cast<__m128i*>(&h[4]), st1);
}

bool cpu_has_shani() {
  unsigned a = 0, b = 0, c = 0, d = 0;
  if (!__get_cpuid_count(7, 0, &a, &b, &c, &d)) return false;
  const bool sha = (b >> 29) & 1u;
  unsigned a1 = 0, b1 = 0, c1 = 0, d1 = 0;
  if (!__get_cpuid(1, &a1, &b1, &c1, &d1)) return false;
  const bool sse41 = (c1 >> 19) & 1u;
  const bool ssse3 = (c1 >> 9) & 1u;
  return sha && sse41 && ssse3;
}

}  // namespace

Sha256::Sha256() : length_(0), used_(0), use_shani_(cpu_has_shani()) {
  static const uint32_t h0[8] = {0x6a09e667u, 0xbb67ae85u, 0x3c6ef372u, 0xa54ff53au,
                                 0x510e527fu, 0x9b05688cu, 0x1f83d9abu, 0x5be0cd19u};
  std::memcpy(h_, h0, sizeof(h0));
}

void Sha256::compress(const uint8_t* block, size_t blocks) {
  if (use_shani_)
    compress_shani(h_, block, blocks);
  else
    compress_portable(h_, block, blocks);
}

void Sha256::update(const void* data, size_t n) {
  const uint8_t* p = static_cast<const uint8_t*>(data);
  length_ += n;
  if (used_) {
    const size_t take = n < 64 - used_ ? n : 64 - used_;
    std::memcpy(buf_ + used_, p, take);
    used_ += take;
    p += take;
    n -= take;
    if (used_ == 64) {
      compress(buf_, 1);
      used_ = 0;
    }
  }
  if (n >= 64) {
    compress(p, n / 64);
    p += (n / 64) * 64;
    n %= 64;
  }
  if (n) {
    std::memcpy(buf_, p, n);
    used_ = n;
  }
}

void Sha256::final(uint8_t out[32]) {
  const uint64_t bits = length_ * 8u;
  uint8_t pad[72] = {0x80};
  const size_t pad_len = (used_ < 56) ? (56 - used_) : (120 - used_);
  update(pad, pad_len);
  uint8_t len_be[8];
  for (int i = 0; i < 8; ++i) len_be[i] = uint8_t(bits >> (56 - 8 * i));
  update(len_be, 8);
  for (int i = 0; i < 8; ++i) {
    out[4 * i] = uint8_t(h_[i] >> 24);
    out[4 * i + 1] = uint8_t(h_[i] >> 16);
    out[4 * i + 2] = uint8_t(h_[i] >> 8);
    out[4 * i + 3] = uint8_t(h_[i]);
  }
}

void Sha256::hex(const uint8_t digest[32], char out[65]) {
  static const char digits[] = "0123456789abcdef";
  for (int i = 0; i < 32; ++i) {
    out[2 * i] = digits[digest[i] >> 4];
    out[2 * i + 1] = digits[digest[i] & 15];
  }
  out[64] = 0;
}

}  // namespace slmopt
