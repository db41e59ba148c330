#include "hostcopy.h"

#include <cstdint>
#include <cstring>

#if defined(__x86_64__)
#include <immintrin.h>
#endif

#ifndef SLM_STREAM_COPY
#define SLM_STREAM_COPY 1  // 0: plain memcpy
#endif

namespace slmopt {

#if defined(__x86_64__)
__attribute__((target("avx2"))) static void stream_copy_avx2(uint8_t* d, const uint8_t* s,
                                                              size_t n) {
  const size_t head = (32u - (reinterpret_cast<uintptr_t>(d) & 31u)) & 31u;
  std::memcpy(d, s, head);
  d += head;
  s += head;
  n -= head;
  const size_t blocks = n / 128u;
  for (size_t b = 0; b < blocks; ++b, d += 128, s += 128) {
    const __m256i x0 = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(s));
    const __m256i x1 = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(s + 32));
    const __m256i x2 = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(s + 64));
    const __m256i x3 = _mm256_loadu_si256(reinterpret_cast<const __m256i*>(s + 96));
    _mm256_stream_si256(reinterpret_cast<__m256i*>(d), x0);
    _mm256_stream_si256(reinterpret_cast<__m256i*>(d + 32), x1);
    _mm256_stream_si256(reinterpret_cast<__m256i*>(d + 64), x2);
    _mm256_stream_si256(reinterpret_cast<__m256i*>(d + 96), x3);
  }
  std::memcpy(d, s, n % 128u);
}
#endif

void stream_copy(void* dst, const void* src, size_t n) {
#if defined(__x86_64__)
  if (SLM_STREAM_COPY && n >= (size_t(1) << 16) && __builtin_cpu_supports("avx2")) {
    stream_copy_avx2(static_cast<uint8_t*>(dst), static_cast<const uint8_t*>(src), n);
    _mm_sfence();
    return;
  }
#endif
  std::memcpy(dst, src, n);
}

}  // namespace slmopt
