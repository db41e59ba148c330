// Host-side copy of pageable gradients into the pinned staging ring.
#pragma once

#include <cstddef>

namespace slmopt {
// Copies n bytes from src to dst (no overlap).  Large copies use 32-byte
// non-temporal stores where the CPU has AVX2: the destination is a pinned
// slot that only the copy engine reads next, so filling it through the cache
// would first read every destination line (read-for-ownership) and then
// evict it again; streaming stores skip both.  Ends with a store fence, so
// the bytes are visible to the copy engine once the caller publishes them.
void stream_copy(void* dst, const void* src, size_t n);
}  // namespace slmopt
