// Gradient-norm pass that allocates no memory (slm_grad_norm_noalloc).
//
// Some callers cannot call cudaMalloc from the place where they need the
// gradient norm: code running while another framework's caching allocator owns
// the whole HBM budget, latency-critical loops in which cudaMalloc's implicit
// device-wide synchronisation would stall every other stream, and hosts that
// reserve all device memory up front and forbid later allocations.  For them
// this entry point computes the same fixed-tree f64 norm, clip scale and
// non-finite flag as the optimizer handle's norm pass, but its scratch (the
// per-chunk partials and two completion counters) lives in one file-scope
// device array of fixed size, loaded with the library.  The caller passes the
// gradients and a device pointer for the result; nothing is allocated.
//
// The array is shared by every call on a device and keeps the last call's
// contents, so each call first clears the counters that must start at zero;
// two calls whose work overlaps on the GPU (e.g. on two streams) race on it.
// Every GPU that loads the library holds the array (about 33 KB) until exit.
// Its device address is looked up once per device and cached; a
// cudaDeviceReset drops the module with the array, so a process that resets a
// device must not call this entry point on that device afterwards.
#include "handle.h"

#include <mutex>

namespace {

using namespace slmopt;

constexpr uint64_t kMaxElements = SLM_NOALLOC_MAX_ELEMENTS;
constexpr uint32_t kMaxChunks = uint32_t((kMaxElements + kChunkElems - 1) / kChunkElems);
constexpr uint32_t kHeaderDoubles = 32;  // 256 bytes: the two counters, padded
constexpr int kMaxDevices = 64;

// [0, 256 B): uint32 blocks_done, uint32 nonfinite; then kMaxChunks f64 partials.
static __device__ __align__(256) double g_noalloc_scratch[kHeaderDoubles + kMaxChunks];

// Device address of g_noalloc_scratch per device, looked up once per device.
std::mutex g_scratch_mutex;
void* g_scratch_addr[kMaxDevices] = {};

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ bool finite32(float x) {
  return (__float_as_uint(x) & 0x7f800000u) != 0x7f800000u;
}

__device__ __forceinline__ float grad_at(const float* g, uint64_t i) { return g[i]; }
__device__ __forceinline__ float grad_at(const uint16_t* g, uint64_t i) {
  return __uint_as_float(static_cast<uint32_t>(g[i]) << 16);
}

// The same reduction shape as the optimizer's norm pass: lane t of a 256-thread
// block takes its 8-element vectors at k*2048 + t*8 (k = 0..31); each vector's
// unscaled values are squared in f32 and summed pairwise in f32
// ((q0+q1)+(q2+q3))+((q4+q5)+(q6+q7)) (elements past n count as +0.0), and
// that sum is added to the lane's f64 accumulator; warps fold with offsets
// 16..1, the 8 warp sums with 4,2,1.
__device__ __forceinline__ double fold256(double v, double* warp_sums) {
  for (int off = 16; off >= 1; off >>= 1) v = __dadd_rn(v, __shfl_down_sync(kFull, v, off));
  if ((threadIdx.x & 31) == 0) warp_sums[threadIdx.x >> 5] = v;
  __syncthreads();
  double r = 0.0;
  if (threadIdx.x == 0) {
    double w[8];
    for (int i = 0; i < 8; ++i) w[i] = warp_sums[i];
    for (int off = 4; off >= 1; off >>= 1)
      for (int i = 0; i < off; ++i) w[i] = __dadd_rn(w[i], w[i + off]);
    r = w[0];
  }
  __syncthreads();
  return r;
}

template <typename GT>
__global__ void __launch_bounds__(kTreeThreads)
    noalloc_norm_kernel(const GT* __restrict__ g, uint64_t n, uint32_t n_chunks, float scale,
                        float max_norm, double* scratch, slm_norm_result* out) {
  __shared__ double warp_sums[kTreeThreads / 32];
  __shared__ uint32_t s_last;
  uint32_t* counters = reinterpret_cast<uint32_t*>(scratch);
  double* partials = scratch + kHeaderDoubles;
  bool bad = false;
  for (uint32_t c = blockIdx.x; c < n_chunks; c += gridDim.x) {
    const uint64_t base = uint64_t(c) * kChunkElems;
    double acc = 0.0;
    for (uint32_t k = 0; k < kChunkIters; ++k) {
      const uint64_t e0 = base + uint64_t(k) * (kTreeThreads * kVec) + uint64_t(threadIdx.x) * kVec;
      if (e0 >= n) break;
      float q[kVec];
      for (uint32_t j = 0; j < kVec; ++j) {
        const float u = e0 + j < n ? __fdiv_rn(grad_at(g, e0 + j), scale) : 0.0f;
        q[j] = __fmul_rn(u, u);
      }
      const float p = __fadd_rn(__fadd_rn(__fadd_rn(q[0], q[1]), __fadd_rn(q[2], q[3])),
                                __fadd_rn(__fadd_rn(q[4], q[5]), __fadd_rn(q[6], q[7])));
      acc = __dadd_rn(acc, static_cast<double>(p));
    }
    bad |= !isfinite(acc);
    const double total = fold256(acc, warp_sums);
    if (threadIdx.x == 0) partials[c] = total;
  }
  const int any_bad = __syncthreads_or(bad ? 1 : 0);
  if (threadIdx.x == 0) {
    if (any_bad) atomicOr(&counters[1], 1u);
    __threadfence();
    s_last = (atomicAdd(&counters[0], 1u) == gridDim.x - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (s_last == 0u) return;
  __threadfence();
  double v = 0.0;
  for (uint32_t c = threadIdx.x; c < n_chunks; c += kTreeThreads)
    v = __dadd_rn(v, __ldcg(partials + c));
  const double sum = fold256(v, warp_sums);
  if (threadIdx.x != 0) return;
  const uint32_t elem_bad = atomicExch(&counters[1], 0u) != 0u ? 1u : 0u;
  const float sumf = __double2float_rn(sum);
  float clip;
  if (!finite32(sumf)) {
    clip = 0.0f;
  } else if (sumf == 0.0f) {
    clip = 1.0f;
  } else {
    clip = __fdiv_rn(max_norm, __fsqrt_rn(sumf));
    clip = clip < 1.0f ? clip : 1.0f;
  }
  out->sum_squares = sum;
  out->grad_norm = __dsqrt_rn(sum);
  out->clip_scale = clip;
  out->nonfinite = (elem_bad || !finite32(sumf)) ? 1u : 0u;
  counters[0] = 0u;
  __threadfence();
}

}  // namespace

extern "C" int slm_grad_norm_noalloc(const void* grads, int dtype, uint64_t n, float loss_scale,
                                     float max_grad_norm, slm_norm_result* out_device,
                                     void* stream) {
  if (!grads || !out_device) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL argument");
  if (dtype != SLM_DTYPE_F32 && dtype != SLM_DTYPE_BF16)
    return fail(SLM_ERR_INVALID_ARGUMENT, "unknown gradient dtype");
  // A misaligned access would fault the caller's context; refuse it here.
  const uintptr_t esize = dtype == SLM_DTYPE_F32 ? 4u : 2u;
  if (reinterpret_cast<uintptr_t>(grads) % esize != 0)
    return fail(SLM_ERR_INVALID_ARGUMENT, "gradients must be aligned to their element size");
  if (reinterpret_cast<uintptr_t>(out_device) % alignof(slm_norm_result) != 0)
    return fail(SLM_ERR_INVALID_ARGUMENT, "out_device must be 8-byte aligned");
  if (n == 0) return fail(SLM_ERR_INVALID_ARGUMENT, "no gradient elements");
  if (n > kMaxElements)
    return fail(SLM_ERR_SIZE_LIMIT,
                "slm_grad_norm_noalloc handles at most SLM_NOALLOC_MAX_ELEMENTS (268,435,456) "
                "gradient elements; use an optimizer handle's norm pass for more");
  if (!(loss_scale > 0.0f) || !finite_f32(loss_scale) || !(max_grad_norm > 0.0f) ||
      !finite_f32(max_grad_norm))
    return fail(SLM_ERR_INVALID_ARGUMENT, "loss scale and max norm must be positive and finite");
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return fail(SLM_ERR_NO_DEVICE, "no current CUDA device");
  if (dev < 0 || dev >= kMaxDevices) return fail(SLM_ERR_INVALID_ARGUMENT, "device ordinal too large");
  void* scratch = nullptr;
  {
    // First call on this device: look up the array's device address while the
    // device is current (the host-side name is only a stand-in for it).
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_addr[dev]) {
      void* p = nullptr;
      const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
      if (e != cudaSuccess)
        return fail(SLM_ERR_CUDA, std::string("cudaGetSymbolAddress: ") + cudaGetErrorString(e));
      g_scratch_addr[dev] = p;
    }
    scratch = g_scratch_addr[dev];
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  // The counters must start at zero; the partials are written before they are read.
  cudaError_t e = cudaMemsetAsync(scratch, 0, kHeaderDoubles * sizeof(double), s);
  if (e != cudaSuccess)
    return fail(SLM_ERR_CUDA, std::string("clearing the scratch counters: ") + cudaGetErrorString(e));
  const uint32_t chunks = uint32_t((n + kChunkElems - 1) / kChunkElems);
  if (dtype == SLM_DTYPE_F32)
    noalloc_norm_kernel<float><<<chunks, kTreeThreads, 0, s>>>(
        static_cast<const float*>(grads), n, chunks, loss_scale, max_grad_norm,
        static_cast<double*>(scratch), out_device);
  else
    noalloc_norm_kernel<uint16_t><<<chunks, kTreeThreads, 0, s>>>(
        static_cast<const uint16_t*>(grads), n, chunks, loss_scale, max_grad_norm,
        static_cast<double*>(scratch), out_device);
  e = cudaGetLastError();
  if (e != cudaSuccess)
    return fail(SLM_ERR_CUDA, std::string("norm kernel launch: ") + cudaGetErrorString(e));
  return SLM_OK;
}
