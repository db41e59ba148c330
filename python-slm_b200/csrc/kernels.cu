// Optimizer-step kernels for sm_100a.
//
// The step is pure streaming arithmetic (no contraction), so the kernels are
// bound by HBM bandwidth: 128-bit coalesced loads/stores, streaming cache
// hints for the state that is touched once, f64 shuffle trees for the norm.
//
//   norm_bulk_kernel         -- (default; norm_partials_kernel is the per-chunk
//                               form) reads the gradient once, unscales, forms
//                               one f64 partial per 65,536-element chunk with
//                               the fixed tree, flags non-finite values; its
//                               last block (atomic completion counter, no
//                               spinning) reduces the partials, computes the
//                               clip and the skip decision and advances the
//                               dynamic loss scaler.
//   adamw_update_bulk_kernel -- (default; adamw_update_kernel is the
//                               register-staged form) persistent grid over
//                               2,048-element tiles streamed through shared
//                               memory: unscale, clip, AdamW (fp32 master/m/v),
//                               bf16 weight copy (also to every peer in ZeRO-1).
//   accumulate*, zero1_*, peer_barrier_kernel, reference_clip_kernel,
//   export_f32_kernel, init / validate -- micro-batch sums, the ZeRO-1
//                               exchange, the strict drop-in's clip check, the
//                               f32 weight export and state set-up.
//
// Exactness: every f32 operation of the AdamW recurrence is an explicit
// round-to-nearest intrinsic (__fmul_rn, __fadd_rn, __fdiv_rn, __fsqrt_rn), so
// nothing is contracted into an FMA and the order is the reference's
// (src/model/oracle.rs:536-543); the file is also built with --fmad=false.
#include "slmopt_internal.h"

namespace slmopt {
namespace {

constexpr unsigned kFull = 0xffffffffu;

__device__ __forceinline__ bool finite_f32(float x) {
  return (__float_as_uint(x) & 0x7f800000u) != 0x7f800000u;
}

// Unscaling by s.  When s is a normal power of two whose reciprocal is also
// normal, x * (1/s) and x / s are the same exact real rounded once, so the
// multiply is bit-identical to the reference's true division; otherwise the
// IEEE division is used.
struct ScaleInfo {
  float s;
  float inv;
  bool mul;
};

__device__ __forceinline__ ScaleInfo decode_scale(float s) {
  const uint32_t b = __float_as_uint(s);
  const uint32_t e = (b >> 23) & 0xffu;
  ScaleInfo r;
  r.s = s;
  r.mul = ((b & 0x807fffffu) == 0u) && e >= 1u && e <= 253u;
  r.inv = __uint_as_float(((254u - e) & 0xffu) << 23);
  return r;
}

template <bool kMul>
__device__ __forceinline__ float unscale(float x, const ScaleInfo& sc) {
  if constexpr (kMul) {
    return __fmul_rn(x, sc.inv);
  } else {
    return __fdiv_rn(x, sc.s);
  }
}

__device__ __forceinline__ uint16_t bf16_rne_bits(float v) {
  // src/model/oracle.rs:300-304: bits + 0x7fff + lowest kept bit, keep the top half.
  const uint32_t b = __float_as_uint(v);
  return static_cast<uint16_t>((b + 0x7fffu + ((b >> 16) & 1u)) >> 16);
}

// ---- gradient loads (8 elements as f32) ------------------------------------
__device__ __forceinline__ void unpack_bf16x8(const uint4 r, float (&x)[8]) {
  x[0] = __uint_as_float(r.x << 16);
  x[1] = __uint_as_float(r.x & 0xffff0000u);
  x[2] = __uint_as_float(r.y << 16);
  x[3] = __uint_as_float(r.y & 0xffff0000u);
  x[4] = __uint_as_float(r.z << 16);
  x[5] = __uint_as_float(r.z & 0xffff0000u);
  x[6] = __uint_as_float(r.w << 16);
  x[7] = __uint_as_float(r.w & 0xffff0000u);
}

// Gradient load for the norm pass: default caching, so the tail of the gradient
// read here can still be in L2 when the update pass starts.
__device__ __forceinline__ void load_grad8(const float* __restrict__ g, uint64_t e0, uint64_t n,
                                           float (&x)[8]) {
  if (e0 + kVec <= n) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(g + e0));
    const float4 b = __ldg(reinterpret_cast<const float4*>(g + e0 + 4));
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
  } else {
#pragma unroll
    for (uint32_t j = 0; j < kVec; ++j) x[j] = (e0 + j < n) ? g[e0 + j] : 0.0f;
  }
}

__device__ __forceinline__ void load_grad8(const uint16_t* __restrict__ g, uint64_t e0,
                                           uint64_t n, float (&x)[8]) {
  if (e0 + kVec <= n) {
    unpack_bf16x8(__ldg(reinterpret_cast<const uint4*>(g + e0)), x);
  } else {
#pragma unroll
    for (uint32_t j = 0; j < kVec; ++j)
      x[j] = (e0 + j < n) ? __uint_as_float(static_cast<uint32_t>(g[e0 + j]) << 16) : 0.0f;
  }
}

__device__ __forceinline__ float ld_grad1(const float* __restrict__ g, uint64_t i) { return g[i]; }
__device__ __forceinline__ float ld_grad1(const uint16_t* __restrict__ g, uint64_t i) {
  return __uint_as_float(static_cast<uint32_t>(g[i]) << 16);
}

// ---- the fixed f64 tree -----------------------------------------------------
// Folds one double per thread of a 256-thread block; result valid in thread 0.
__device__ __forceinline__ double block_fold(double v, double* warp_sums) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v = __dadd_rn(v, __shfl_down_sync(kFull, v, off));
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  if (lane == 0) warp_sums[warp] = v;
  __syncthreads();
  double r = 0.0;
  if (threadIdx.x == 0) {
    double w[kTreeThreads / 32];
#pragma unroll
    for (int i = 0; i < int(kTreeThreads / 32); ++i) w[i] = warp_sums[i];
#pragma unroll
    for (int off = 4; off >= 1; off >>= 1) {
#pragma unroll
      for (int i = 0; i < off; ++i) w[i] = __dadd_rn(w[i], w[i + off]);
    }
    r = w[0];
  }
  __syncthreads();
  return r;
}

// Raw 8-element vectors, kept packed while a batch of loads is in flight.
template <typename GT>
struct RawVec;
template <>
struct RawVec<uint16_t> {
  uint4 r;
  __device__ __forceinline__ void load(const uint16_t* p) {
    r = __ldg(reinterpret_cast<const uint4*>(p));
  }
  __device__ __forceinline__ void unpack(float (&x)[8]) const { unpack_bf16x8(r, x); }
};
template <>
struct RawVec<float> {
  float4 a, b;
  __device__ __forceinline__ void load(const float* p) {
    a = __ldg(reinterpret_cast<const float4*>(p));
    b = __ldg(reinterpret_cast<const float4*>(p + 4));
  }
  __device__ __forceinline__ void unpack(float (&x)[8]) const {
    x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
    x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
  }
};

// One 8-element vector's contribution to a tree lane: the values are
// unscaled, squared in f32, the 8 squares added pairwise in f32
// ((q0+q1)+(q2+q3))+((q4+q5)+(q6+q7)), and that sum added to the lane's f64
// accumulator.  Every term is >= 0, so the relative error of the partial stays
// below ~2.4e-7 (4 f32 roundings); one f32 -> f64 conversion per 8 elements
// keeps the conversion pipe off the critical path.  A non-finite or
// overflowing value makes the sum non-finite.
template <bool kMul>
__device__ __forceinline__ double add_squares8(double acc, float (&x)[8], const ScaleInfo& sc) {
  float q[kVec];
#pragma unroll
  for (uint32_t j = 0; j < kVec; ++j) {
    const float u = unscale<kMul>(x[j], sc);
    q[j] = __fmul_rn(u, u);
  }
  const float p = __fadd_rn(__fadd_rn(__fadd_rn(q[0], q[1]), __fadd_rn(q[2], q[3])),
                            __fadd_rn(__fadd_rn(q[4], q[5]), __fadd_rn(q[6], q[7])));
  return __dadd_rn(acc, static_cast<double>(p));
}

template <typename GT, bool kMul>
__device__ __forceinline__ double chunk_thread_sum(const GT* __restrict__ g, uint64_t base,
                                                   uint64_t n, const ScaleInfo& sc) {
  // 128 bytes of gradient per thread in flight per batch.
  constexpr uint32_t kBatch = sizeof(GT) == 2 ? kNormBatch : kNormBatch / 2;
  double acc = 0.0;
  if (base + kChunkElems <= n) {
    // Whole chunk in range: kBatch unguarded loads go out together, then
    // their squares are added in the tree's element order.
    const GT* p = g + base + static_cast<uint64_t>(threadIdx.x) * kVec;
#pragma unroll 1
    for (uint32_t k0 = 0; k0 < kChunkIters; k0 += kBatch) {
      RawVec<GT> raw[kBatch];
#pragma unroll
      for (uint32_t b = 0; b < kBatch; ++b)
        raw[b].load(p + static_cast<uint64_t>(k0 + b) * (kTreeThreads * kVec));
#pragma unroll
      for (uint32_t b = 0; b < kBatch; ++b) {
        float x[kVec];
        raw[b].unpack(x);
        acc = add_squares8<kMul>(acc, x, sc);
      }
    }
    return acc;
  }
  for (uint32_t k = 0; k < kChunkIters; ++k) {
    const uint64_t e0 = base + static_cast<uint64_t>(k) * (kTreeThreads * kVec) +
                        static_cast<uint64_t>(threadIdx.x) * kVec;
    if (e0 >= n) break;  // the rest adds +0.0
    float x[kVec];
    load_grad8(g, e0, n, x);  // zeros past n square to +0.0
    acc = add_squares8<kMul>(acc, x, sc);
  }
  return acc;
}

// Chunk partials in global chunk order.  A single replica stores them densely;
// a ZeRO-1 group all-gathers per-rank blocks of per_rank partials followed by
// one flag slot, so chunk c lives at (c / per_rank) * stride + c % per_rank.
struct PartialsView {
  const double* p;
  uint32_t per_rank;
  uint32_t stride;
  __device__ __forceinline__ double operator()(uint32_t c) const {
    const uint32_t q = c / per_rank;
    return __ldcg(p + static_cast<uint64_t>(q) * stride + (c - q * per_rank));
  }
};

// Thread t's share of the finalize tree: partials t, t+256, ... added in that
// order; up to 8 of its loads go out together (2,065 partials at 135M: one
// round trip instead of 9).
__device__ __forceinline__ double finalize_lane_sum(const PartialsView& partials,
                                                   uint32_t total_chunks, uint32_t t) {
  double v = 0.0;
  for (uint32_t c0 = t; c0 < total_chunks; c0 += 8 * kTreeThreads) {
    double q[8];
#pragma unroll
    for (uint32_t b = 0; b < 8; ++b) {
      const uint32_t c = c0 + b * kTreeThreads;
      q[b] = c < total_chunks ? partials(c) : 0.0;
    }
#pragma unroll
    for (uint32_t b = 0; b < 8; ++b)
      if (c0 + b * kTreeThreads < total_chunks) v = __dadd_rn(v, q[b]);
  }
  return v;
}

// The step's decision from the reduced sum: clip, skip / reject, and the
// dynamic scaler's next state.
struct StepDecision {
  float clip;        // min(max_norm / sqrtf((float)sum), 1); 1 for a zero sum; 0 if non-finite
  float clip_apply;  // what the update multiplies by
  float next_scale;
  uint32_t good;
  uint32_t skipped, rejected;
  int32_t status;
};

__device__ __forceinline__ StepDecision decide_step(double sum, uint32_t nonfinite, float scale,
                                                    uint32_t good_in, const FinalizeParams& fp) {
  StepDecision d;
  const float sumf = __double2float_rn(sum);
  const bool norm_bad = !finite_f32(sumf);
  if (norm_bad) {
    d.clip = 0.0f;
  } else if (sumf == 0.0f) {
    d.clip = 1.0f;
  } else {
    d.clip = __fdiv_rn(fp.max_grad_norm, __fsqrt_rn(sumf));
    d.clip = d.clip < 1.0f ? d.clip : 1.0f;
  }
  d.clip_apply = fp.apply_clip ? d.clip : 1.0f;
  d.skipped = 0u;
  d.rejected = 0u;
  d.status = kStatusOk;
  d.next_scale = scale;
  d.good = fp.dynamic ? good_in : 0u;
  if (nonfinite || norm_bad) {
    d.skipped = 1u;
    if (fp.nonfinite_policy == 1)
      d.status = nonfinite ? kStatusGradientNonfinite : kStatusNormNonfinite;
    if (fp.dynamic) {
      d.next_scale = __fmul_rn(scale, 0.5f);
      d.good = 0u;
    }
  } else if (fp.min_clip_accept > 0.0f && d.clip < fp.min_clip_accept) {
    d.skipped = 1u;
    d.rejected = 1u;
    d.status = kStatusGradientInvalid;
  } else if (fp.dynamic) {
    d.good += 1u;
    if (d.good >= fp.growth_interval) {
      d.next_scale = __fmul_rn(scale, 2.0f);
      d.good = 0u;
    }
  }
  return d;
}

// Publishes a decision: the step record and, for a dynamic scale, the scaler.
// result_nonfinite is left alone: the update kernels raise it, and it is
// cleared before they start.
__device__ __forceinline__ void write_decision(const StepDecision& d, double sum, uint32_t nonfinite,
                                               float scale, DeviceStepState* st,
                                               DeviceScaler* scaler, const FinalizeParams& fp) {
  st->sum_squares = sum;
  st->grad_norm = __dsqrt_rn(sum);
  st->clip_scale = d.clip;
  st->clip_apply = d.clip_apply;
  st->loss_scale_used = scale;
  st->nonfinite = nonfinite;
  st->rejected = d.rejected;
  st->skipped = d.skipped;
  st->status = d.status;
  if (fp.dynamic) {
    scaler->scale = d.next_scale;
    scaler->good_steps = d.good;
  }
  st->next_loss_scale = d.next_scale;
  st->good_steps = d.good;
}

// Reduce the partials with the fixed tree, decide clip / skip, advance the
// scaler.  Called by one whole 256-thread block; `nonfinite` is read from
// thread 0 only.
__device__ __forceinline__ void finalize_block(const PartialsView& partials, uint32_t nonfinite,
                               DeviceStepState* st, DeviceScaler* scaler,
                               const FinalizeParams& fp, double* warp_sums) {
  const double sum = block_fold(finalize_lane_sum(partials, fp.total_chunks, threadIdx.x),
                                warp_sums);
  if (threadIdx.x != 0) return;
  const float scale = fp.dynamic ? scaler->scale : fp.static_scale;
  const StepDecision d =
      decide_step(sum, nonfinite, scale, fp.dynamic ? scaler->good_steps : 0u, fp);
  write_decision(d, sum, nonfinite, scale, st, scaler, fp);
  st->result_nonfinite = 0u;  // the update pass runs after this kernel
  st->blocks_done = 0u;
  __threadfence();
}

template <typename GT>
__global__ void __launch_bounds__(kTreeThreads, 3)
    norm_partials_kernel(const GT* __restrict__ g, uint64_t n, uint64_t chunk_begin,
                         uint32_t n_chunks, DeviceScaler* scaler, double* __restrict__ partials,
                         DeviceStepState* st, FinalizeParams fp) {
  __shared__ double warp_sums[kTreeThreads / 32];
  __shared__ uint32_t s_last;
  const ScaleInfo sc = decode_scale(fp.dynamic ? scaler->scale : fp.static_scale);
  bool bad = false;
  for (uint32_t c = blockIdx.x; c < n_chunks; c += gridDim.x) {
    const uint64_t chunk = chunk_begin + c;
    const uint64_t base = chunk * kChunkElems;
    // Squares are >= 0, so the partial is finite exactly when every unscaled
    // element and its f32 square is finite.
    const double acc = sc.mul ? chunk_thread_sum<GT, true>(g, base, n, sc)
                              : chunk_thread_sum<GT, false>(g, base, n, sc);
    bad |= !isfinite(acc);
    const double total = block_fold(acc, warp_sums);
    if (threadIdx.x == 0) partials[chunk] = total;
  }
  const int any_bad = __syncthreads_or(bad ? 1 : 0);
  if (threadIdx.x == 0) {
    if (any_bad) atomicOr(&st->nonfinite_accum, 1u);
    __threadfence();
    s_last = (atomicAdd(&st->blocks_done, 1u) == gridDim.x - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (s_last == 0u) return;
  __threadfence();
  const uint32_t nonfinite =
      threadIdx.x == 0 ? (atomicExch(&st->nonfinite_accum, 0u) != 0u ? 1u : 0u) : 0u;
  finalize_block(PartialsView{partials, fp.total_chunks, fp.total_chunks}, nonfinite, st, scaler,
                 fp, warp_sums);
}

// ---- micro-batch accumulation ----------------------------------------------------
// acc[i] = acc[i] + micro[i] in f32, one micro-batch after another -- the
// reference's host loop `total += value` (src/train/trainer.rs:865-877) moved
// onto the device.  `overwrite` starts a new update (acc = micro).
__device__ __forceinline__ void ld8f_stream(const float* __restrict__ p, float (&x)[8]) {
  const float4 a = __ldcs(reinterpret_cast<const float4*>(p));
  const float4 b = __ldcs(reinterpret_cast<const float4*>(p + 4));
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
  x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

template <typename GT>
__device__ __forceinline__ void accumulate8(float* __restrict__ acc, const GT* __restrict__ micro,
                                            uint64_t e0, uint64_t n, bool overwrite,
                                            float (&s)[8]) {
  if (e0 + kVec <= n) {
    float x[kVec];
    load_grad8(micro, e0, n, x);
    if (overwrite) {
#pragma unroll
      for (uint32_t j = 0; j < kVec; ++j) s[j] = x[j];
    } else {
      ld8f_stream(acc + e0, s);
#pragma unroll
      for (uint32_t j = 0; j < kVec; ++j) s[j] = __fadd_rn(s[j], x[j]);
    }
    __stcs(reinterpret_cast<float4*>(acc + e0), make_float4(s[0], s[1], s[2], s[3]));
    __stcs(reinterpret_cast<float4*>(acc + e0 + 4), make_float4(s[4], s[5], s[6], s[7]));
  } else {
#pragma unroll
    for (uint32_t j = 0; j < kVec; ++j) {
      const uint64_t i = e0 + j;
      if (i < n) {
        const float x = ld_grad1(micro, i);
        s[j] = overwrite ? x : __fadd_rn(acc[i], x);
        acc[i] = s[j];
      } else {
        s[j] = 0.0f;  // adds +0.0 to the partial
      }
    }
  }
}

template <typename GT>
__global__ void __launch_bounds__(256)
    accumulate_kernel(float* __restrict__ acc, const GT* __restrict__ micro, uint64_t n,
                      int overwrite) {
  const uint64_t vecs = (n + kVec - 1) / kVec;
  for (uint64_t v = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; v < vecs;
       v += uint64_t(gridDim.x) * blockDim.x) {
    float s[kVec];
    accumulate8(acc, micro, v * kVec, n, overwrite != 0, s);
  }
}

// The last micro-batch fused with the norm pass: each element is accumulated
// by the thread that owns it in the fixed tree, which then adds the square of
// the unscaled sum -- the same partials norm_partials_kernel<float> would form
// from the finished accumulator, without reading it again.
template <typename GT, bool kMul, bool kOverwrite>
__device__ __forceinline__ double accum_thread_sum(float* __restrict__ acc,
                                                   const GT* __restrict__ micro, uint64_t base,
                                                   uint64_t n, const ScaleInfo& sc) {
  double a = 0.0;
#pragma unroll 2
  for (uint32_t k = 0; k < kChunkIters; ++k) {
    const uint64_t e0 = base + static_cast<uint64_t>(k) * (kTreeThreads * kVec) +
                        static_cast<uint64_t>(threadIdx.x) * kVec;
    if (e0 >= n) break;
    float s[kVec];
    accumulate8(acc, micro, e0, n, kOverwrite, s);
    a = add_squares8<kMul>(a, s, sc);
  }
  return a;
}

template <typename GT>
__global__ void __launch_bounds__(kTreeThreads)
    accumulate_norm_kernel(float* __restrict__ acc, const GT* __restrict__ micro, uint64_t n,
                           int overwrite, uint32_t n_chunks, DeviceScaler* scaler,
                           double* __restrict__ partials, DeviceStepState* st,
                           FinalizeParams fp) {
  __shared__ double warp_sums[kTreeThreads / 32];
  __shared__ uint32_t s_last;
  const ScaleInfo sc = decode_scale(fp.dynamic ? scaler->scale : fp.static_scale);
  bool bad = false;
  for (uint32_t c = blockIdx.x; c < n_chunks; c += gridDim.x) {
    const uint64_t base = static_cast<uint64_t>(c) * kChunkElems;
    const double a =
        overwrite ? (sc.mul ? accum_thread_sum<GT, true, true>(acc, micro, base, n, sc)
                            : accum_thread_sum<GT, false, true>(acc, micro, base, n, sc))
                  : (sc.mul ? accum_thread_sum<GT, true, false>(acc, micro, base, n, sc)
                            : accum_thread_sum<GT, false, false>(acc, micro, base, n, sc));
    bad |= !isfinite(a);
    const double total = block_fold(a, warp_sums);
    if (threadIdx.x == 0) partials[c] = total;
  }
  const int any_bad = __syncthreads_or(bad ? 1 : 0);
  if (threadIdx.x == 0) {
    if (any_bad) atomicOr(&st->nonfinite_accum, 1u);
    __threadfence();
    s_last = (atomicAdd(&st->blocks_done, 1u) == gridDim.x - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (s_last == 0u) return;
  __threadfence();
  const uint32_t nonfinite =
      threadIdx.x == 0 ? (atomicExch(&st->nonfinite_accum, 0u) != 0u ? 1u : 0u) : 0u;
  finalize_block(PartialsView{partials, fp.total_chunks, fp.total_chunks}, nonfinite, st, scaler,
                 fp, warp_sums);
}

// ---- ZeRO-1 -----------------------------------------------------------------------
// After the all-to-all, recv holds `ranks` slices of this rank's shard (slice q
// from rank q, `stride` elements apart).  One pass sums them in rank order
// 0..N-1 in f32 (the reference's accumulation order, trainer.rs:865-877),
// stores the raw sums for the update pass, and forms the chunk partials of the
// unscaled sums with the same fixed tree as a single replica.  The last block
// appends the non-finite flag as slot n_chunks of the send buffer.
template <typename GT, bool kMul>
__device__ __forceinline__ double zero1_thread_sum(const GT* __restrict__ recv, uint32_t ranks,
                                                   uint64_t stride, uint64_t base, uint64_t n,
                                                   float* __restrict__ gsum,
                                                   const ScaleInfo& sc) {
  double acc = 0.0;
#pragma unroll 2
  for (uint32_t k = 0; k < kChunkIters; ++k) {
    const uint64_t e0 = base + static_cast<uint64_t>(k) * (kTreeThreads * kVec) +
                        static_cast<uint64_t>(threadIdx.x) * kVec;
    if (e0 >= n) break;
    float s[kVec];
    load_grad8(recv, e0, n, s);
    for (uint32_t q = 1; q < ranks; ++q) {
      float x[kVec];
      load_grad8(recv + static_cast<uint64_t>(q) * stride, e0, n, x);
#pragma unroll
      for (uint32_t j = 0; j < kVec; ++j) s[j] = __fadd_rn(s[j], x[j]);
    }
    if (e0 + kVec <= n) {
      __stcg(reinterpret_cast<float4*>(gsum + e0), make_float4(s[0], s[1], s[2], s[3]));
      __stcg(reinterpret_cast<float4*>(gsum + e0 + 4), make_float4(s[4], s[5], s[6], s[7]));
    } else {
      for (uint32_t j = 0; j < kVec && e0 + j < n; ++j) gsum[e0 + j] = s[j];
    }
    acc = add_squares8<kMul>(acc, s, sc);
  }
  return acc;
}

template <typename GT>
__global__ void __launch_bounds__(kTreeThreads)
    zero1_reduce_kernel(const GT* __restrict__ recv, uint32_t ranks, uint64_t stride,
                        uint64_t n_valid, uint32_t n_chunks, const DeviceScaler* scaler,
                        FinalizeParams fp, float* __restrict__ gsum, double* __restrict__ send,
                        DeviceStepState* st) {
  __shared__ double warp_sums[kTreeThreads / 32];
  __shared__ uint32_t s_last;
  const ScaleInfo sc = decode_scale(fp.dynamic ? scaler->scale : fp.static_scale);
  bool bad = false;
  for (uint32_t c = blockIdx.x; c < n_chunks; c += gridDim.x) {
    const uint64_t base = static_cast<uint64_t>(c) * kChunkElems;
    const double acc =
        sc.mul ? zero1_thread_sum<GT, true>(recv, ranks, stride, base, n_valid, gsum, sc)
               : zero1_thread_sum<GT, false>(recv, ranks, stride, base, n_valid, gsum, sc);
    bad |= !isfinite(acc);
    const double total = block_fold(acc, warp_sums);
    if (threadIdx.x == 0) send[c] = total;
  }
  const int any_bad = __syncthreads_or(bad ? 1 : 0);
  if (threadIdx.x == 0) {
    if (any_bad) atomicOr(&st->nonfinite_accum, 1u);
    __threadfence();
    s_last = (atomicAdd(&st->blocks_done, 1u) == gridDim.x - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (s_last == 0u || threadIdx.x != 0) return;
  __threadfence();
  send[n_chunks] = atomicExch(&st->nonfinite_accum, 0u) != 0u ? 1.0 : 0.0;
  st->blocks_done = 0u;
  __threadfence();
}

// Every rank reduces the all-gathered partials of all ranks in global chunk
// order, so the norm, clip and skip decision are bit-identical on all ranks
// and equal to a single replica's.
__global__ void __launch_bounds__(kTreeThreads)
    zero1_finalize_kernel(const double* __restrict__ gathered, uint32_t ranks,
                          uint32_t per_rank, DeviceScaler* scaler, DeviceStepState* st,
                          FinalizeParams fp) {
  __shared__ double warp_sums[kTreeThreads / 32];
  uint32_t nonfinite = 0u;
  if (threadIdx.x == 0)
    for (uint32_t q = 0; q < ranks; ++q)
      nonfinite |= gathered[static_cast<uint64_t>(q) * (per_rank + 1) + per_rank] != 0.0 ? 1u : 0u;
  finalize_block(PartialsView{gathered, per_rank, per_rank + 1}, nonfinite, st, scaler, fp,
                 warp_sums);
}

// ---- AdamW update -------------------------------------------------------------
__device__ __forceinline__ float adamw_elem(float th, float gv, float& m, float& v, float wd,
                                            const AdamwParams& p, bool& bad) {
  const float m1 = __fadd_rn(__fmul_rn(p.beta1, m), __fmul_rn(p.omb1, gv));
  const float v1 = __fadd_rn(__fmul_rn(p.beta2, v), __fmul_rn(__fmul_rn(p.omb2, gv), gv));
  const float mh = __fdiv_rn(m1, p.bc1);
  const float vh = __fdiv_rn(v1, p.bc2);
  const float den = __fadd_rn(__fsqrt_rn(vh), p.eps);
  const float upd = __fadd_rn(__fdiv_rn(mh, den), __fmul_rn(wd, th));
  const float t1 = __fsub_rn(th, __fmul_rn(p.lr, upd));
  bad |= !(finite_f32(m1) && finite_f32(v1) && finite_f32(t1));
  m = m1;
  v = v1;
  return t1;
}

__device__ __forceinline__ void ld8_stream(const float* __restrict__ p, float (&x)[8]) {
  const float4 a = __ldcs(reinterpret_cast<const float4*>(p));
  const float4 b = __ldcs(reinterpret_cast<const float4*>(p + 4));
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
  x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}

[[maybe_unused]] __device__ __forceinline__ void st8_stream(float* __restrict__ p, const float (&x)[8]) {
  __stcs(reinterpret_cast<float4*>(p), make_float4(x[0], x[1], x[2], x[3]));
  __stcs(reinterpret_cast<float4*>(p + 4), make_float4(x[4], x[5], x[6], x[7]));
}

[[maybe_unused]] __device__ __forceinline__ void ld_grad8_stream(const float* __restrict__ g, float (&x)[8]) {
  ld8_stream(g, x);
}

[[maybe_unused]] __device__ __forceinline__ void ld_grad8_stream(const uint16_t* __restrict__ g, float (&x)[8]) {
  unpack_bf16x8(__ldcs(reinterpret_cast<const uint4*>(g)), x);
}


// Decay weight of global element e, scanning forward from tensor k.
__device__ __forceinline__ float decay_of(uint64_t e, uint32_t& k,
                                          const uint64_t* __restrict__ offsets,
                                          const uint8_t* __restrict__ decay,
                                          const AdamwParams& p) {
  while (e >= __ldg(offsets + k + 1)) ++k;
  return __ldg(decay + k) ? p.decay_weight : p.no_decay_weight;
}

template <typename GT, bool kMul, bool kPeers>
__device__ __forceinline__ bool update_loop(const GT* __restrict__ g, uint64_t n,
                                            uint64_t elem_base, float* __restrict__ master,
                                            float* __restrict__ mom, float* __restrict__ var,
                                            uint16_t* __restrict__ w16,
                                            const uint64_t* __restrict__ offsets,
                                            const uint8_t* __restrict__ decay,
                                            const uint32_t* __restrict__ tile_first,
                                            const AdamwParams& p, const ScaleInfo& sc,
                                            float clip, const PeerStores& ps) {
  bool bad = false;
  const uint64_t n_tiles = (n + kTileElems - 1) / kTileElems;
  for (uint64_t tile = blockIdx.x; tile < n_tiles; tile += gridDim.x) {
    const uint32_t first = __ldg(tile_first + tile);
    uint64_t i0[kUpdateUnroll];
    bool full[kUpdateUnroll];
    float gx[kUpdateUnroll][kVec], th[kUpdateUnroll][kVec], mm[kUpdateUnroll][kVec],
        vv[kUpdateUnroll][kVec];
    // Phase 1: issue every load of this tile before any arithmetic.
#pragma unroll
    for (uint32_t u = 0; u < kUpdateUnroll; ++u) {
      i0[u] = tile * kTileElems + u * (kUpdateThreads * kVec) +
              static_cast<uint64_t>(threadIdx.x) * kVec;
      full[u] = i0[u] + kVec <= n;
      if (full[u]) {
        ld_grad8_stream(g + i0[u], gx[u]);
        ld8_stream(master + i0[u], th[u]);
        ld8_stream(mom + i0[u], mm[u]);
        ld8_stream(var + i0[u], vv[u]);
      }
    }
    // Phase 2: arithmetic and stores.
#pragma unroll
    for (uint32_t u = 0; u < kUpdateUnroll; ++u) {
      uint32_t k = first;
      if (full[u]) {
        const uint64_t e0 = elem_base + i0[u];
        const float wd0 = decay_of(e0, k, offsets, decay, p);
        const bool uniform = e0 + kVec <= __ldg(offsets + k + 1);
        uint32_t bits[kVec];
#pragma unroll
        for (uint32_t j = 0; j < kVec; ++j) {
          const float wd = uniform ? wd0 : decay_of(e0 + j, k, offsets, decay, p);
          const float gv = __fmul_rn(unscale<kMul>(gx[u][j], sc), clip);
          th[u][j] = adamw_elem(th[u][j], gv, mm[u][j], vv[u][j], wd, p, bad);
          bits[j] = bf16_rne_bits(th[u][j]);
        }
        st8_stream(master + i0[u], th[u]);
        st8_stream(mom + i0[u], mm[u]);
        st8_stream(var + i0[u], vv[u]);
        uint4 packed;
        packed.x = bits[0] | (bits[1] << 16);
        packed.y = bits[2] | (bits[3] << 16);
        packed.z = bits[4] | (bits[5] << 16);
        packed.w = bits[6] | (bits[7] << 16);
        __stcs(reinterpret_cast<uint4*>(w16 + i0[u]), packed);
        if constexpr (kPeers) {
#pragma unroll
          for (uint32_t q = 0; q < uint32_t(kMaxRanks); ++q)
            if (q < ps.count) __stcs(reinterpret_cast<uint4*>(ps.w16[q] + i0[u]), packed);
        }
      } else if (i0[u] < n) {
        // Ragged tail: scalar accesses for the last < 8 elements.
        for (uint32_t j = 0; j < kVec && i0[u] + j < n; ++j) {
          const uint64_t i = i0[u] + j;
          const float wd = decay_of(elem_base + i, k, offsets, decay, p);
          const float gv = __fmul_rn(unscale<kMul>(ld_grad1(g, i), sc), clip);
          float m = mom[i], v = var[i];
          const float t1 = adamw_elem(master[i], gv, m, v, wd, p, bad);
          master[i] = t1;
          mom[i] = m;
          var[i] = v;
          w16[i] = bf16_rne_bits(t1);
          if constexpr (kPeers) {
#pragma unroll
            for (uint32_t q = 0; q < uint32_t(kMaxRanks); ++q)
              if (q < ps.count) ps.w16[q][i] = bf16_rne_bits(t1);
          }
        }
      }
    }
  }
  return bad;
}

template <typename GT, bool kPeers>
__global__ void __launch_bounds__(kUpdateThreads, kUpdateMinBlocks)
    adamw_update_kernel(const GT* __restrict__ g, uint64_t n, uint64_t elem_base,
                        float* __restrict__ master, float* __restrict__ mom,
                        float* __restrict__ var, uint16_t* __restrict__ w16,
                        const uint64_t* __restrict__ offsets, const uint8_t* __restrict__ decay,
                        const uint32_t* __restrict__ tile_first, AdamwParams p,
                        DeviceStepState* st, PeerStores ps) {
  // Written by the previous kernel on this stream; uniform for the grid.
  if (st->skipped || st->kernel_error) return;
  const ScaleInfo sc = decode_scale(st->loss_scale_used);
  const float clip = st->clip_apply;
  const bool bad =
      sc.mul ? update_loop<GT, true, kPeers>(g, n, elem_base, master, mom, var, w16, offsets,
                                             decay, tile_first, p, sc, clip, ps)
             : update_loop<GT, false, kPeers>(g, n, elem_base, master, mom, var, w16, offsets,
                                              decay, tile_first, p, sc, clip, ps);
  if (__any_sync(kFull, bad) && (threadIdx.x & 31) == 0) atomicOr(&st->result_nonfinite, 1u);
  if constexpr (kPeers) __threadfence_system();  // peer stores visible before the closing barrier
}

// ---- bulk-copy pipelined update (SLM_UPDATE_BULK=1) ---------------------------
// Register pressure caps the plain kernel at two resident blocks per SM, so
// only ~2 tiles of loads per SM are in flight.  Here a producer warp moves each
// 2,048-element tile of g / master / m / v from HBM into one of kBulkStages
// shared-memory stages with cp.async.bulk (completion counted in bytes on an
// mbarrier), and 8 consumer warps compute from shared memory and stream the
// results straight to global memory; in-flight bytes no longer cost registers.
// Consumer thread t owns elements [4t, 4t+4) and [1024+4t, 1024+4t+4) of a
// tile, so its shared-memory reads and its global stores are conflict-free and
// coalesced.  Every wait is bounded (a few seconds of %globaltimer); on expiry
// the kernel records kernel_error and leaves instead of hanging.
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Waits for the phase with the given parity; false after ~4 s.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0u && global_ns() - t0 > 4000000000ull) return false;
  }
}

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes,
                                          uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
          "r"(smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

template <typename GT>
struct BulkStage {
  static constexpr uint32_t kG = kBulkTile * sizeof(GT);
  static constexpr uint32_t kF = kBulkTile * 4;
  static constexpr uint32_t kBytes = kG + 3 * kF;
};

// Shared memory: kBulkStages stages, the full/empty mbarriers (one 128-byte
// slot), and on the peer path two bf16 staging tiles for the weight stores.
constexpr uint32_t kBarrierBytes = 128;
static_assert(2 * kBulkStages * sizeof(uint64_t) <= kBarrierBytes, "mbarrier slot too small");
constexpr uint32_t kStagingBytes = kBulkTile * 2;

template <typename GT, bool kPeers>
constexpr size_t bulk_smem_bytes() {
  return size_t(kBulkStages) * BulkStage<GT>::kBytes + kBarrierBytes +
         (kPeers ? 2 * kStagingBytes : 0);
}

// Bulk (TMA engine) store of `bytes` from shared to global memory, tracked in
// this thread's bulk async-group; dst, src and bytes are multiples of 16.
__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst),
               "r"(smem_u32(src)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void bulk_commit() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Every committed group of this thread has finished reading shared memory.
__device__ __forceinline__ void bulk_wait_read_all() {
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
// Every committed group of this thread has completed its writes.
__device__ __forceinline__ void bulk_wait_all() {
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
// Generic-proxy writes to shared memory become visible to the bulk engine.
__device__ __forceinline__ void fence_smem_to_async() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// AND of `ok` over the 256 consumer threads (named barrier 1; the producer
// warp never takes part).
__device__ __forceinline__ bool consumers_all(bool ok) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, %2, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(ok ? 1u : 0u), "n"(kBulkConsumers)
      : "memory");
  return r != 0;
}

__device__ __forceinline__ void lds4(const float* p, float (&x)[4]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
}

__device__ __forceinline__ void lds_grad4(const float* p, float (&x)[4]) { lds4(p, x); }
__device__ __forceinline__ void lds_grad4(const uint16_t* p, float (&x)[4]) {
  const uint2 r = *reinterpret_cast<const uint2*>(p);
  x[0] = __uint_as_float(r.x << 16);
  x[1] = __uint_as_float(r.x & 0xffff0000u);
  x[2] = __uint_as_float(r.y << 16);
  x[3] = __uint_as_float(r.y & 0xffff0000u);
}

// AdamW on 4 consecutive local elements starting at i (global elem_base + i)
// whose g / master / m / v are already in registers; streams master / m / v
// out and returns the 4 bf16 weights packed.
template <bool kMul>
__device__ __forceinline__ uint2 update4(uint64_t i, uint64_t elem_base, float (&gx)[4],
                                        float (&th)[4], float (&mm)[4], float (&vv)[4],
                                        float* __restrict__ master, float* __restrict__ mom,
                                        float* __restrict__ var,
                                        const uint64_t* __restrict__ offsets,
                                        const uint8_t* __restrict__ decay, uint32_t k,
                                        const AdamwParams& p, const ScaleInfo& sc, float clip,
                                        bool& bad) {
  const uint64_t e0 = elem_base + i;
  const float wd0 = decay_of(e0, k, offsets, decay, p);
  const bool uniform = e0 + 4 <= __ldg(offsets + k + 1);
  uint32_t bits[4];
#pragma unroll
  for (uint32_t j = 0; j < 4; ++j) {
    const float wd = uniform ? wd0 : decay_of(e0 + j, k, offsets, decay, p);
    const float gv = __fmul_rn(unscale<kMul>(gx[j], sc), clip);
    th[j] = adamw_elem(th[j], gv, mm[j], vv[j], wd, p, bad);
    bits[j] = bf16_rne_bits(th[j]);
  }
  __stcs(reinterpret_cast<float4*>(master + i), make_float4(th[0], th[1], th[2], th[3]));
  __stcs(reinterpret_cast<float4*>(mom + i), make_float4(mm[0], mm[1], mm[2], mm[3]));
  __stcs(reinterpret_cast<float4*>(var + i), make_float4(vv[0], vv[1], vv[2], vv[3]));
  return make_uint2(bits[0] | (bits[1] << 16), bits[2] | (bits[3] << 16));
}

// Peer path (kPeers): the tile's bf16 weights go through a shared-memory
// staging tile and leave as one 4 KB bulk store per destination (this rank's
// copy and every peer's), issued by consumer thread 0, so the consumer warps
// never wait on NVLink stores.  Staging tile i % 2 is rewritten two tiles
// later; thread 0 waits for every earlier store group to finish reading before
// the consumers' barrier of the tile in between, which makes that safe.  The
// barrier also ANDs the threads' wait outcomes so that all 256 leave together.
template <typename GT, bool kMul, bool kPeers>
__device__ __forceinline__ bool bulk_consume(uint8_t* smem, uint64_t* full_bar,
                                             uint64_t* empty_bar, uint8_t* staging,
                                             uint64_t n_full, uint64_t elem_base,
                                             float* __restrict__ master, float* __restrict__ mom,
                                             float* __restrict__ var, uint16_t* __restrict__ w16,
                                             const uint64_t* __restrict__ offsets,
                                             const uint8_t* __restrict__ decay,
                                             const uint32_t* __restrict__ tile_first,
                                             const AdamwParams& p, const ScaleInfo& sc,
                                             float clip, const PeerStores& ps, bool& bad) {
  using Stage = BulkStage<GT>;
  const uint32_t t = threadIdx.x;
  uint32_t i = 0;
  for (uint64_t tile = blockIdx.x; tile < n_full; tile += gridDim.x, ++i) {
    const uint32_t s = i % kBulkStages;
    const bool ready = mbar_wait(&full_bar[s], (i / kBulkStages) & 1u);
    if constexpr (!kPeers) {
      if (!ready) return false;
    }
    const uint64_t tile0 = tile * kBulkTile;
    uint16_t* stage_w16 = reinterpret_cast<uint16_t*>(staging + (i & 1u) * kStagingBytes);
    if (ready) {
      const uint8_t* base = smem + size_t(s) * Stage::kBytes;
      const GT* sg = reinterpret_cast<const GT*>(base);
      const float* sm = reinterpret_cast<const float*>(base + Stage::kG);
      const float* s1 = sm + kBulkTile;
      const float* s2 = s1 + kBulkTile;
      const uint32_t k = __ldg(tile_first + tile0 / kTileElems);
#pragma unroll
      for (uint32_t h = 0; h < 2; ++h) {
        const uint32_t o = h * (kBulkTile / 2) + 4 * t;
        float gx[4], th[4], mm[4], vv[4];
        lds_grad4(sg + o, gx);
        lds4(sm + o, th);
        lds4(s1 + o, mm);
        lds4(s2 + o, vv);
        const uint2 packed = update4<kMul>(tile0 + o, elem_base, gx, th, mm, vv, master, mom,
                                           var, offsets, decay, k, p, sc, clip, bad);
        if constexpr (kPeers)
          *reinterpret_cast<uint2*>(stage_w16 + o) = packed;
        else
          __stcs(reinterpret_cast<uint2*>(w16 + tile0 + o), packed);
      }
      __syncwarp();
      if ((t & 31) == 0) mbar_arrive(&empty_bar[s]);
    }
    if constexpr (kPeers) {
      fence_smem_to_async();
      if (t == 0) bulk_wait_read_all();  // staging tile (i + 1) % 2 is free again
      if (!consumers_all(ready)) return false;
      if (t == 0) {
        bulk_store(w16 + tile0, stage_w16, kStagingBytes);
#pragma unroll
        for (uint32_t q = 0; q < uint32_t(kMaxRanks); ++q)
          if (q < ps.count) bulk_store(ps.w16[q] + tile0, stage_w16, kStagingBytes);
        bulk_commit();
      }
    }
  }
  return true;
}

// Programmatic dependent launch: the norm pass lets the update grid launch
// while its own blocks are still running; the update's producer warps start
// streaming tiles at once (the norm pass writes none of g / master / m / v),
// and its consumers wait for the norm pass to complete before they read the
// step's decision.  Without the launch attribute (or after a kernel that does
// not trigger) the wait returns at once.
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

template <typename GT>
__global__ void __launch_bounds__(kBulkThreads)
    adamw_update_bulk_kernel(const GT* __restrict__ g, uint64_t n, uint64_t elem_base,
                             float* __restrict__ master, float* __restrict__ mom,
                             float* __restrict__ var, uint16_t* __restrict__ w16,
                             const uint64_t* __restrict__ offsets,
                             const uint8_t* __restrict__ decay,
                             const uint32_t* __restrict__ tile_first, AdamwParams p,
                             DeviceStepState* st) {
  using Stage = BulkStage<GT>;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ float s_scale, s_clip;
  __shared__ uint32_t s_go, s_stop;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + size_t(kBulkStages) * Stage::kBytes);
  uint64_t* empty_bar = full_bar + kBulkStages;
  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < kBulkStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kBulkConsumers / 32);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_stop = 0u;
  }
  __syncthreads();
  const uint64_t n_full = n / kBulkTile;
  const uint64_t mine = n_full > blockIdx.x ? (n_full - 1u - blockIdx.x) / gridDim.x + 1u : 0u;
  bool ok = true;
  bool bad = false;
  uint32_t i = 0;  // producer: tiles issued
  if (threadIdx.x >= kBulkConsumers) {
    // Producer warp: lane 0 keeps kBulkStages tiles in flight; it stops once
    // the consumers have found that this step does not update.
    if (threadIdx.x == kBulkConsumers) {
      for (uint64_t tile = blockIdx.x; tile < n_full; tile += gridDim.x, ++i) {
        const uint32_t s = i % kBulkStages;
        if (i >= kBulkStages) {
          if (!mbar_wait(&empty_bar[s], ((i / kBulkStages) - 1u) & 1u)) {
            ok = false;
            break;
          }
          if (*reinterpret_cast<volatile uint32_t*>(&s_stop)) break;
        }
        uint8_t* base = smem + size_t(s) * Stage::kBytes;
        const uint64_t e0 = tile * kBulkTile;
        mbar_arrive_expect_tx(&full_bar[s], Stage::kBytes);
        bulk_load(base, g + e0, Stage::kG, &full_bar[s]);
        bulk_load(base + Stage::kG, master + e0, Stage::kF, &full_bar[s]);
        bulk_load(base + Stage::kG + Stage::kF, mom + e0, Stage::kF, &full_bar[s]);
        bulk_load(base + Stage::kG + 2 * Stage::kF, var + e0, Stage::kF, &full_bar[s]);
      }
    }
  } else {
    const uint32_t t = threadIdx.x;
    pdl_wait();  // the norm pass (decision, loss scale) is complete and visible
    if (t == 0) {
      s_go = (st->skipped == 0u && st->kernel_error == 0u) ? 1u : 0u;
      s_scale = st->loss_scale_used;
      s_clip = st->clip_apply;
      if (!s_go) s_stop = 1u;
    }
    asm volatile("bar.sync 1, %0;" ::"n"(kBulkConsumers) : "memory");
    if (!s_go) {
      // No update: take back the tiles the producer already started (each
      // stage's first use), so no copy lands after the block exits.
      const uint32_t started = mine < kBulkStages ? uint32_t(mine) : kBulkStages;
      for (uint32_t u = 0; u < started; ++u) {
        ok &= mbar_wait(&full_bar[u], 0u);
        __syncwarp();
        if ((t & 31) == 0) mbar_arrive(&empty_bar[u]);
      }
    } else {
      const ScaleInfo sc = decode_scale(s_scale);
      const float clip = s_clip;
      const PeerStores none{};
      ok = sc.mul ? bulk_consume<GT, true, false>(smem, full_bar, empty_bar, nullptr, n_full,
                                                  elem_base, master, mom, var, w16, offsets,
                                                  decay, tile_first, p, sc, clip, none, bad)
                  : bulk_consume<GT, false, false>(smem, full_bar, empty_bar, nullptr, n_full,
                                                   elem_base, master, mom, var, w16, offsets,
                                                   decay, tile_first, p, sc, clip, none, bad);
      // Ragged tail after the last whole tile: element by element, block 0.
      if (blockIdx.x == 0) {
        for (uint64_t e = n_full * kBulkTile + t; e < n; e += kBulkConsumers) {
          uint32_t k = __ldg(tile_first + e / kTileElems);
          const float wd = decay_of(elem_base + e, k, offsets, decay, p);
          const float gv = __fmul_rn(
              sc.mul ? unscale<true>(ld_grad1(g, e), sc) : unscale<false>(ld_grad1(g, e), sc),
              clip);
          float m = mom[e], v = var[e];
          const float t1 = adamw_elem(master[e], gv, m, v, wd, p, bad);
          master[e] = t1;
          mom[e] = m;
          var[e] = v;
          w16[e] = bf16_rne_bits(t1);
        }
      }
    }
  }
  // After an expired wait the producer waits (bounded) for the tiles it still
  // has in flight, so no copy lands in shared memory after the block exits.
  if (__syncthreads_or(ok ? 0 : 1) && threadIdx.x == kBulkConsumers)
    for (uint32_t u = i > kBulkStages ? i - kBulkStages : 0u; u < i; ++u)
      mbar_wait(&full_bar[u % kBulkStages], (u / kBulkStages) & 1u);
  if (!ok) atomicOr(&st->kernel_error, 1u);
  if (bad) atomicOr(&st->result_nonfinite, 1u);
}

// ---- bulk-copy norm pass (SLM_NORM_BULK=1) ------------------------------------
// The same fixed tree as norm_partials_kernel, fed through shared memory: a
// persistent grid (2 blocks per SM) walks its whole chunks in order, and
// thread 0 keeps kNormStages 16 KB bulk copies in flight across chunk
// boundaries, so no per-block launch, no per-thread load batches and no tail
// wave.  A stage holds kIters consecutive 2,048-element tree rows; thread t
// reads its 8 elements of each row (16 or 32 contiguous bytes per thread,
// conflict-free) in row order, so each lane's f64 accumulation order is the
// tree's.  The ragged last chunk (if any) is summed from global memory by the
// last block.  Waits are bounded; on expiry every thread of the block leaves
// (block-wide vote) after thread 0 has waited, again bounded, for the copies it
// still has in flight, and kernel_error records it.
template <typename GT>
struct NormStage {
  static constexpr uint32_t kElems = kNormStageBytes / sizeof(GT);
  static constexpr uint32_t kIters = kElems / (kTreeThreads * kVec);  // tree rows per stage
  static constexpr uint32_t kPerChunk = kChunkIters / kIters;
  static_assert(kIters * kTreeThreads * kVec == kElems, "stage must hold whole rows");
  static_assert(kPerChunk * kIters == kChunkIters, "chunk must hold whole stages");
};

__device__ __forceinline__ void lds_grad8(const float* p, float (&x)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  x[0] = a.x; x[1] = a.y; x[2] = a.z; x[3] = a.w;
  x[4] = b.x; x[5] = b.y; x[6] = b.z; x[7] = b.w;
}
__device__ __forceinline__ void lds_grad8(const uint16_t* p, float (&x)[8]) {
  unpack_bf16x8(*reinterpret_cast<const uint4*>(p), x);
}

constexpr size_t norm_bulk_smem_bytes() {
  return size_t(kNormStages) * kNormStageBytes + kBarrierBytes;
}

template <typename GT, bool kMul>
__device__ __forceinline__ bool norm_bulk_chunks(const GT* __restrict__ g, uint64_t chunk_begin,
                                                 uint32_t n_full, uint8_t* smem, uint64_t* full,
                                                 double* __restrict__ partials,
                                                 double* warp_sums, const ScaleInfo& sc,
                                                 bool& bad) {
  using Stage = NormStage<GT>;
  const uint32_t mine =
      n_full > blockIdx.x ? (n_full - 1u - blockIdx.x) / gridDim.x + 1u : 0u;
  const uint32_t total = mine * Stage::kPerChunk;  // stages this block consumes
  // Thread 0 only: stage j of this block's stream.
  auto issue = [&](uint32_t j) {
    const uint32_t s = j % kNormStages;
    const uint64_t chunk = chunk_begin + blockIdx.x + uint64_t(j / Stage::kPerChunk) * gridDim.x;
    const uint64_t e0 = chunk * kChunkElems + uint64_t(j % Stage::kPerChunk) * Stage::kElems;
    mbar_arrive_expect_tx(&full[s], kNormStageBytes);
    bulk_load(smem + size_t(s) * kNormStageBytes, g + e0, kNormStageBytes, &full[s]);
  };
  uint32_t issued = 0;
  if (threadIdx.x == 0)
    for (; issued < kNormStages && issued < total; ++issued) issue(issued);
  double acc = 0.0;
  bool ok = true;
  for (uint32_t j = 0; j < total; ++j) {
    const uint32_t s = j % kNormStages;
    ok = mbar_wait(&full[s], (j / kNormStages) & 1u);
    if (ok) {
      const GT* sg = reinterpret_cast<const GT*>(smem + size_t(s) * kNormStageBytes) +
                     threadIdx.x * kVec;
#pragma unroll
      for (uint32_t k = 0; k < Stage::kIters; ++k) {
        float x[kVec];
        lds_grad8(sg + k * (kTreeThreads * kVec), x);
        acc = add_squares8<kMul>(acc, x, sc);
      }
    }
    // Stage s is fully read (or someone gave up): refill it or leave together.
    if (__syncthreads_or(ok ? 0 : 1)) {
      if (threadIdx.x == 0)
        for (uint32_t i = j; i < issued; ++i)  // copies still in flight
          mbar_wait(&full[i % kNormStages], (i / kNormStages) & 1u);
      return false;
    }
    if (threadIdx.x == 0 && issued < total) issue(issued++);
    if ((j + 1) % Stage::kPerChunk == 0) {
      bad |= !isfinite(acc);
      const double sum = block_fold(acc, warp_sums);
      if (threadIdx.x == 0)
        partials[chunk_begin + blockIdx.x + uint64_t(j / Stage::kPerChunk) * gridDim.x] = sum;
      acc = 0.0;
    }
  }
  return true;
}

template <typename GT>
__global__ void __launch_bounds__(kTreeThreads, 2)
    norm_bulk_kernel(const GT* __restrict__ g, uint64_t n, uint64_t chunk_begin,
                     uint32_t n_chunks, DeviceScaler* scaler, double* __restrict__ partials,
                     DeviceStepState* st, FinalizeParams fp) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ double warp_sums[kTreeThreads / 32];
  __shared__ uint32_t s_last;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + size_t(kNormStages) * kNormStageBytes);
  // The update pass may launch now: it only prefetches data this kernel does
  // not write until it has waited for this kernel to complete.
  pdl_trigger();
  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < kNormStages; ++s) mbar_init(&full[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  const ScaleInfo sc = decode_scale(fp.dynamic ? scaler->scale : fp.static_scale);
  // Whole chunks of [chunk_begin, chunk_begin + n_chunks) go through shared memory.
  const uint64_t end_elem = (chunk_begin + n_chunks) * uint64_t(kChunkElems);
  const uint32_t n_full = end_elem <= n ? n_chunks : n_chunks - 1u;
  bool bad = false;
  const bool ok = sc.mul ? norm_bulk_chunks<GT, true>(g, chunk_begin, n_full, smem, full,
                                                      partials, warp_sums, sc, bad)
                         : norm_bulk_chunks<GT, false>(g, chunk_begin, n_full, smem, full,
                                                       partials, warp_sums, sc, bad);
  if (ok && n_full < n_chunks && blockIdx.x == gridDim.x - 1) {
    const uint64_t chunk = chunk_begin + n_full;
    const double acc = sc.mul ? chunk_thread_sum<GT, true>(g, chunk * kChunkElems, n, sc)
                              : chunk_thread_sum<GT, false>(g, chunk * kChunkElems, n, sc);
    bad |= !isfinite(acc);
    const double sum = block_fold(acc, warp_sums);
    if (threadIdx.x == 0) partials[chunk] = sum;
  }
  const int any_bad = __syncthreads_or(bad ? 1 : 0);
  if (threadIdx.x == 0) {
    if (!ok) atomicOr(&st->kernel_error, 1u);
    if (any_bad) atomicOr(&st->nonfinite_accum, 1u);
    __threadfence();
    s_last = (atomicAdd(&st->blocks_done, 1u) == gridDim.x - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (s_last == 0u) return;
  __threadfence();
  const uint32_t nonfinite =
      threadIdx.x == 0 ? (atomicExch(&st->nonfinite_accum, 0u) != 0u ? 1u : 0u) : 0u;
  finalize_block(PartialsView{partials, fp.total_chunks, fp.total_chunks}, nonfinite, st, scaler,
                 fp, warp_sums);
}

// ---- the reference's sequential clip scale, exact and parallel ---------------------
// gradient_clip_scale (src/model/oracle.rs:486-507) adds the squares one after
// another in f32, s <- fl(s + fl(g*g)), then clip = min(1 / sqrt(s), 1).  At
// 135M terms that sum drifts far from the exact one (it drops most terms once
// s is large), and the drop-ins must reproduce it bit for bit.  It is computed
// here in parallel, exactly:
//
//   While s stays in one binade, s = m * 2^E with an integer m < 2^24 and a
//   fixed ulp 2^E.  Adding q >= 0 then gives fl(s + q) = (m + r) * 2^E with
//   r = q / 2^E rounded to the nearest integer -- an increment that does not
//   depend on m, except when q / 2^E lies exactly halfway (ties go to the even
//   m + r) or when m + r reaches 2^24 (the sum leaves the binade and the ulp
//   doubles).  So a window of terms is one integer prefix sum of increments;
//   at the first term that ties or would leave the binade, the prefix before it
//   is applied, that one term is added with a real f32 add, and the rest of the
//   window is redone with the new binade.  Only a few dozen terms of 135M ever
//   take that path (binade changes are logarithmic in the sum's growth).
//
// One CTA of 1024 threads walks 8,192-term windows in order (thread t owns
// terms 8t..8t+7 of a window, so thread order is term order); thread 0 keeps
// kSeqStages windows in flight with cp.async.bulk.  Increments are reduced
// with warp shuffles and shared memory; unsigned 32-bit wrap-around can only
// corrupt prefixes after the first term whose exact prefix already reached
// 2^24, which is never used.  A non-finite gradient anywhere makes the status
// MODEL_GRADIENT_NONFINITE (the reference stops at the first one; the outcome
// is the same); a sum that overflows makes it MODEL_GRADIENT_NORM_NONFINITE.
// Waits are bounded as in the other pipelines.
constexpr uint32_t kSeqThreads = 1024;
constexpr uint32_t kSeqPer = 8;
constexpr uint32_t kSeqWindow = kSeqThreads * kSeqPer;  // 8,192 terms
constexpr uint32_t kSeqWindowBytes = kSeqWindow * 4;    // 32 KB
constexpr uint32_t kSeqStages = 6;
constexpr uint32_t kNoStop = 0xffffffffu;

// s = m * 2^E: E >= -149, m < 2^24 (for E > -149, m >= 2^23).
__device__ __forceinline__ void seq_decompose(float s, int32_t& E, uint32_t& m) {
  const uint32_t b = __float_as_uint(s);
  const uint32_t exp = (b >> 23) & 0xffu;
  const uint32_t man = b & 0x7fffffu;
  E = exp == 0u ? -149 : int32_t(exp) - 150;
  m = exp == 0u ? man : (man | 0x800000u);
}
__device__ __forceinline__ float seq_compose(int32_t E, uint32_t m) {
  return __uint_as_float((uint32_t(E + 149) << 23) + m);
}
// q / 2^E rounded to nearest (exact halves flagged as ties); anything that
// certainly leaves the binade returns 2^25.
// Branch-free: the terms of one warp have different exponents.
__device__ __forceinline__ uint32_t seq_increment(float q, int32_t E, bool& tie) {
  const uint32_t b = __float_as_uint(q);
  const uint32_t exp = (b >> 23) & 0xffu;
  const uint32_t man = b & 0x7fffffu;
  const uint32_t Q = exp == 0u ? man : (man | 0x800000u);
  const int32_t F = exp == 0u ? -149 : int32_t(exp) - 150;
  const int32_t d = E - F;
  // For d in [1, 31] the shift arithmetic below is exact; d > 25 gives 0 and
  // no tie there (Q < 2^24 <= half).  d == 0 adds Q ulps exactly; d < 0 means
  // q is at least 2^24 ulps of s (or not finite): it certainly leaves the binade.
  const uint32_t dc = uint32_t(d < 1 ? 1 : (d > 31 ? 31 : d));
  const uint32_t half = 1u << (dc - 1u);
  const uint32_t rem = Q & ((half << 1) - 1u);
  const uint32_t r = (Q >> dc) + (rem > half ? 1u : 0u);
  tie = d > 0 && rem == half;
  return d < 0 ? (1u << 25) : (d == 0 ? Q : r);
}

// Shared state of the sequential sum within one CTA.
struct SeqShared {
  uint32_t warp_val[kSeqThreads / 32];
  uint32_t warp_stop[kSeqThreads / 32];
  int32_t E;           // the running sum is m * 2^E ...
  uint32_t m;
  uint32_t sum_bad;    // ... unless it became non-finite (then sum_bits holds it)
  float sum_bits;
  uint32_t restart[2];  // by pass parity: a pass's value is read before it is reset
  uint32_t fast_total[2], fast_tie[2];
  uint32_t gbad_before;  // a non-finite gradient in an earlier slice
};

__device__ __forceinline__ void seq_begin(SeqShared& sh, const SeqCarry* carry, int resume) {
  if (resume) {  // continue the sum of the slices before this one
    sh.E = carry->E;
    sh.m = carry->m;
    sh.sum_bad = carry->sum_bad;
    sh.sum_bits = carry->sum_bits;
    sh.gbad_before = carry->gbad;
  } else {
    sh.E = -149;
    sh.m = 0u;
    sh.sum_bad = 0u;
    sh.sum_bits = 0.0f;
    sh.gbad_before = 0u;
  }
}

// Adds one window's terms (thread t holds terms 8t..8t+7 as q[], already
// squared) to the running sum, exactly: a block-wide prefix of increments
// finds the first term that ties or leaves the binade, the prefix before it
// is applied, that term is added with a real f32 add, and the rest of the
// window is redone with the new binade.  Called by all threads of the CTA.
// Two barriers per pass: each warp publishes its total (thread totals
// clamped at 2^24, which keeps every sum below 2^29 and every comparison with
// 2^24 - m as it was) and its first tie; then every warp scans the 32 warp
// summaries itself, so all threads know the first tie and the first warp
// whose running total leaves the binade, and only that warp looks for the
// exact term.  The one thread owning the stopping term publishes the new sum
// and where to resume; `restart` defaults to the window's end, so every pass
// moves forward (two slots by pass parity: thread 0 resets the next pass's
// slot while others may still read this one's).
__device__ __forceinline__ void seq_window_exact(SeqShared& sh, const float (&q)[kSeqPer]) {
  constexpr uint32_t kWarps = kSeqThreads / 32;
  constexpr uint32_t kWarpTerms = 32 * kSeqPer;
  static_assert(kWarps == 32, "one lane per warp in the block-wide scans");
  const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5;
  uint32_t start = 0;  // first term of the window not yet added
  for (uint32_t pass = 0; pass <= kSeqWindow; ++pass) {  // block-uniform
    if (sh.sum_bad) break;
    const int32_t E = sh.E;
    const uint32_t m = sh.m;
    uint32_t pre[kSeqPer], run = 0, tie_at = kNoStop;
#pragma unroll
    for (uint32_t j = 0; j < kSeqPer; ++j) {
      const uint32_t idx = 8 * t + j;
      bool tie = false;
      const uint32_t r = idx < start ? 0u : seq_increment(q[j], E, tie);
      run += r;  // 8 x 2^25 at most
      pre[j] = run;
      if (tie && tie_at == kNoStop) tie_at = idx;
    }
    const uint32_t runc = run < (1u << 24) ? run : (1u << 24);
    uint32_t incl = runc;  // this warp's inclusive prefix of clamped thread totals
#pragma unroll
    for (uint32_t off = 1; off < 32; off <<= 1) {
      const uint32_t y = __shfl_up_sync(kFull, incl, off);
      if (lane >= off) incl += y;
    }
    const uint32_t wtie = __reduce_min_sync(kFull, tie_at);
    if (lane == 31) sh.warp_val[warp] = incl < (1u << 24) ? incl : (1u << 24);
    if (lane == 0) sh.warp_stop[warp] = wtie;
    uint32_t& restart = sh.restart[pass & 1u];
    if (t == 0) restart = kSeqWindow;
    __syncthreads();
    uint32_t scan = sh.warp_val[lane];  // lane l: inclusive total through warp l
#pragma unroll
    for (uint32_t off = 1; off < 32; off <<= 1) {
      const uint32_t y = __shfl_up_sync(kFull, scan, off);
      if (lane >= off) scan += y;
    }
    const uint32_t first_tie = __reduce_min_sync(kFull, sh.warp_stop[lane]);
    const uint32_t leaves = __ballot_sync(kFull, uint64_t(m) + scan >= (1ull << 24));
    const uint32_t wstar = leaves ? uint32_t(__ffs(leaves)) - 1u : kWarps;
    const uint32_t total = __shfl_sync(kFull, scan, 31);
    if (wstar == kWarps && first_tie == kNoStop) {  // the rest stays in the binade
      if (t == 0) sh.m = m + total;
      __syncthreads();
      break;
    }
    // The stop is the first tie if it comes before warp wstar's terms; else
    // it lies in warp wstar (its first tie or its first term leaving the binade).
    const bool in_wstar = wstar < kWarps && first_tie >= kWarpTerms * wstar;
    const uint32_t below = __shfl_sync(kFull, scan, warp ? warp - 1u : 0u);
    const uint32_t excl = (warp ? below : 0u) + (incl - runc);  // exact up to the stop
    uint32_t first = first_tie;
    if (in_wstar && warp == wstar) {
      uint32_t cross = kNoStop;
#pragma unroll
      for (uint32_t j = 0; j < kSeqPer; ++j) {
        const uint32_t idx = 8 * t + j;
        if (idx >= start && cross == kNoStop && uint64_t(m) + excl + pre[j] >= (1ull << 24))
          cross = idx;
      }
      const uint32_t c = __reduce_min_sync(kFull, cross);
      first = c < first_tie ? c : first_tie;
    }
    const bool knows = !in_wstar || warp == wstar;
    if (knows && first >= 8 * t && first < 8 * t + kSeqPer) {  // the owner of the stop
      const uint32_t j0 = first - 8 * t;
      uint32_t before = excl;
      float qj = 0.0f;
#pragma unroll
      for (uint32_t j = 0; j < kSeqPer; ++j) {  // no dynamic register indexing
        if (j + 1 == j0) before += pre[j];
        if (j == j0) qj = q[j];
      }
      const float sum = __fadd_rn(seq_compose(E, m + before), qj);
      if (!finite_f32(sum)) {
        sh.sum_bad = 1u;
        sh.sum_bits = sum;
      } else {
        int32_t E2;
        uint32_t m2;
        seq_decompose(sum, E2, m2);
        sh.E = E2;
        sh.m = m2;
      }
      restart = first + 1;
    }
    __syncthreads();
    start = restart;
    if (start >= kSeqWindow) break;
  }
}

// Thread 0: the result (or, between slices, the running state).
__device__ __forceinline__ void seq_store(const SeqShared& sh, bool any_bad, bool ok,
                                          const SeqClipOut& out, uint32_t* kernel_error,
                                          SeqCarry* carry, int finish) {
  if (!ok) {
    atomicOr(kernel_error, 1u);
    return;
  }
  if (!finish) {  // hand the running sum to the launch for the next slice
    carry->E = sh.E;
    carry->m = sh.m;
    carry->sum_bad = sh.sum_bad;
    carry->sum_bits = sh.sum_bits;
    carry->gbad = any_bad ? 1u : 0u;
    return;
  }
  const float sum = sh.sum_bad ? sh.sum_bits : seq_compose(sh.E, sh.m);
  int32_t status = kStatusOk;
  float clip = 1.0f;
  if (any_bad) {
    status = kStatusGradientNonfinite;
  } else if (!finite_f32(sum)) {
    status = kStatusNormNonfinite;
  } else if (sum != 0.0f) {
    const float c = __fdiv_rn(1.0f, __fsqrt_rn(sum));
    clip = c < 1.0f ? c : 1.0f;
  }
  if (out.st) {
    DeviceStepState* st = out.st;
    st->sum_squares = double(sum);
    st->grad_norm = double(__fsqrt_rn(sum));
    st->clip_scale = clip;
    st->clip_apply = 1.0f;  // the gradients arrive clipped
    st->loss_scale_used = 1.0f;
    st->next_loss_scale = 1.0f;
    st->skipped = status == kStatusOk ? 0u : 1u;
    st->nonfinite = status == kStatusOk ? 0u : 1u;
    st->result_nonfinite = 0u;
    st->rejected = 0u;
    st->status = status;
  } else {
    *out.sum = sum;
    *out.clip = clip;
    *out.status = status;
  }
}

// One CTA streaming every window through a bulk-copy ring (used when no
// workspace for the parallel passes below is given).
__global__ void __launch_bounds__(kSeqThreads, 1)
    sequential_clip_kernel(const float* __restrict__ g, uint64_t n, SeqClipOut out,
                           uint32_t* kernel_error, SeqCarry* carry, int resume, int finish) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ SeqShared sh;
  const float* ring = reinterpret_cast<const float*>(smem);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + size_t(kSeqStages) * kSeqWindowBytes);
  const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5;
  if (t == 0) {
    for (uint32_t s = 0; s < kSeqStages; ++s) mbar_init(&full[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    seq_begin(sh, carry, resume);
  }
  __syncthreads();
  const uint64_t n_full = n / kSeqWindow;
  const uint64_t n_windows = n_full + (n % kSeqWindow ? 1u : 0u);
  auto issue = [&](uint64_t w) {
    const uint32_t s = uint32_t(w % kSeqStages);
    mbar_arrive_expect_tx(&full[s], kSeqWindowBytes);
    bulk_load(smem + size_t(s) * kSeqWindowBytes, g + w * kSeqWindow, kSeqWindowBytes, &full[s]);
  };
  uint64_t issued = 0;
  if (t == 0)
    for (; issued < kSeqStages && issued < n_full; ++issued) issue(issued);
  bool ok = true, gbad = false;
  for (uint64_t w = 0; w < n_windows; ++w) {
    float q[kSeqPer];
    if (w < n_full) {
      const uint32_t s = uint32_t(w % kSeqStages);
      ok = mbar_wait(&full[s], uint32_t(w / kSeqStages) & 1u);
      if (ok) {
        const float4 a = *reinterpret_cast<const float4*>(ring + size_t(s) * kSeqWindow + 8 * t);
        const float4 c =
            *reinterpret_cast<const float4*>(ring + size_t(s) * kSeqWindow + 8 * t + 4);
        q[0] = a.x; q[1] = a.y; q[2] = a.z; q[3] = a.w;
        q[4] = c.x; q[5] = c.y; q[6] = c.z; q[7] = c.w;
      }
    } else {  // the ragged last window: zeros past n add nothing
#pragma unroll
      for (uint32_t j = 0; j < kSeqPer; ++j) {
        const uint64_t i = w * kSeqWindow + 8 * t + j;
        q[j] = i < n ? g[i] : 0.0f;
      }
    }
    if (__syncthreads_or(ok ? 0 : 1)) {  // a copy never arrived: leave together
      ok = false;
      break;
    }
    if (t == 0 && issued < n_full) issue(issued++);  // this window's stage is read
#pragma unroll
    for (uint32_t j = 0; j < kSeqPer; ++j) {
      gbad |= !finite_f32(q[j]);
      q[j] = __fmul_rn(q[j], q[j]);
    }
    // Fast path: the window's total increment for the current binade and
    // whether any term ties; if nothing ties and the sum stays in the binade
    // the whole window is one integer add.  Totals are clamped at 2^24 (any
    // such total leaves the binade, which is all that is tested).
    if (!sh.sum_bad) {
      const int32_t E = sh.E;
      const uint32_t m = sh.m;
      uint32_t tsum = 0;
      bool tie_any = false;
#pragma unroll
      for (uint32_t j = 0; j < kSeqPer; ++j) {
        bool tie;
        tsum += seq_increment(q[j], E, tie);  // <= 8 * 2^25: no wrap
        tie_any |= tie;
      }
      const uint32_t wsum = __reduce_add_sync(kFull, tsum < (1u << 24) ? tsum : (1u << 24));
      const uint32_t wtie = __reduce_or_sync(kFull, tie_any ? 1u : 0u);
      if (lane == 0) {
        sh.warp_val[warp] = wsum < (1u << 24) ? wsum : (1u << 24);
        sh.warp_stop[warp] = wtie;
      }
      __syncthreads();
      // The window's verdict goes to slot w % 2, so the next window's write
      // never meets a thread still reading this one (no third barrier).
      const uint32_t slot = uint32_t(w & 1u);
      if (warp == 0) {
        const uint32_t v = __reduce_add_sync(kFull, sh.warp_val[lane]);
        const uint32_t tw = __reduce_or_sync(kFull, sh.warp_stop[lane]);
        if (lane == 0) {
          sh.fast_total[slot] = v;
          sh.fast_tie[slot] = tw;
        }
      }
      __syncthreads();
      const uint32_t total = sh.fast_total[slot];
      if (sh.fast_tie[slot] == 0u && uint64_t(m) + total < (1ull << 24)) {
        if (t == 0) sh.m = m + total;
        continue;  // the next window starts with a barrier
      }
      seq_window_exact(sh, q);
    }
  }
  // After a failed wait thread 0 waits (bounded) for its copies in flight.
  if (!ok && t == 0)
    for (uint64_t u = issued > kSeqStages ? issued - kSeqStages : 0; u < issued; ++u)
      mbar_wait(&full[u % kSeqStages], uint32_t(u / kSeqStages) & 1u);
  const bool any_bad = __syncthreads_or(gbad ? 1 : 0) || sh.gbad_before;
  if (t == 0) seq_store(sh, any_bad, ok, out, kernel_error, carry, finish);
}

// ---- the same sum with every SM: candidate binades, then one chain ----------------
// While the sum stays in a binade, a whole window adds an integer number of
// ulps that depends only on that binade.  So windows are summarised in
// parallel first -- for each, its total increment and tie flag under the
// kSeqCandUsed binades the running sum can plausibly be in there (the binade
// of the window's exact f64 prefix sum and its neighbours: the in-order f32
// sum drifts from that prefix by well under a factor of 2 in practice) -- and one CTA
// then chains the windows in order through those summaries, adding the exact
// window procedure above only where the sum's binade is not among the
// candidates, a term ties, or the window's total leaves the binade.  Which
// binades are candidates affects only how many windows take the exact path,
// never the result.
constexpr int kSeqCand = 4;  // slots per window record
#ifndef SLM_SEQ_CANDS
#define SLM_SEQ_CANDS 3  // candidate binades computed (the rest of the record never fits)
#endif
#ifndef SLM_SEQ_CAND_BELOW
#define SLM_SEQ_CAND_BELOW 1  // the first candidate's distance below the prefix's binade
#endif
#ifndef SLM_SEQ_XU_CANDS
#define SLM_SEQ_XU_CANDS 2
#endif
constexpr int kSeqCandUsed = SLM_SEQ_CANDS;
constexpr int kSeqCandBelow = SLM_SEQ_CAND_BELOW;
constexpr int kSeqXuCands = SLM_SEQ_XU_CANDS;  // candidates rounded with rintf
static_assert(kSeqCandUsed >= 1 && kSeqCandUsed <= kSeqCand, "1..4 candidates per record");
constexpr uint32_t kSeqPassThreads = 256;
constexpr uint32_t kSeqChainBatch = 1024;  // window summaries per shared-memory batch

struct SeqWorkspace {  // per window: totals, exact sum, candidate base, flags
  uint32_t* total;  // kSeqCand per window (16 bytes), clamped at 2^24
  double* sums;
  int32_t* base;
  uint8_t* flags;   // bit c: candidate c ties; bit 7: a non-finite gradient
};
static_assert(kSeqCand == 4, "a window's candidate totals are one 16-byte record");

__device__ __forceinline__ uint32_t seq_pick(const uint4& v, int32_t c) {
  return c == 0 ? v.x : (c == 1 ? v.y : (c == 2 ? v.z : v.w));
}

__device__ __forceinline__ int32_t seq_binade(float s) {
  const uint32_t exp = (__float_as_uint(s) >> 23) & 0xffu;
  return exp == 0u ? -149 : int32_t(exp) - 150;
}

// Thread t's 32 terms of window w, as 8 coalesced 16-byte loads for a whole
// window (the passes below need no particular order within a window); the
// ragged last window element by element, zeros past n.
__device__ __forceinline__ void seq_pass_load(const float* __restrict__ g, uint64_t n,
                                              uint64_t w, float (&x)[kSeqWindow / kSeqPassThreads]) {
  const uint32_t t = threadIdx.x;
  if ((w + 1) * kSeqWindow <= n) {
    const float4* v = reinterpret_cast<const float4*>(g + w * kSeqWindow);
#pragma unroll
    for (uint32_t k = 0; k < kSeqWindow / kSeqPassThreads / 4; ++k) {
      const float4 a = __ldg(v + t + kSeqPassThreads * k);
      x[4 * k] = a.x;
      x[4 * k + 1] = a.y;
      x[4 * k + 2] = a.z;
      x[4 * k + 3] = a.w;
    }
  } else {
#pragma unroll
    for (uint32_t k = 0; k < kSeqWindow / kSeqPassThreads; ++k) {
      const uint64_t i = w * kSeqWindow + uint64_t(t + kSeqPassThreads * (k / 4)) * 4 + k % 4;
      x[k] = i < n ? g[i] : 0.0f;
    }
  }
}

__global__ void __launch_bounds__(kSeqPassThreads)
    seqclip_sums_kernel(const float* __restrict__ g, uint64_t n, uint64_t n_windows,
                        SeqWorkspace ws) {
  __shared__ double wsum[kSeqPassThreads / 32];
  __shared__ uint32_t wbad[kSeqPassThreads / 32];
  const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5;
  for (uint64_t w = blockIdx.x; w < n_windows; w += gridDim.x) {
    float x[kSeqWindow / kSeqPassThreads];
    seq_pass_load(g, n, w, x);
    double acc = 0.0;
    bool bad = false;
#pragma unroll
    for (uint32_t k = 0; k < kSeqWindow / kSeqPassThreads; ++k) {
      bad |= !finite_f32(x[k]);
      acc += double(__fmul_rn(x[k], x[k]));
    }
#pragma unroll
    for (int off = 16; off >= 1; off >>= 1) acc += __shfl_down_sync(kFull, acc, off);
    const uint32_t b = __reduce_or_sync(kFull, bad ? 1u : 0u);
    if (lane == 0) {
      wsum[warp] = acc;
      wbad[warp] = b;
    }
    __syncthreads();
    if (t == 0) {
      double s = 0.0;
      uint32_t bb = 0;
      for (uint32_t i = 0; i < kSeqPassThreads / 32; ++i) {
        s += wsum[i];
        bb |= wbad[i];
      }
      ws.sums[w] = s;
      ws.flags[w] = bb ? 0x80u : 0u;
    }
    __syncthreads();
  }
}

// Exclusive prefix of the window sums (continuing the previous slice's) and
// each window's first candidate binade.  One CTA: warp w owns a run of
// `steps` x 32 consecutive windows, lane l the windows l, l + 32, ... of it
// (coalesced loads, all issued before they are added); the warps' totals are
// scanned across the block, then every warp scans its run 32 windows at a
// time.  Any order of the f64 additions will do: the prefix only chooses
// candidates.
__global__ void __launch_bounds__(kSeqThreads)
    seqclip_prefix_kernel(uint64_t n_windows, SeqWorkspace ws, SeqCarry* carry, int resume,
                          int keep) {
  __shared__ double warp_tot[kSeqThreads / 32];
  __shared__ double s_start;
  const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5;
  const uint64_t steps = (n_windows + kSeqThreads - 1) / kSeqThreads;
  const uint64_t w_lo = uint64_t(warp) * steps * 32;
  auto load8 = [&](uint64_t j0, double (&v)[8]) {
#pragma unroll
    for (uint32_t j = 0; j < 8; ++j) {
      const uint64_t idx = w_lo + (j0 + j) * 32 + lane;
      v[j] = j0 + j < steps && idx < n_windows ? ws.sums[idx] : 0.0;
    }
  };
  double mine = 0.0;
  for (uint64_t j0 = 0; j0 < steps; j0 += 8) {
    double v[8];
    load8(j0, v);
#pragma unroll
    for (uint32_t j = 0; j < 8; ++j) mine += v[j];
  }
#pragma unroll
  for (uint32_t off = 16; off >= 1; off >>= 1) mine += __shfl_xor_sync(kFull, mine, off);
  if (lane == 0) warp_tot[warp] = mine;
  if (t == 0) s_start = resume ? carry->prefix : 0.0;
  __syncthreads();
  if (warp == 0) {
    double v = warp_tot[lane];
#pragma unroll
    for (uint32_t off = 1; off < 32; off <<= 1) {
      const double y = __shfl_up_sync(kFull, v, off);
      if (lane >= off) v += y;
    }
    warp_tot[lane] = v;  // inclusive
  }
  __syncthreads();
  double run = s_start + (warp ? warp_tot[warp - 1] : 0.0);
  for (uint64_t j0 = 0; j0 < steps; j0 += 8) {
    double v[8];
    load8(j0, v);
#pragma unroll
    for (uint32_t j = 0; j < 8; ++j) {
      double incl = v[j];
#pragma unroll
      for (uint32_t off = 1; off < 32; off <<= 1) {
        const double y = __shfl_up_sync(kFull, incl, off);
        if (lane >= off) incl += y;
      }
      const uint64_t idx = w_lo + (j0 + j) * 32 + lane;
      if (j0 + j < steps && idx < n_windows)
        ws.base[idx] = seq_binade(float(run + (incl - v[j]))) - kSeqCandBelow;
      run += __shfl_sync(kFull, incl, 31);
    }
  }
  if (keep && t == 0) carry->prefix = s_start + warp_tot[kSeqThreads / 32 - 1];
}

// 2^k as an f32, k in [-149, 127].
__device__ __forceinline__ float seq_pow2(int32_t k) {
  return k >= -126 ? __uint_as_float(uint32_t(k + 127) << 23) : __uint_as_float(1u << (k + 149));
}

// Per window and candidate binade E = base + c: the window's total increment
// sum(round(q / 2^E)) and whether some q / 2^E has a fractional part of
// exactly one half (a tie, which the chain resolves term by term).  In f32:
// y = q / 2^E is exact (a power-of-two scaling; an overflow means y >= 2^24
// anyway, an underflow means y < 2^-126, an increment of 0 that cannot tie),
// rintf(y) is the increment wherever there is no tie, y - rintf(y) is exact
// and is +-0.5 exactly at a tie, and an f32 running total of non-negative
// integers is exact below 2^24 and stays >= 2^24 once the exact total gets
// there -- all the chain needs (totals are clamped at 2^24).  An infinite or
// NaN term gives a total of 2^24 (the chain then adds that window exactly).
__global__ void __launch_bounds__(kSeqPassThreads)
    seqclip_candidates_kernel(const float* __restrict__ g, uint64_t n, uint64_t n_windows,
                              SeqWorkspace ws) {
  __shared__ uint32_t wtot[kSeqCandUsed][kSeqPassThreads / 32];
  __shared__ uint32_t wtie[kSeqPassThreads / 32];
  const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5;
  for (uint64_t w = blockIdx.x; w < n_windows; w += gridDim.x) {
    float x[kSeqWindow / kSeqPassThreads];
    seq_pass_load(g, n, w, x);
    const int32_t k = -ws.base[w];  // in [-104, 151]: base >= -151
    const bool split = k > 127;
    const float s0 = seq_pow2(split ? k - 64 : (k < -149 ? -149 : k));
    const float s1 = split ? seq_pow2(64) : 1.0f;
    float tot[kSeqCandUsed] = {}, dev[kSeqCandUsed] = {};
#pragma unroll
    for (uint32_t j = 0; j < kSeqWindow / kSeqPassThreads; ++j) {
      float y = __fmul_rn(__fmul_rn(__fmul_rn(x[j], x[j]), s0), s1);
#pragma unroll
      for (int c = 0; c < kSeqCandUsed; ++c) {
        // rintf issues on the conversion unit; the first kSeqXuCands
        // candidates use it, the rest round by adding and removing 2^23 (below
        // 2^23, y + 2^23 lands where the f32 spacing is 1 and rounds to
        // nearest-even there, 2^23 being even; from 2^23 on y is an integer
        // already, inf and NaN pass), which spreads the work over two pipes.
        const float r = c < kSeqXuCands ? rintf(y)
                        : (y < 8388608.0f ? __fsub_rn(__fadd_rn(y, 8388608.0f), 8388608.0f) : y);
        tot[c] = __fadd_rn(tot[c], r);
        dev[c] = fmaxf(dev[c], fabsf(__fsub_rn(y, r)));
        y = __fmul_rn(y, 0.5f);
      }
    }
    uint32_t ties = 0;
#pragma unroll
    for (int c = 0; c < kSeqCandUsed; ++c) {
      const uint32_t v = tot[c] < 16777216.0f ? uint32_t(tot[c]) : (1u << 24);  // NaN too
      const uint32_t sum = __reduce_add_sync(kFull, v);  // 32 x 2^24: no wrap
      if (lane == 0) wtot[c][warp] = sum < (1u << 24) ? sum : (1u << 24);
      ties |= dev[c] == 0.5f ? (1u << c) : 0u;
    }
    const uint32_t tw = __reduce_or_sync(kFull, ties);
    if (lane == 0) wtie[warp] = tw;
    __syncthreads();
    if (t < kSeqCand) {  // slots past the used candidates never fit
      uint32_t v = 1u << 24;
      if (t < uint32_t(kSeqCandUsed)) {
        v = 0;
        for (uint32_t i = 0; i < kSeqPassThreads / 32; ++i) v += wtot[t][i];
      }
      ws.total[w * kSeqCand + t] = v < (1u << 24) ? v : (1u << 24);
    }
    if (t == 0) {
      uint32_t tb = 0;
      for (uint32_t i = 0; i < kSeqPassThreads / 32; ++i) tb |= wtie[i];
      ws.flags[w] = uint8_t(ws.flags[w] | tb);
    }
    __syncthreads();
  }
}

// One CTA chains the window summaries in order.  A batch of 1,024 windows is
// read into shared memory and summarised once more per group of 32 windows
// (warp j: group j): for each candidate binade from the group's first base,
// the group's total and whether every window of the group has that binade
// among its candidates without a tie.  Warp 0 then walks the batch, a group
// per lane while whole groups fit and a window per lane inside a group that
// does not; at a window no summary fits, all threads add it exactly.
__global__ void __launch_bounds__(kSeqThreads, 1)
    seqclip_chain_kernel(const float* __restrict__ g, uint64_t n, uint64_t n_windows,
                         SeqWorkspace ws, SeqClipOut out, uint32_t* kernel_error,
                         SeqCarry* carry, int resume, int finish) {
  constexpr uint32_t kGroups = kSeqChainBatch / 32;
  static_assert(kSeqChainBatch == kSeqThreads, "one window per thread when a batch is read");
  __shared__ SeqShared sh;
  __shared__ uint4 b_total[kSeqChainBatch];
  __shared__ int32_t b_base[kSeqChainBatch];
  __shared__ uint8_t b_flags[kSeqChainBatch];
  __shared__ uint4 g_total[kGroups];
  __shared__ int32_t g_base[kGroups];
  __shared__ uint32_t g_fit[kGroups];  // bit e: every window fits binade g_base + e
  __shared__ uint32_t s_next, s_miss;
  const uint32_t t = threadIdx.x, lane = t & 31u, warp = t >> 5;
  const uint4* totals = reinterpret_cast<const uint4*>(ws.total);
  if (t == 0) seq_begin(sh, carry, resume);
  bool gbad = false;
  for (uint64_t b0 = 0; b0 < n_windows; b0 += kSeqChainBatch) {
    const uint32_t nb = uint32_t(n_windows - b0 < kSeqChainBatch ? n_windows - b0
                                                                  : kSeqChainBatch);
    __syncthreads();  // the previous batch is no longer read
    if (t < nb) {
      b_total[t] = totals[b0 + t];
      b_base[t] = ws.base[b0 + t];
      const uint8_t f = ws.flags[b0 + t];
      b_flags[t] = f;
      gbad |= (f & 0x80u) != 0u;  // every window is added, by summary or exactly
    }
    __syncthreads();
    if (32 * warp < nb) {
      const uint32_t i = 32 * warp + lane;
      const bool present = i < nb;
      const int32_t gb = b_base[32 * warp];
      uint32_t fit = 0u;
      uint32_t gt[kSeqCand] = {1u << 24, 1u << 24, 1u << 24, 1u << 24};
#pragma unroll
      for (int e = 0; e < kSeqCandUsed; ++e) {
        bool ok = true;
        uint32_t tot = 0u;
        if (present) {
          const int32_t c = gb + e - b_base[i];
          ok = c >= 0 && c < kSeqCandUsed && ((b_flags[i] >> c) & 1u) == 0u;
          if (ok) tot = seq_pick(b_total[i], c);
        }
        const uint32_t sum = __reduce_add_sync(kFull, tot);  // 32 x 2^24: no wrap
        gt[e] = sum < (1u << 24) ? sum : (1u << 24);
        fit |= __all_sync(kFull, ok) ? (1u << e) : 0u;
      }
      if (lane == 0) {
        g_total[warp] = make_uint4(gt[0], gt[1], gt[2], gt[3]);
        g_base[warp] = gb;
        g_fit[warp] = fit;
      }
    }
    if (t == 0) s_next = 0u;
    __syncthreads();
    for (;;) {  // block-uniform: s_next and s_miss are read after a barrier
      if (warp == 0) {
        uint32_t k = s_next;
        uint32_t miss = 0u;
        if (sh.sum_bad) {  // the sum is no longer finite: nothing more to add
          k = nb;
        } else {
          // Within one binade every window (group) adds its own total, so
          // the 32 from k are accepted up to the first one that does not fit
          // this binade or whose running total leaves it.
          const int32_t E = sh.E;
          uint32_t m = sh.m;
          bool fine = (k & 31u) != 0u;  // inside a group: window by window
          while (k < nb) {
            uint32_t tot = 0u, avail;
            bool ok = false, present;
            if (fine) {
              const uint32_t end = ((k | 31u) + 1u) < nb ? ((k | 31u) + 1u) : nb;
              const uint32_t i = k + lane;
              avail = end - k;
              present = i < end;
              if (present) {
                const int32_t c = E - b_base[i];
                ok = c >= 0 && c < kSeqCandUsed && ((b_flags[i] >> c) & 1u) == 0u;
                if (ok) tot = seq_pick(b_total[i], c);
              }
            } else {
              const uint32_t g0 = k >> 5, ng = (nb + 31u) >> 5;
              const uint32_t gi = g0 + lane;
              avail = ng - g0;
              present = gi < ng;
              if (present) {
                const int32_t c = E - g_base[gi];
                ok = c >= 0 && c < kSeqCandUsed && ((g_fit[gi] >> c) & 1u) != 0u;
                if (ok) tot = seq_pick(g_total[gi], c);
              }
            }
            uint32_t pre = tot;  // 32 totals of at most 2^24: no wrap
#pragma unroll
            for (uint32_t off = 1; off < 32; off <<= 1) {
              const uint32_t y = __shfl_up_sync(kFull, pre, off);
              if (lane >= off) pre += y;
            }
            const bool stop = present && (!ok || uint64_t(m) + pre >= (1ull << 24));
            const uint32_t stops = __ballot_sync(kFull, stop);
            const uint32_t first = stops ? uint32_t(__ffs(stops)) - 1u : avail;
            if (first > 0u) m += __shfl_sync(kFull, pre, first - 1u);
            if (fine) {
              k += first;
              if (stops) {  // this window needs the exact procedure
                miss = 1u;
                break;
              }
              fine = false;  // the group is done
            } else {
              k = k + 32u * first < nb ? k + 32u * first : nb;
              fine = stops != 0u;  // walk the group that did not fit window by window
            }
          }
          if (lane == 0) sh.m = m;
        }
        if (lane == 0) {
          s_next = k;
          s_miss = miss;
        }
      }
      __syncthreads();
      if (!s_miss) break;
      // The window the summaries could not add: every thread takes its 8 terms.
      const uint64_t w = b0 + s_next;
      float q[kSeqPer];
      if ((w + 1) * kSeqWindow <= n) {  // a whole window: two 16-byte loads per thread
        const float4 a = *reinterpret_cast<const float4*>(g + w * kSeqWindow + 8 * t);
        const float4 c = *reinterpret_cast<const float4*>(g + w * kSeqWindow + 8 * t + 4);
        q[0] = a.x; q[1] = a.y; q[2] = a.z; q[3] = a.w;
        q[4] = c.x; q[5] = c.y; q[6] = c.z; q[7] = c.w;
      } else {
#pragma unroll
        for (uint32_t j = 0; j < kSeqPer; ++j) {
          const uint64_t i = w * kSeqWindow + 8 * t + j;
          q[j] = i < n ? g[i] : 0.0f;
        }
      }
#pragma unroll
      for (uint32_t j = 0; j < kSeqPer; ++j) {
        gbad |= !finite_f32(q[j]);
        q[j] = __fmul_rn(q[j], q[j]);
      }
      seq_window_exact(sh, q);
      if (t == 0) s_next += 1u;
      __syncthreads();
    }
  }
  const bool any_bad = __syncthreads_or(gbad ? 1 : 0) || sh.gbad_before;
  if (t == 0) seq_store(sh, any_bad, true, out, kernel_error, carry, finish);
}

// ---- state initialisation / validation ----------------------------------------
// bf16 weights -> f32 (the bits shifted into the high half, as the
// reference's bf16_bits_to_f32 does for every parameter it reloads into the
// graph); 8 elements per thread step, streaming.
__global__ void __launch_bounds__(256)
    export_f32_kernel(const uint16_t* __restrict__ w16, float* __restrict__ dst, uint64_t n) {
  const uint64_t vecs = n / kVec;
  for (uint64_t v = blockIdx.x * uint64_t(blockDim.x) + threadIdx.x; v < vecs;
       v += uint64_t(gridDim.x) * blockDim.x) {
    float x[kVec];
    unpack_bf16x8(__ldcs(reinterpret_cast<const uint4*>(w16) + v), x);
    __stcs(reinterpret_cast<float4*>(dst + v * kVec), make_float4(x[0], x[1], x[2], x[3]));
    __stcs(reinterpret_cast<float4*>(dst + v * kVec + 4), make_float4(x[4], x[5], x[6], x[7]));
  }
  const uint64_t i = vecs * kVec + blockIdx.x * uint64_t(blockDim.x) + threadIdx.x;
  if (i < n) dst[i] = __uint_as_float(static_cast<uint32_t>(w16[i]) << 16);
}

__global__ void init_from_master_kernel(const float* __restrict__ master,
                                        uint16_t* __restrict__ w16, uint64_t n) {
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x)
    w16[i] = bf16_rne_bits(master[i]);
}

__global__ void validate_state_kernel(const float* __restrict__ master,
                                      const float* __restrict__ mom,
                                      const float* __restrict__ var,
                                      const uint16_t* __restrict__ w16, uint64_t n,
                                      uint32_t* bad_flag) {
  bool bad = false;
  for (uint64_t i = blockIdx.x * static_cast<uint64_t>(blockDim.x) + threadIdx.x; i < n;
       i += static_cast<uint64_t>(gridDim.x) * blockDim.x) {
    const float t = master[i];
    bad |= !(finite_f32(t) && finite_f32(mom[i]) && finite_f32(var[i]) &&
             bf16_rne_bits(t) == w16[i]);
  }
  if (__any_sync(kFull, bad) && (threadIdx.x & 31) == 0) atomicOr(bad_flag, 1u);
}

// ---- ZeRO-1 over peer memory: two kernels per step ---------------------------------
// zero1_peer_reduce_kernel: one block per chunk of this rank's shard.  Its
// prologue is the gradient barrier (every block announces this rank's epoch to
// every rank and waits, bounded, for every rank's announcement).  Then the
// chunk streams through kPeerStages shared-memory stages: thread 0 issues, per
// stage, one bulk copy (cp.async.bulk, no multicast) of `rows` tree rows from
// every rank's gradient buffer -- over NVLink for the peers -- so the bytes in
// flight cost no registers; the 256 threads add their 8-element vectors in
// rank order 0..N-1 in f32, store the sums for the update, and accumulate the
// unscaled squares in the single-replica tree order.  The chunk partial goes
// straight into every rank's gathered area; the last block appends the
// non-finite flag and raises every rank's partials flag.
// zero1_peer_update_kernel: the bulk-copy update with the finalize in its
// prologue (every block reduces all ranks' partials with the same tree, so
// every block and every rank takes the same decision; block 0 publishes it)
// and the weight barrier in its epilogue (the last block to finish announces
// this rank's weights and waits, bounded, for every rank's).
// Every wait is bounded by timeout_ns; after a wait of a step has given up
// (kernel_error), later waits of the step return at once.
#ifndef SLM_PEER_LOADS
#define SLM_PEER_LOADS 1
#endif
#ifndef SLM_PEER_STAGES
#define SLM_PEER_STAGES 3
#endif
#ifndef SLM_PEER_STAGE_BYTES
#define SLM_PEER_STAGE_BYTES 32768
#endif
// At world <= 2 a rank's shard has ~1,033 chunks: one tree row per thread in
// flight and 8 blocks per SM (32 registers) make them all resident at once,
// one wave instead of 1.75 (0.619 against 0.628 ms per 135M step with 4 rows
// and 4 blocks per SM).
#ifndef SLM_PEER_BATCH2
#define SLM_PEER_BATCH2 1  // tree rows in flight per thread at world <= 2
#endif
#ifndef SLM_PEER_BATCH8
#define SLM_PEER_BATCH8 1  // tree rows in flight per thread at world > 4
#endif
#ifndef SLM_PEER_MINBLOCKS2
#define SLM_PEER_MINBLOCKS2 8  // resident blocks per SM asked of the compiler at world <= 2 (0: none)
#endif
constexpr bool kPeerLoads = SLM_PEER_LOADS != 0;     // plain loads instead of bulk copies
constexpr uint32_t kPeerStages = SLM_PEER_STAGES;
constexpr uint32_t kPeerStageTarget = SLM_PEER_STAGE_BYTES;  // one stage over all ranks

__device__ __forceinline__ uint32_t ld_volatile(const uint32_t* p) {
  return *reinterpret_cast<const volatile uint32_t*>(p);
}

// Waits until flag >= epoch (wrap-safe); false on timeout or once another wait
// of this step has given up.
__device__ __forceinline__ bool wait_epoch(const uint32_t* flag, uint32_t epoch,
                                           const DeviceStepState* st, uint64_t timeout_ns) {
  if (static_cast<int32_t>(ld_volatile(flag) - epoch) >= 0) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (static_cast<int32_t>(ld_volatile(flag) - epoch) >= 0) return true;
    if ((it & 63u) == 0u) {
      if (ld_volatile(&st->kernel_error) != 0u) return false;
      if (global_ns() - t0 > timeout_ns) return false;
    }
  }
}

// One chunk of the shard from every rank, streamed through shared memory.
// src_elem: the chunk's first element in the (global) gradient buffers;
// local: its first element in the shard (gsum index).
template <typename GT, bool kMul>
__device__ __forceinline__ bool peer_chunk_bulk(const PeerTable& pt, int world, uint64_t src_elem,
                                                uint64_t local, uint32_t rows,
                                                uint32_t stage_bytes, uint8_t* smem,
                                                uint64_t* full, float* __restrict__ gsum,
                                                const ScaleInfo& sc, double& acc) {
  constexpr uint32_t kRowElems = kTreeThreads * kVec;
  constexpr uint32_t kRowBytes = kRowElems * sizeof(GT);
  const uint32_t slice = rows * kRowBytes;  // one rank's part of a stage
  const uint32_t total = kChunkIters / rows;
  auto issue = [&](uint32_t j) {
    const uint32_t s = j % kPeerStages;
    uint8_t* dst = smem + size_t(s) * stage_bytes;
    const uint64_t e0 = src_elem + uint64_t(j) * rows * kRowElems;
    mbar_arrive_expect_tx(&full[s], stage_bytes);
    for (int q = 0; q < world; ++q)
      bulk_load(dst + size_t(q) * slice, static_cast<const GT*>(pt.grads[q]) + e0, slice,
                &full[s]);
  };
  uint32_t issued = 0;
  if (threadIdx.x == 0)
    for (; issued < kPeerStages && issued < total; ++issued) issue(issued);
  for (uint32_t j = 0; j < total; ++j) {
    const uint32_t s = j % kPeerStages;
    const bool ok = mbar_wait(&full[s], (j / kPeerStages) & 1u);
    if (ok) {
      const uint8_t* base = smem + size_t(s) * stage_bytes + threadIdx.x * kVec * sizeof(GT);
      for (uint32_t k = 0; k < rows; ++k) {
        float sum[kVec];
        lds_grad8(reinterpret_cast<const GT*>(base + k * kRowBytes), sum);
        for (int q = 1; q < world; ++q) {
          float x[kVec];
          lds_grad8(reinterpret_cast<const GT*>(base + size_t(q) * slice + k * kRowBytes), x);
#pragma unroll
          for (uint32_t e = 0; e < kVec; ++e) sum[e] = __fadd_rn(sum[e], x[e]);
        }
        float* out = gsum + local + uint64_t(j * rows + k) * kRowElems + threadIdx.x * kVec;
        __stcg(reinterpret_cast<float4*>(out), make_float4(sum[0], sum[1], sum[2], sum[3]));
        __stcg(reinterpret_cast<float4*>(out + 4), make_float4(sum[4], sum[5], sum[6], sum[7]));
        acc = add_squares8<kMul>(acc, sum, sc);
      }
    }
    // Stage s is fully read (or someone gave up): refill it or leave together.
    if (__syncthreads_or(ok ? 0 : 1)) {
      if (threadIdx.x == 0)
        for (uint32_t i = j; i < issued; ++i)  // copies still in flight
          mbar_wait(&full[i % kPeerStages], (i / kPeerStages) & 1u);
      return false;
    }
    if (threadIdx.x == 0 && issued < total) issue(issued++);
  }
  return true;
}

// The same whole chunk with plain 16/32-byte loads instead of bulk copies:
// kBatch tree rows of every rank (kBatch * kRanks loads per thread, mostly over
// NVLink) go out before any is added.
template <typename GT, bool kMul, int kBatch, int kRanks>
__device__ __forceinline__ double peer_chunk_loads(const PeerTable& pt, int world,
                                                   uint64_t src_elem, uint64_t local,
                                                   float* __restrict__ gsum,
                                                   const ScaleInfo& sc) {
  double acc = 0.0;
#pragma unroll 1
  for (uint32_t k0 = 0; k0 < kChunkIters; k0 += kBatch) {
    RawVec<GT> raw[kBatch][kRanks];
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      const uint64_t e0 = src_elem + uint64_t(k0 + b) * (kTreeThreads * kVec) +
                          uint64_t(threadIdx.x) * kVec;
#pragma unroll
      for (int q = 0; q < kRanks; ++q)
        if (q < world) raw[b][q].load(static_cast<const GT*>(pt.grads[q]) + e0);
    }
#pragma unroll
    for (int b = 0; b < kBatch; ++b) {
      float sum[kVec];
      raw[b][0].unpack(sum);
#pragma unroll
      for (int q = 1; q < kRanks; ++q)
        if (q < world) {
          float x[kVec];
          raw[b][q].unpack(x);
#pragma unroll
          for (uint32_t e = 0; e < kVec; ++e) sum[e] = __fadd_rn(sum[e], x[e]);
        }
      float* out = gsum + local + uint64_t(k0 + b) * (kTreeThreads * kVec) + threadIdx.x * kVec;
      __stcg(reinterpret_cast<float4*>(out), make_float4(sum[0], sum[1], sum[2], sum[3]));
      __stcg(reinterpret_cast<float4*>(out + 4), make_float4(sum[4], sum[5], sum[6], sum[7]));
      acc = add_squares8<kMul>(acc, sum, sc);
    }
  }
  return acc;
}

// The ragged last chunk (fewer than 65,536 valid elements), element-wise from
// global memory with the same order of additions.
template <typename GT, bool kMul>
__device__ __forceinline__ double peer_chunk_ragged(const PeerTable& pt, int world,
                                                    uint64_t shard_begin, uint64_t base,
                                                    uint64_t n, float* __restrict__ gsum,
                                                    const ScaleInfo& sc) {
  double acc = 0.0;
  for (uint32_t k = 0; k < kChunkIters; ++k) {
    const uint64_t e0 = base + static_cast<uint64_t>(k) * (kTreeThreads * kVec) +
                        static_cast<uint64_t>(threadIdx.x) * kVec;
    if (e0 >= n) break;
    float s[kVec];
    load_grad8(static_cast<const GT*>(pt.grads[0]) + shard_begin, e0, n, s);
    for (int q = 1; q < world; ++q) {
      float x[kVec];
      load_grad8(static_cast<const GT*>(pt.grads[q]) + shard_begin, e0, n, x);
#pragma unroll
      for (uint32_t j = 0; j < kVec; ++j) s[j] = __fadd_rn(s[j], x[j]);
    }
    for (uint32_t j = 0; j < kVec && e0 + j < n; ++j) gsum[e0 + j] = s[j];
    acc = add_squares8<kMul>(acc, s, sc);
  }
  return acc;
}

// kBatch == 0: bulk copies through shared memory; otherwise plain loads,
// kBatch rows x kRanks ranks in flight per thread.
template <typename GT, int kBatch, int kRanks, int kMinBlocks = 0>
__global__ void __launch_bounds__(kTreeThreads, kMinBlocks)
    zero1_peer_reduce_kernel(PeerTable pt, int rank, int world, uint64_t shard_begin,
                             uint64_t n_valid, uint32_t n_chunks, const DeviceScaler* scaler,
                             FinalizeParams fp, float* __restrict__ gsum, uint32_t rows,
                             uint32_t stage_bytes, uint32_t epoch, DeviceStepState* st,
                             uint64_t timeout_ns) {
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ double warp_sums[kTreeThreads / 32];
  __shared__ uint32_t s_last;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + size_t(kPeerStages) * stage_bytes);
  const uint32_t c = blockIdx.x;
  // The update kernel may launch once every block of this grid has started:
  // its producers wait for this grid to complete before they load, and its
  // consumers wait for the partials flags.
  pdl_trigger();
  // Gradient barrier.  This rank's gradient buffer was written by work that
  // completed before this kernel started; announce it, then wait for all.
  bool ok = true;
  if (threadIdx.x < static_cast<unsigned>(world)) {
    __threadfence_system();
    *reinterpret_cast<volatile uint32_t*>(pt.flags[threadIdx.x] + kSlotGrads * kMaxRanks +
                                          rank) = epoch;
    ok = wait_epoch(pt.flags[rank] + kSlotGrads * kMaxRanks + threadIdx.x, epoch, st,
                    timeout_ns);
    if (!ok) atomicOr(&st->kernel_error, 2u);
    // Acquire: the peer's gradients were published before its flag.  The
    // block barrier below orders the other threads' reads after this fence;
    // the bulk copy engine reads through the async proxy, hence its fence.
    __threadfence_system();
    if (kBatch == 0) asm volatile("fence.proxy.async;" ::: "memory");
  }
  if (kBatch == 0 && threadIdx.x == 0) {
    for (uint32_t s = 0; s < kPeerStages; ++s) mbar_init(&full[s], 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  ok = __syncthreads_or(ok ? 0 : 1) == 0;
  const ScaleInfo sc = decode_scale(fp.dynamic ? scaler->scale : fp.static_scale);
  const uint64_t base = uint64_t(c) * kChunkElems;
  double acc = 0.0;
  if (ok && base < n_valid) {
    if (base + kChunkElems <= n_valid) {
      if constexpr (kBatch == 0) {
        ok = sc.mul ? peer_chunk_bulk<GT, true>(pt, world, shard_begin + base, base, rows,
                                                stage_bytes, smem, full, gsum, sc, acc)
                    : peer_chunk_bulk<GT, false>(pt, world, shard_begin + base, base, rows,
                                                 stage_bytes, smem, full, gsum, sc, acc);
      } else {
        acc = sc.mul ? peer_chunk_loads<GT, true, kBatch, kRanks>(pt, world, shard_begin + base,
                                                                  base, gsum, sc)
                     : peer_chunk_loads<GT, false, kBatch, kRanks>(pt, world, shard_begin + base,
                                                                   base, gsum, sc);
      }
    } else {
      acc = sc.mul ? peer_chunk_ragged<GT, true>(pt, world, shard_begin, base, n_valid, gsum, sc)
                   : peer_chunk_ragged<GT, false>(pt, world, shard_begin, base, n_valid, gsum,
                                                  sc);
    }
  }
  const int any_bad = __syncthreads_or(isfinite(acc) ? 0 : 1);
  const double partial = block_fold(acc, warp_sums);
  if (threadIdx.x == 0) {
    if (ok) {
      const uint64_t slot = uint64_t(rank) * (n_chunks + 1) + c;
      for (int q = 0; q < world; ++q) pt.gathered[q][slot] = partial;
    } else {
      atomicOr(&st->kernel_error, 1u);
    }
    if (any_bad) atomicOr(&st->nonfinite_accum, 1u);
    if (c == 0) {
      st->loss_scale_used = sc.s;  // the update unscales with the same value
      st->result_nonfinite = 0u;   // raised by the update kernel
    }
    __threadfence_system();
    s_last = (atomicAdd(&st->blocks_done, 1u) == gridDim.x - 1) ? 1u : 0u;
  }
  __syncthreads();
  if (s_last == 0u || threadIdx.x != 0) return;
  // Last block: the non-finite flag, then the partials flag on every rank.  A
  // rank whose step failed here announces nothing: its partials are
  // incomplete, and the others' bounded waits report the failure.
  __threadfence_system();
  const double flag = ld_volatile(&st->nonfinite_accum) != 0u ? 1.0 : 0.0;
  const uint64_t slot = uint64_t(rank) * (n_chunks + 1) + n_chunks;
  for (int q = 0; q < world; ++q) pt.gathered[q][slot] = flag;
  __threadfence_system();
  if (ld_volatile(&st->kernel_error) == 0u)
    for (int q = 0; q < world; ++q)
      *reinterpret_cast<volatile uint32_t*>(pt.flags[q] + kSlotPartials * kMaxRanks + rank) =
          epoch;
  st->nonfinite_accum = 0u;
  st->blocks_done = 0u;
  __threadfence_system();
}

// Fold of one double per consumer thread (256, named barrier 1; the producer
// warp never takes part); result valid in consumer thread 0.
__device__ __forceinline__ double consumer_fold(double v, double* warp_sums) {
#pragma unroll
  for (int off = 16; off >= 1; off >>= 1) v = __dadd_rn(v, __shfl_down_sync(kFull, v, off));
  const int lane = threadIdx.x & 31;
  const int warp = threadIdx.x >> 5;
  if (lane == 0) warp_sums[warp] = v;
  asm volatile("bar.sync 1, %0;" ::"n"(kBulkConsumers) : "memory");
  double r = 0.0;
  if (threadIdx.x == 0) {
    double w[kBulkConsumers / 32];
#pragma unroll
    for (int i = 0; i < int(kBulkConsumers / 32); ++i) w[i] = warp_sums[i];
#pragma unroll
    for (int off = 4; off >= 1; off >>= 1) {
#pragma unroll
      for (int i = 0; i < off; ++i) w[i] = __dadd_rn(w[i], w[i + off]);
    }
    r = w[0];
  }
  asm volatile("bar.sync 1, %0;" ::"n"(kBulkConsumers) : "memory");
  return r;
}

__global__ void __launch_bounds__(kBulkThreads)
    zero1_peer_update_kernel(const float* __restrict__ gsum, uint64_t n, uint64_t elem_base,
                             float* __restrict__ master, float* __restrict__ mom,
                             float* __restrict__ var, uint16_t* __restrict__ w16,
                             const uint64_t* __restrict__ offsets,
                             const uint8_t* __restrict__ decay,
                             const uint32_t* __restrict__ tile_first, AdamwParams p,
                             DeviceStepState* st, DeviceScaler* scaler, PeerTable pt,
                             PeerStores ps, int rank, int world, uint32_t per_rank,
                             uint32_t epoch, FinalizeParams fp, uint64_t timeout_ns) {
  using Stage = BulkStage<float>;
  extern __shared__ __align__(128) uint8_t smem[];
  __shared__ double warp_sums[kBulkConsumers / 32];
  __shared__ float s_clip;
  __shared__ uint32_t s_go;
  __shared__ uint32_t s_stop;
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + size_t(kBulkStages) * Stage::kBytes);
  uint64_t* empty_bar = full_bar + kBulkStages;
  uint8_t* staging = smem + size_t(kBulkStages) * Stage::kBytes + kBarrierBytes;
  if (threadIdx.x == 0) {
    for (uint32_t s = 0; s < kBulkStages; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], kBulkConsumers / 32);
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    s_go = 0u;
    s_stop = 0u;
  }
  __syncthreads();
  // The reduce kernel's outcome: this kernel may start while the reduce's
  // last blocks still run (programmatic launch), so it is read after waiting
  // for the reduce grid; only the producer warp's loads go ahead without it.
  __shared__ uint32_t s_prior_ok;
  __shared__ float s_scale;
  if (threadIdx.x == 0) {
    pdl_wait();
    s_prior_ok = st->kernel_error == 0u ? 1u : 0u;
    s_scale = st->loss_scale_used;
  }
  __syncthreads();
  const bool prior_ok = s_prior_ok != 0u;
  const float scale = s_scale;
  const uint64_t n_full = n / kBulkTile;
  const uint64_t mine = n_full > blockIdx.x ? (n_full - 1u - blockIdx.x) / gridDim.x + 1u : 0u;
  bool ok = true;
  bool bad = false;
  uint32_t i = 0;  // producer: tiles issued
  if (threadIdx.x >= kBulkConsumers) {
    // Producer warp: once the reduce kernel has completed (its sums are this
    // kernel's input), lane 0 starts streaming this block's first tiles while
    // the consumers finalize (those loads do not depend on the clip); it stops
    // once the consumers have decided not to update.
    if (threadIdx.x == kBulkConsumers) {
      pdl_wait();
      for (uint64_t tile = blockIdx.x; tile < n_full; tile += gridDim.x, ++i) {
        const uint32_t s = i % kBulkStages;
        if (i >= kBulkStages) {
          if (!mbar_wait(&empty_bar[s], ((i / kBulkStages) - 1u) & 1u)) {
            ok = false;
            break;
          }
          if (*reinterpret_cast<volatile uint32_t*>(&s_stop)) break;
        }
        uint8_t* base = smem + size_t(s) * Stage::kBytes;
        const uint64_t e0 = tile * kBulkTile;
        mbar_arrive_expect_tx(&full_bar[s], Stage::kBytes);
        bulk_load(base, gsum + e0, Stage::kG, &full_bar[s]);
        bulk_load(base + Stage::kG, master + e0, Stage::kF, &full_bar[s]);
        bulk_load(base + Stage::kG + Stage::kF, mom + e0, Stage::kF, &full_bar[s]);
        bulk_load(base + Stage::kG + 2 * Stage::kF, var + e0, Stage::kF, &full_bar[s]);
      }
    }
  } else {
    const uint32_t t = threadIdx.x;
    // Finalize: wait (bounded) for every rank's partials, reduce them with the
    // single-replica tree, decide.
    bool wok = prior_ok;
    if (wok && t < static_cast<unsigned>(world)) {
      wok = wait_epoch(pt.flags[rank] + kSlotPartials * kMaxRanks + t, epoch, st, timeout_ns);
      if (!wok) atomicOr(&st->kernel_error, 2u);
      __threadfence_system();  // acquire rank t's partials; the barrier orders the others
    }
    if (consumers_all(wok)) {
      const PartialsView view{pt.gathered[rank], per_rank, per_rank + 1};
      const double sum =
          consumer_fold(finalize_lane_sum(view, uint32_t(world) * per_rank, t), warp_sums);
      if (t == 0) {
        uint32_t nonfinite = 0u;
        for (int q = 0; q < world; ++q)
          nonfinite |= __ldcg(pt.gathered[rank] + uint64_t(q) * (per_rank + 1) + per_rank) != 0.0
                           ? 1u
                           : 0u;
        // Only block 0 reads and writes the scaler; the clip and the skip
        // decision do not depend on the scaler's step count.
        const StepDecision d = decide_step(
            sum, nonfinite, scale, fp.dynamic && blockIdx.x == 0 ? scaler->good_steps : 0u, fp);
        if (blockIdx.x == 0) {
          write_decision(d, sum, nonfinite, scale, st, scaler, fp);
          __threadfence();
        }
        s_clip = d.clip_apply;
        s_go = d.skipped ? 0u : 1u;
      }
    }
    if (t == 0 && s_go == 0u) s_stop = 1u;
    asm volatile("bar.sync 1, %0;" ::"n"(kBulkConsumers) : "memory");
    if (s_go == 0u) {
      // No update: take back the tiles the producer already started (each
      // stage's first use), so no copy lands after the block exits.
      const uint32_t started = mine < kBulkStages ? uint32_t(mine) : kBulkStages;
      for (uint32_t u = 0; u < started; ++u) {
        ok &= mbar_wait(&full_bar[u], 0u);
        __syncwarp();
        if ((t & 31) == 0) mbar_arrive(&empty_bar[u]);
      }
    } else {
      const ScaleInfo sc = decode_scale(scale);
      const float clip = s_clip;
      ok = sc.mul ? bulk_consume<float, true, true>(smem, full_bar, empty_bar, staging, n_full,
                                                    elem_base, master, mom, var, w16, offsets,
                                                    decay, tile_first, p, sc, clip, ps, bad)
                  : bulk_consume<float, false, true>(smem, full_bar, empty_bar, staging, n_full,
                                                     elem_base, master, mom, var, w16, offsets,
                                                     decay, tile_first, p, sc, clip, ps, bad);
      if (t == 0) {
        bulk_wait_all();  // the weight stores are complete before the barrier
        asm volatile("fence.proxy.async;" ::: "memory");
      }
      if (blockIdx.x == 0) {  // ragged tail after the last whole tile
        for (uint64_t e = n_full * kBulkTile + t; e < n; e += kBulkConsumers) {
          uint32_t k = __ldg(tile_first + e / kTileElems);
          const float wd = decay_of(elem_base + e, k, offsets, decay, p);
          const float gv = __fmul_rn(
              sc.mul ? unscale<true>(gsum[e], sc) : unscale<false>(gsum[e], sc), clip);
          float m = mom[e], v = var[e];
          const float t1 = adamw_elem(master[e], gv, m, v, wd, p, bad);
          master[e] = t1;
          mom[e] = m;
          var[e] = v;
          const uint16_t b = bf16_rne_bits(t1);
          w16[e] = b;
#pragma unroll
          for (uint32_t q = 0; q < uint32_t(kMaxRanks); ++q)
            if (q < ps.count) ps.w16[q][e] = b;
        }
      }
    }
  }
  // Peer stores before the block counts as done: thread 0's bulk stores, and
  // the ragged tail's plain stores in block 0.
  if (blockIdx.x == 0 || threadIdx.x == 0) __threadfence_system();
  if (__syncthreads_or(ok ? 0 : 1) && threadIdx.x == kBulkConsumers)
    for (uint32_t u = i > kBulkStages ? i - kBulkStages : 0u; u < i; ++u)
      mbar_wait(&full_bar[u % kBulkStages], (u / kBulkStages) & 1u);
  if (threadIdx.x != 0) {
    if (bad) atomicOr(&st->result_nonfinite, 1u);
    return;
  }
  if (!ok) atomicOr(&st->kernel_error, 1u);
  if (bad) atomicOr(&st->result_nonfinite, 1u);
  // Weight barrier: the last block to finish announces this rank's weights
  // (every block's stores completed and were fenced before it counted) and
  // waits for every rank's.  Without an update nothing was stored, and after a
  // failure it only announces.
  __threadfence_system();
  if (atomicAdd(&st->blocks_done, 1u) != gridDim.x - 1) return;
  __threadfence_system();
  const bool failed = ld_volatile(&st->kernel_error) != 0u;
  if (s_go) {
    for (int q = 0; q < world; ++q)
      *reinterpret_cast<volatile uint32_t*>(pt.flags[q] + kSlotWeights * kMaxRanks + rank) =
          epoch;
    if (!failed)
      for (int q = 0; q < world; ++q)
        if (!wait_epoch(pt.flags[rank] + kSlotWeights * kMaxRanks + q, epoch, st, timeout_ns)) {
          atomicOr(&st->kernel_error, 2u);
          break;
        }
  }
  st->blocks_done = 0u;
  __threadfence_system();
}

int sm_count(int device) {
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
      sms <= 0)
    sms = 148;
  return sms;
}

int current_sms() {
  int device = 0;
  if (cudaGetDevice(&device) != cudaSuccess) device = 0;
  return sm_count(device);
}

}  // namespace

int norm_bulk_grid(int device) {
  const int bytes = int(norm_bulk_smem_bytes());
  cudaFuncSetAttribute(norm_bulk_kernel<float>, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  cudaFuncSetAttribute(norm_bulk_kernel<uint16_t>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       bytes);
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, norm_bulk_kernel<uint16_t>,
                                                    kTreeThreads, bytes) != cudaSuccess ||
      per_sm <= 0)
    per_sm = 1;
  return sm_count(device) * per_sm;
}

int norm_partials_grid(int device) {
  int per_sm = 0;
  if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, norm_partials_kernel<uint16_t>,
                                                    kTreeThreads, 0) != cudaSuccess ||
      per_sm <= 0)
    per_sm = 4;
  return sm_count(device) * per_sm;
}

namespace {
template <typename GT>
void allow_bulk_smem() {
  cudaFuncSetAttribute(adamw_update_bulk_kernel<GT>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                       int(bulk_smem_bytes<GT, false>()));
}

template <typename GT>
int update_blocks_per_sm() {
  int per_sm = 0;
  cudaError_t e;
  if constexpr (kUpdateBulk) {
    allow_bulk_smem<GT>();
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, adamw_update_bulk_kernel<GT>,
                                                      kBulkThreads, bulk_smem_bytes<GT, false>());
  } else {
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, adamw_update_kernel<GT, false>,
                                                      kUpdateThreads, 0);
  }
  return (e != cudaSuccess || per_sm <= 0) ? (kUpdateBulk ? 1 : 2) : per_sm;
}

template <typename GT>
cudaError_t launch_update_typed(const void* grads, uint64_t n, uint64_t elem_base, float* master,
                                float* moment, float* variance, uint16_t* w16,
                                const uint64_t* offsets, const uint8_t* decay,
                                const uint32_t* tile_first, const AdamwParams& p,
                                DeviceStepState* st, int grid, cudaStream_t stream) {
  const GT* g = static_cast<const GT*>(grads);
  if constexpr (kUpdateBulk) {
    const uint64_t tiles = n / kBulkTile;
    const unsigned blocks =
        static_cast<unsigned>(tiles == 0 ? 1 : (uint64_t(grid) < tiles ? uint64_t(grid) : tiles));
    // Programmatic stream serialization: may start before the kernel ahead of
    // it on the stream completes, if that kernel triggers (the norm pass does).
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(kBulkThreads);
    cfg.dynamicSmemBytes = bulk_smem_bytes<GT, false>();
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, adamw_update_bulk_kernel<GT>, g, n, elem_base, master, moment,
                              variance, w16, offsets, decay, tile_first, p, st);
  } else {
    const uint64_t tiles = (n + kTileElems - 1) / kTileElems;
    const unsigned blocks =
        static_cast<unsigned>(uint64_t(grid) < tiles ? uint64_t(grid) : tiles);
    adamw_update_kernel<GT, false><<<blocks, kUpdateThreads, 0, stream>>>(
        g, n, elem_base, master, moment, variance, w16, offsets, decay, tile_first, p, st,
        PeerStores{});
    return cudaGetLastError();
  }
}
}  // namespace

int adamw_update_grid(int device, int dtype) {
  const int per_sm = dtype == 0 ? update_blocks_per_sm<float>() : update_blocks_per_sm<uint16_t>();
  return sm_count(device) * per_sm;
}

cudaError_t launch_norm_partials(int dtype, const void* grads, uint64_t n, uint64_t chunk_begin,
                                 uint32_t n_chunks, DeviceScaler* scaler, double* partials,
                                 DeviceStepState* st, const FinalizeParams& fp, int grid,
                                 cudaStream_t stream) {
  if (n_chunks == 0) return cudaErrorInvalidValue;
  if constexpr (kNormBulk) {
    // Persistent: `grid` (from norm_bulk_grid) blocks walk the chunks.
    const unsigned blocks = static_cast<unsigned>(uint32_t(grid) < n_chunks ? grid : n_chunks);
    if (dtype == 0)
      norm_bulk_kernel<float><<<blocks, kTreeThreads, norm_bulk_smem_bytes(), stream>>>(
          static_cast<const float*>(grads), n, chunk_begin, n_chunks, scaler, partials, st, fp);
    else
      norm_bulk_kernel<uint16_t><<<blocks, kTreeThreads, norm_bulk_smem_bytes(), stream>>>(
          static_cast<const uint16_t*>(grads), n, chunk_begin, n_chunks, scaler, partials, st,
          fp);
    return cudaGetLastError();
  }
  // One block per chunk: the block scheduler balances the ragged last wave.
  const unsigned blocks = n_chunks;
  if (dtype == 0)
    norm_partials_kernel<float><<<blocks, kTreeThreads, 0, stream>>>(
        static_cast<const float*>(grads), n, chunk_begin, n_chunks, scaler, partials, st, fp);
  else
    norm_partials_kernel<uint16_t><<<blocks, kTreeThreads, 0, stream>>>(
        static_cast<const uint16_t*>(grads), n, chunk_begin, n_chunks, scaler, partials, st, fp);
  return cudaGetLastError();
}

cudaError_t launch_adamw_update(int dtype, const void* grads, uint64_t n, uint64_t elem_base,
                                float* master, float* moment, float* variance, uint16_t* w16,
                                const uint64_t* offsets, const uint8_t* decay,
                                const uint32_t* tile_first_tensor, const AdamwParams& p,
                                DeviceStepState* st, int grid, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  if (dtype == 0)
    return launch_update_typed<float>(grads, n, elem_base, master, moment, variance, w16, offsets,
                                      decay, tile_first_tensor, p, st, grid, stream);
  return launch_update_typed<uint16_t>(grads, n, elem_base, master, moment, variance, w16,
                                       offsets, decay, tile_first_tensor, p, st, grid, stream);
}

cudaError_t launch_zero1_reduce(int dtype, const void* recv, uint32_t ranks, uint64_t stride,
                                uint64_t n_valid, uint32_t n_chunks, const DeviceScaler* scaler,
                                const FinalizeParams& fp, float* gsum, double* send,
                                DeviceStepState* st, int grid, cudaStream_t stream) {
  if (n_chunks == 0) return cudaErrorInvalidValue;
  const unsigned blocks = static_cast<unsigned>(grid < int(n_chunks) ? grid : int(n_chunks));
  if (dtype == 0)
    zero1_reduce_kernel<float><<<blocks, kTreeThreads, 0, stream>>>(
        static_cast<const float*>(recv), ranks, stride, n_valid, n_chunks, scaler, fp, gsum, send,
        st);
  else
    zero1_reduce_kernel<uint16_t><<<blocks, kTreeThreads, 0, stream>>>(
        static_cast<const uint16_t*>(recv), ranks, stride, n_valid, n_chunks, scaler, fp, gsum,
        send, st);
  return cudaGetLastError();
}

cudaError_t launch_zero1_finalize(const double* gathered, uint32_t ranks, uint32_t per_rank,
                                  DeviceScaler* scaler, DeviceStepState* st,
                                  const FinalizeParams& fp, cudaStream_t stream) {
  zero1_finalize_kernel<<<1, kTreeThreads, 0, stream>>>(gathered, ranks, per_rank, scaler, st,
                                                        fp);
  return cudaGetLastError();
}

namespace {
// Largest power of two of tree rows per rank such that one stage (every
// rank's rows) stays within kPeerStageTarget; at least one row.
uint32_t peer_rows_per_stage(int dtype, int world) {
  const uint32_t row = kTreeThreads * kVec * (dtype == 0 ? 4u : 2u);
  const uint32_t fit = kPeerStageTarget / (row * uint32_t(world));
  uint32_t r = 1;
  while (r * 2 <= fit && r * 2 <= kChunkIters) r *= 2;
  return r;
}

size_t peer_reduce_smem(int dtype, int world) {
  const uint32_t row = kTreeThreads * kVec * (dtype == 0 ? 4u : 2u);
  return size_t(kPeerStages) * peer_rows_per_stage(dtype, world) * row * uint32_t(world) +
         kBarrierBytes;
}
}  // namespace

int prepare_peer_kernels(int device, int world) {
  cudaError_t e = cudaFuncSetAttribute(zero1_peer_reduce_kernel<float, 0, 0>,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       int(peer_reduce_smem(0, world)));
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(zero1_peer_reduce_kernel<uint16_t, 0, 0>,
                             cudaFuncAttributeMaxDynamicSharedMemorySize,
                             int(peer_reduce_smem(1, world)));
  const int bytes = int(bulk_smem_bytes<float, true>());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(zero1_peer_update_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             bytes);
  int per_sm = 0;
  if (e == cudaSuccess)
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, zero1_peer_update_kernel,
                                                      kBulkThreads, bytes);
  if (e != cudaSuccess || per_sm <= 0) return -1;
  return sm_count(device) * per_sm;
}

cudaError_t launch_zero1_peer_reduce(int dtype, const PeerTable& pt, int rank, int world,
                                     uint64_t shard_begin, uint64_t n_valid, uint32_t n_chunks,
                                     const DeviceScaler* scaler, const FinalizeParams& fp,
                                     float* gsum, uint32_t epoch, DeviceStepState* st,
                                     uint64_t timeout_ns, cudaStream_t stream) {
  if (n_chunks == 0 || world < 1 || world > kMaxRanks) return cudaErrorInvalidValue;
  if constexpr (kPeerLoads) {
    // Plain loads: B rows x R ranks in flight per thread (8 loads per batch).
#define SLM_PEER_LAUNCH(GT, B, R, M)                                                          \
  zero1_peer_reduce_kernel<GT, B, R, M><<<n_chunks, kTreeThreads, 0, stream>>>(               \
      pt, rank, world, shard_begin, n_valid, n_chunks, scaler, fp, gsum, 0u, 0u, epoch, st,  \
      timeout_ns)
    if (dtype == 0) {
      if (world <= 2) SLM_PEER_LAUNCH(float, 4, 2, 0);
      else if (world <= 4) SLM_PEER_LAUNCH(float, 2, 4, 0);
      else SLM_PEER_LAUNCH(float, 1, 8, 0);
    } else {
      if (world <= 2) SLM_PEER_LAUNCH(uint16_t, SLM_PEER_BATCH2, 2, SLM_PEER_MINBLOCKS2);
      else if (world <= 4) SLM_PEER_LAUNCH(uint16_t, 2, 4, 0);
      else SLM_PEER_LAUNCH(uint16_t, SLM_PEER_BATCH8, 8, 0);
    }
#undef SLM_PEER_LAUNCH
    return cudaGetLastError();
  }
  const uint32_t rows = peer_rows_per_stage(dtype, world);
  const size_t smem = peer_reduce_smem(dtype, world);
  const uint32_t stage = uint32_t((smem - kBarrierBytes) / kPeerStages);
  if (dtype == 0)
    zero1_peer_reduce_kernel<float, 0, 0><<<n_chunks, kTreeThreads, smem, stream>>>(
        pt, rank, world, shard_begin, n_valid, n_chunks, scaler, fp, gsum, rows, stage, epoch, st,
        timeout_ns);
  else
    zero1_peer_reduce_kernel<uint16_t, 0, 0><<<n_chunks, kTreeThreads, smem, stream>>>(
        pt, rank, world, shard_begin, n_valid, n_chunks, scaler, fp, gsum, rows, stage, epoch, st,
        timeout_ns);
  return cudaGetLastError();
}

cudaError_t launch_zero1_peer_update(const float* gsum, uint64_t n, uint64_t elem_base,
                                     float* master, float* moment, float* variance, uint16_t* w16,
                                     const uint64_t* offsets, const uint8_t* decay,
                                     const uint32_t* tile_first_tensor, const AdamwParams& p,
                                     DeviceStepState* st, DeviceScaler* scaler,
                                     const PeerTable& pt, const PeerStores& ps, int rank,
                                     int world, uint32_t per_rank, uint32_t epoch,
                                     const FinalizeParams& fp, uint64_t timeout_ns, int grid,
                                     cudaStream_t stream) {
  const uint64_t tiles = n / kBulkTile;
  const unsigned blocks =
      static_cast<unsigned>(tiles == 0 ? 1 : (uint64_t(grid) < tiles ? uint64_t(grid) : tiles));
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks);
  cfg.blockDim = dim3(kBulkThreads);
  cfg.dynamicSmemBytes = bulk_smem_bytes<float, true>();
  cfg.stream = stream;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, zero1_peer_update_kernel, gsum, n, elem_base, master, moment,
                            variance, w16, offsets, decay, tile_first_tensor, p, st, scaler, pt,
                            ps, rank, world, per_rank, epoch, fp, timeout_ns);
}

cudaError_t launch_accumulate(int dtype, float* acc, const void* micro, uint64_t n,
                              int overwrite, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  const uint64_t vecs = (n + kVec - 1) / kVec;
  const uint64_t want = (vecs + 255) / 256;
  const unsigned blocks = static_cast<unsigned>(want < 148u * 16u ? want : 148u * 16u);
  if (dtype == 0)
    accumulate_kernel<float><<<blocks, 256, 0, stream>>>(acc, static_cast<const float*>(micro),
                                                         n, overwrite);
  else
    accumulate_kernel<uint16_t><<<blocks, 256, 0, stream>>>(
        acc, static_cast<const uint16_t*>(micro), n, overwrite);
  return cudaGetLastError();
}

cudaError_t launch_accumulate_norm(int dtype, float* acc, const void* micro, uint64_t n,
                                   int overwrite, uint32_t n_chunks, DeviceScaler* scaler,
                                   double* partials, DeviceStepState* st,
                                   const FinalizeParams& fp, cudaStream_t stream) {
  if (n_chunks == 0) return cudaErrorInvalidValue;
  if (dtype == 0)
    accumulate_norm_kernel<float><<<n_chunks, kTreeThreads, 0, stream>>>(
        acc, static_cast<const float*>(micro), n, overwrite, n_chunks, scaler, partials, st, fp);
  else
    accumulate_norm_kernel<uint16_t><<<n_chunks, kTreeThreads, 0, stream>>>(
        acc, static_cast<const uint16_t*>(micro), n, overwrite, n_chunks, scaler, partials, st,
        fp);
  return cudaGetLastError();
}

cudaError_t launch_init_from_master(float* master, float* moment, float* variance, uint16_t* w16,
                                    uint64_t n, cudaStream_t stream) {
  cudaError_t e = cudaMemsetAsync(moment, 0, n * sizeof(float), stream);
  if (e != cudaSuccess) return e;
  e = cudaMemsetAsync(variance, 0, n * sizeof(float), stream);
  if (e != cudaSuccess) return e;
  init_from_master_kernel<<<current_sms() * 8, 256, 0, stream>>>(master, w16, n);
  return cudaGetLastError();
}

cudaError_t launch_reference_clip(const float* g, uint64_t n, DeviceStepState* st,
                                  cudaStream_t stream, void* workspace, size_t workspace_bytes) {
  SeqClipOut out{st, nullptr, nullptr, nullptr};
  return launch_sequential_clip(g, n, out, &st->kernel_error, stream, nullptr, false, true,
                                workspace, workspace_bytes);
}

size_t seq_clip_workspace_bytes(uint64_t n) {
  const uint64_t nw = (n + kSeqWindow - 1) / kSeqWindow;
  const uint64_t bytes = nw * (sizeof(double) + sizeof(int32_t) + kSeqCand * sizeof(uint32_t) + 1);
  return size_t((bytes + 15) & ~uint64_t(15));
}

cudaError_t launch_sequential_clip(const float* g, uint64_t n, const SeqClipOut& out,
                                   uint32_t* kernel_error, cudaStream_t stream, SeqCarry* carry,
                                   bool resume, bool finish, void* workspace,
                                   size_t workspace_bytes) {
  if ((resume || !finish) && carry == nullptr) return cudaErrorInvalidValue;
  const uint64_t n_windows = (n + kSeqWindow - 1) / kSeqWindow;
  if (workspace != nullptr && n_windows > 0) {
    if (workspace_bytes < seq_clip_workspace_bytes(n) ||
        reinterpret_cast<uintptr_t>(workspace) % 16 != 0)
      return cudaErrorInvalidValue;
    uint8_t* base = static_cast<uint8_t*>(workspace);
    SeqWorkspace ws;
    ws.total = reinterpret_cast<uint32_t*>(base);
    ws.sums = reinterpret_cast<double*>(base + n_windows * kSeqCand * sizeof(uint32_t));
    ws.base = reinterpret_cast<int32_t*>(base + n_windows * (kSeqCand * sizeof(uint32_t) +
                                                            sizeof(double)));
    ws.flags = base + n_windows * (kSeqCand * sizeof(uint32_t) + sizeof(double) + sizeof(int32_t));
    const uint64_t cap = uint64_t(current_sms()) * 8;
    const unsigned grid = unsigned(n_windows < cap ? n_windows : cap);
    seqclip_sums_kernel<<<grid, kSeqPassThreads, 0, stream>>>(g, n, n_windows, ws);
    seqclip_prefix_kernel<<<1, kSeqThreads, 0, stream>>>(n_windows, ws, carry, resume ? 1 : 0,
                                                         !finish ? 1 : 0);
    seqclip_candidates_kernel<<<grid, kSeqPassThreads, 0, stream>>>(g, n, n_windows, ws);
    seqclip_chain_kernel<<<1, kSeqThreads, 0, stream>>>(g, n, n_windows, ws, out, kernel_error,
                                                        carry, resume ? 1 : 0, finish ? 1 : 0);
    return cudaGetLastError();
  }
  const int bytes = int(kSeqStages * kSeqWindowBytes + kBarrierBytes);
  cudaError_t e = cudaFuncSetAttribute(sequential_clip_kernel,
                                       cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return e;
  sequential_clip_kernel<<<1, kSeqThreads, bytes, stream>>>(g, n, out, kernel_error, carry,
                                                            resume ? 1 : 0, finish ? 1 : 0);
  return cudaGetLastError();
}

cudaError_t launch_export_f32(const uint16_t* w16, float* dst, uint64_t n, cudaStream_t stream) {
  if (n == 0) return cudaSuccess;
  export_f32_kernel<<<current_sms() * 8, 256, 0, stream>>>(w16, dst, n);
  return cudaGetLastError();
}

cudaError_t launch_validate_state(const float* master, const float* moment,
                                  const float* variance, const uint16_t* w16, uint64_t n,
                                  uint32_t* bad_flag, cudaStream_t stream) {
  validate_state_kernel<<<current_sms() * 8, 256, 0, stream>>>(master, moment, variance, w16, n,
                                                             bad_flag);
  return cudaGetLastError();
}

}  // namespace slmopt
