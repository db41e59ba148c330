// Internal declarations shared by the kernels and the C-ABI host code.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>

namespace slmopt {

// Fixed reduction tree of the global norm.  A chunk is 65,536 consecutive
// elements of the flat PARAM-001 buffer; its f64 partial is formed by a
// 256-thread block in which thread t owns, for k = 0..31, the 8 elements at
// chunk_base + k*2048 + t*8: their unscaled values are squared in f32, the 8
// squares summed pairwise in f32 ((q0+q1)+(q2+q3))+((q4+q5)+(q6+q7)), and the
// sums added in k order to the thread's f64 accumulator; each warp folds with
// shuffle offsets 16,8,4,2,1 and the 8 warp results fold with offsets 4,2,1.
// The partials of all chunks are reduced by the same shape (thread t adds
// partials t, t+256, ... in order).  The shape never depends on the grid, the
// device, the gradient dtype or the number of ranks, so the norm is
// bit-identical run to run, between the fp32 and bf16 paths and between one
// GPU and a ZeRO-1 group.
constexpr uint32_t kChunkElems = 65536;
constexpr uint32_t kTreeThreads = 256;
constexpr uint32_t kVec = 8;
constexpr uint32_t kChunkIters = kChunkElems / (kTreeThreads * kVec);  // 32

// Update kernel tiling: one 256-thread block step covers kTileElems elements
// (kUpdateUnroll 8-element vectors per thread).  The build may override the
// unroll and the minimum resident blocks per SM (register cap).
#ifndef SLM_UPDATE_UNROLL
#define SLM_UPDATE_UNROLL 2
#endif
#ifndef SLM_UPDATE_MIN_BLOCKS
#define SLM_UPDATE_MIN_BLOCKS 1
#endif
constexpr uint32_t kUpdateThreads = 256;
constexpr uint32_t kUpdateUnroll = SLM_UPDATE_UNROLL;
constexpr uint32_t kUpdateMinBlocks = SLM_UPDATE_MIN_BLOCKS;
constexpr uint32_t kTileElems = kUpdateThreads * kVec * kUpdateUnroll;
// Bulk-copy update kernel (SLM_UPDATE_BULK=1): a producer warp streams
// 2,048-element tiles of g / master / m / v into a ring of shared-memory stages
// with cp.async.bulk; 8 consumer warps compute from shared memory.
#ifndef SLM_UPDATE_BULK
#define SLM_UPDATE_BULK 1
#endif
#ifndef SLM_BULK_STAGES
#define SLM_BULK_STAGES 2
#endif
constexpr uint32_t kBulkTile = 2048;
constexpr uint32_t kBulkConsumers = 256;
constexpr uint32_t kBulkThreads = kBulkConsumers + 32;
constexpr uint32_t kBulkStages = SLM_BULK_STAGES;
constexpr bool kUpdateBulk = SLM_UPDATE_BULK != 0;
// Norm pass: vector loads issued together before their squares are added.
constexpr uint32_t kNormBatch = 8;
// Bulk-copy norm pass (SLM_NORM_BULK=1): a persistent grid streams each whole
// chunk through kNormStages shared-memory stages of kNormStageBytes.
#ifndef SLM_NORM_BULK
#define SLM_NORM_BULK 1
#endif
#ifndef SLM_NORM_STAGES
#define SLM_NORM_STAGES 6
#endif
constexpr bool kNormBulk = SLM_NORM_BULK != 0;
constexpr uint32_t kNormStages = SLM_NORM_STAGES;
constexpr uint32_t kNormStageBytes = 16384;

struct DeviceScaler {
  float scale;
  uint32_t good_steps;
};

// Step record in device memory.  The partial-sum kernel's last block fills it
// (norm, clip, skip decision, scaler update); the update kernel reads it and
// may set result_nonfinite; the host copies it out for slm_step_result.
struct __align__(16) DeviceStepState {
  double sum_squares;
  double grad_norm;
  float clip_scale;
  float clip_apply;
  float loss_scale_used;
  float next_loss_scale;
  uint32_t skipped;
  uint32_t nonfinite;
  uint32_t result_nonfinite;
  uint32_t rejected;
  uint32_t good_steps;
  int32_t status;
  // Accumulators owned by the partial-sum kernel, consumed and reset to zero by
  // its last block, so every launch starts from zero without a memset.
  uint32_t nonfinite_accum;
  uint32_t blocks_done;
  // Set when a bounded in-kernel wait gave up (never expected; reported as an
  // internal error instead of hanging the GPU).
  uint32_t kernel_error;
  uint32_t reserved[3];
};
static_assert(sizeof(DeviceStepState) == 80, "DeviceStepState layout");

// ZeRO-1 over peer memory: device addresses (mapped into this process with
// CUDA IPC) of every rank's gradient buffer, gathered-partials area, flag
// array and bf16 weights; index = rank, own buffers included.
constexpr int kMaxRanks = 8;
constexpr uint32_t kSlotGrads = 0;     // gradients of this step are written
constexpr uint32_t kSlotPartials = 1;  // partials delivered; peers done reading my gradients
constexpr uint32_t kSlotWeights = 2;   // bf16 weights delivered
constexpr uint32_t kFlagSlots = 3;
struct PeerTable {
  const void* grads[kMaxRanks];
  double* gathered[kMaxRanks];
  uint32_t* flags[kMaxRanks];
  uint16_t* w16[kMaxRanks];
};
// bf16 destinations an update kernel also writes (the peers' weight buffers at
// this shard's offset); count 0 for a single replica.
struct PeerStores {
  uint16_t* w16[kMaxRanks];
  uint32_t count;
};

struct FinalizeParams {
  float max_grad_norm;
  float min_clip_accept;
  int32_t apply_clip;
  int32_t nonfinite_policy;  // 0 skip, 1 error
  int32_t dynamic;           // read/update the device scaler
  uint32_t growth_interval;
  float static_scale;
  uint32_t total_chunks;     // partials reduced by the finalize tree
};

struct AdamwParams {
  float lr, beta1, beta2, omb1, omb2, bc1, bc2, eps, decay_weight, no_decay_weight;
};

// Status numbers mirrored from include/slmopt.h for device-side decisions.
constexpr int32_t kStatusOk = 0;
constexpr int32_t kStatusGradientNonfinite = 10;
constexpr int32_t kStatusNormNonfinite = 11;
constexpr int32_t kStatusResultNonfinite = 13;
constexpr int32_t kStatusGradientInvalid = 20;

// ---- launchers (kernels.cu) -------------------------------------------------
// dtype: 0 = f32, 1 = bf16 (raw u16 bits).
cudaError_t launch_norm_partials(int dtype, const void* grads, uint64_t n, uint64_t chunk_begin,
                                 uint32_t n_chunks, DeviceScaler* scaler, double* partials,
                                 DeviceStepState* st, const FinalizeParams& fp, int grid,
                                 cudaStream_t stream);
// Updates local elements [0, n); element i is global flat index elem_base + i
// (the tensor table holds global offsets).  grads/master/moment/variance/w16
// are all indexed by the local i.
cudaError_t launch_adamw_update(int dtype, const void* grads, uint64_t n, uint64_t elem_base,
                                float* master, float* moment, float* variance, uint16_t* w16,
                                const uint64_t* offsets, const uint8_t* decay,
                                const uint32_t* tile_first_tensor, const AdamwParams& p,
                                DeviceStepState* st, int grid, cudaStream_t stream);
// ZeRO-1 over peer memory (see zero1.cu): two kernels per step.
// The reduce: gradient barrier, rank-ordered sum of this shard's slices of
// every rank's gradient buffer (bulk copies over NVLink), unscale, chunk
// partials into every rank's gathered area, then the partials flag.
cudaError_t launch_zero1_peer_reduce(int dtype, const PeerTable& pt, int rank, int world,
                                     uint64_t shard_begin, uint64_t n_valid, uint32_t n_chunks,
                                     const DeviceScaler* scaler, const FinalizeParams& fp,
                                     float* gsum, uint32_t epoch, DeviceStepState* st,
                                     uint64_t timeout_ns, cudaStream_t stream);
// The update: finalize of all ranks' partials in every block, AdamW on the
// shard with the bf16 tiles stored to every rank, then the weight barrier.
cudaError_t launch_zero1_peer_update(const float* gsum, uint64_t n, uint64_t elem_base,
                                     float* master, float* moment, float* variance, uint16_t* w16,
                                     const uint64_t* offsets, const uint8_t* decay,
                                     const uint32_t* tile_first_tensor, const AdamwParams& p,
                                     DeviceStepState* st, DeviceScaler* scaler,
                                     const PeerTable& pt, const PeerStores& ps, int rank,
                                     int world, uint32_t per_rank, uint32_t epoch,
                                     const FinalizeParams& fp, uint64_t timeout_ns, int grid,
                                     cudaStream_t stream);
// Sets the peer kernels' shared-memory limits on the current device; returns
// the update kernel's persistent grid (-1 on failure).
int prepare_peer_kernels(int device, int world);
// ZeRO-1: rank-ordered sum of the received gradient slices + unscale + chunk
// partials (send[n_chunks] receives the non-finite flag), then the finalize of
// the all-gathered partials.
cudaError_t launch_zero1_reduce(int dtype, const void* recv, uint32_t ranks, uint64_t stride,
                                uint64_t n_valid, uint32_t n_chunks, const DeviceScaler* scaler,
                                const FinalizeParams& fp, float* gsum, double* send,
                                DeviceStepState* st, int grid, cudaStream_t stream);
cudaError_t launch_zero1_finalize(const double* gathered, uint32_t ranks, uint32_t per_rank,
                                  DeviceScaler* scaler, DeviceStepState* st,
                                  const FinalizeParams& fp, cudaStream_t stream);
// Micro-batch accumulation (acc = acc + micro, or acc = micro), and the last
// micro-batch fused with the norm pass over the accumulated values.
cudaError_t launch_accumulate(int dtype, float* acc, const void* micro, uint64_t n,
                              int overwrite, cudaStream_t stream);
cudaError_t launch_accumulate_norm(int dtype, float* acc, const void* micro, uint64_t n,
                                   int overwrite, uint32_t n_chunks, DeviceScaler* scaler,
                                   double* partials, DeviceStepState* st,
                                   const FinalizeParams& fp, cudaStream_t stream);
// f32 copy of the bf16 weights (n elements, both 16-byte aligned).
cudaError_t launch_export_f32(const uint16_t* w16, float* dst, uint64_t n, cudaStream_t stream);
// The reference's own clip check for the strict drop-in: a sequential f32
// sum of squares over g[0..n) (16-byte aligned), then min(1/sqrt(sum), 1);
// fills st as the norm pass would for a static scale of 1 without clipping.
cudaError_t launch_reference_clip(const float* g, uint64_t n, DeviceStepState* st,
                                  cudaStream_t stream, void* workspace = nullptr,
                                  size_t workspace_bytes = 0);
// The same sequential clip scale with its result sent elsewhere: into the step
// record (st != NULL) or into the three caller-provided device words.
struct SeqClipOut {
  DeviceStepState* st;
  float* sum;
  float* clip;
  int32_t* status;
};
// The running state of the sequential sum between launches over consecutive
// slices (each slice but the last a whole number of 8,192-term windows).
struct SeqCarry {
  int32_t E;          // the sum is m * 2^E
  uint32_t m;
  uint32_t sum_bad;   // the sum became non-finite (sum_bits holds it)
  float sum_bits;
  uint32_t gbad;      // a non-finite gradient was seen
  uint32_t reserved;
  double prefix;      // exact (f64) sum of the slices before, for the parallel form
};
constexpr uint64_t kSeqSliceAlign = 8192;  // terms per window of the sequential sum
// resume: start from *carry (else from zero); finish: write the result to
// `out` (else save the running state to *carry).  With a workspace of
// seq_clip_workspace_bytes(n) bytes (16-byte aligned) the windows are
// summarised by every SM first and one CTA chains the summaries; without one
// a single CTA streams all n terms.  Both give the same bits.
size_t seq_clip_workspace_bytes(uint64_t n);
cudaError_t launch_sequential_clip(const float* g, uint64_t n, const SeqClipOut& out,
                                   uint32_t* kernel_error, cudaStream_t stream,
                                   SeqCarry* carry = nullptr, bool resume = false,
                                   bool finish = true, void* workspace = nullptr,
                                   size_t workspace_bytes = 0);
cudaError_t launch_init_from_master(float* master, float* moment, float* variance, uint16_t* w16,
                                    uint64_t n, cudaStream_t stream);
cudaError_t launch_validate_state(const float* master, const float* moment,
                                  const float* variance, const uint16_t* w16, uint64_t n,
                                  uint32_t* bad_flag, cudaStream_t stream);
int norm_partials_grid(int device);
// Persistent grid of the bulk-copy norm pass (sets its shared-memory limit on
// the current device).
int norm_bulk_grid(int device);
int adamw_update_grid(int device, int dtype);

}  // namespace slmopt
