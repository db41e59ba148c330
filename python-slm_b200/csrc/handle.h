// The optimizer handle and host helpers shared by the C-ABI translation units
// (api.cu: single replica; zero1.cu: ZeRO-1 data parallel over NCCL).
#pragma once

#include "../../include/slmopt.h"
#include "slmopt_internal.h"

#include <cuda_runtime.h>

#include <cmath>
#include <cstring>
#include <string>
#include <vector>

namespace slmopt {

// Last failure message of this thread (slm_last_error_message).
extern thread_local std::string g_last_error;

inline int fail(int status, const std::string& msg) {
  g_last_error = msg;
  return status;
}

inline uint32_t f32_bits(float v) {
  uint32_t b;
  std::memcpy(&b, &v, 4);
  return b;
}

inline bool finite_f32(float v) { return std::isfinite(v); }

// Restores the caller's current device on scope exit.
struct DeviceGuard {
  int prev = -1;
  bool ok = false;
  explicit DeviceGuard(int device) {
    if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
    ok = cudaSetDevice(device) == cudaSuccess;
  }
  ~DeviceGuard() {
    if (prev >= 0) cudaSetDevice(prev);
  }
};

// Host-side step helpers implemented in api.cu.
float powi_f32(float base, int32_t exponent);
AdamwParams adamw_params(const slm_step_config* cfg);

}  // namespace slmopt

namespace slmopt {
// Optional device timing of each slm_opt_step by phase (slm_opt_phase_timing):
// CUDA events recorded on the step's stream at the phase boundaries.
struct PhaseTimer {
  static constexpr int kMaxMarks = 8;
  bool enabled = false;
  bool created = false;
  cudaEvent_t ev[kMaxMarks] = {};
  int marks = 0;     // events recorded so far for the step being enqueued
  int finished = 0;  // events of the last complete step, not yet folded into acc
  double acc[kMaxMarks - 1] = {};
  uint64_t steps = 0;
  uint32_t phases = 0;
  // Which entry point the sums describe (kStepCall, kApplyUpdateCall): a call
  // of the other kind restarts them, so the phase names always fit the sums.
  int kind = 0;
  int finished_kind = 0;
};
constexpr int kStepCall = 0;
constexpr int kApplyUpdateCall = 1;
}  // namespace slmopt

struct slm_opt_handle {
  int device = 0;
  uint64_t P = 0;  // global parameter count
  std::vector<std::string> names;
  std::vector<uint64_t> offsets;  // n_tensors + 1 global offsets
  std::vector<uint8_t> decay;
  // Elements [shard_begin, shard_begin + shard_len) of the flat buffer are
  // owned here (the whole buffer for a single replica).
  uint64_t shard_begin = 0, shard_len = 0;

  float* master = nullptr;  // shard_len
  float* m1 = nullptr;      // shard_len
  float* m2 = nullptr;      // shard_len
  uint16_t* w16 = nullptr;  // full flat buffer (padded to world * shard_stride)
  uint64_t* d_offsets = nullptr;
  uint8_t* d_decay = nullptr;
  uint32_t* d_tile_first = nullptr;  // per 4,096-element tile of the shard
  double* d_partials = nullptr;
  uint32_t n_chunks = 0;  // chunks of the whole flat buffer
  slmopt::DeviceStepState* d_state = nullptr;
  slmopt::DeviceScaler* d_scaler = nullptr;
  uint32_t* d_flag = nullptr;
  void* d_staging = nullptr;
  size_t staging_bytes = 0;
  slmopt::DeviceStepState* h_state = nullptr;  // pinned

  int grid_norm = 0;       // resident blocks of the per-chunk tree kernels
  int grid_norm_bulk = 0;  // persistent grid of the bulk-copy norm pass
  int grid_update[2] = {0, 0};
  // Gradients seen by the last norm pass (consumed by the update pass).
  const void* pass_grads = nullptr;
  int pass_dtype = -1;
  cudaStream_t pending_stream = nullptr;
  bool pending = false;
  std::string last_error = "no error";

  // Pipelined gradient uploads (slm_opt_upload_gradients / slm_opt_step_uploaded):
  // two device slots filled from host memory on the handle's own copy stream.
  struct UploadSlot {
    void* dev = nullptr;
    size_t bytes = 0;
    int dtype = -1;
    bool filled = false;             // uploaded, not yet handed to a step
    bool consumed_recorded = false;  // `consumed` marks the last step that read it
    cudaEvent_t uploaded = nullptr;
    cudaEvent_t consumed = nullptr;
  } up[2];
  cudaStream_t copy_stream = nullptr;
  int next_up = 0;

  // Pageable host gradients (slm_opt_apply_update's slice, slm_opt_step on
  // host memory that is not pinned) travel through a ring of pinned slots
  // filled by host threads, one DMA per slot on copy_stream (stage_pageable).
  struct PinnedRing {
    static constexpr int kSlots = 3;
    static constexpr size_t kSlotBytes = size_t(32) << 20;  // 8M f32: whole clip windows
    void* slot[kSlots] = {};
    cudaEvent_t drained[kSlots] = {};  // the slot's last DMA has read it
    bool used[kSlots] = {};
  } ring;
  slmopt::SeqCarry* d_seq_carry = nullptr;  // sequential clip's state between slices
  void* d_seq_ws = nullptr;                 // its window summaries (all P gradients)
  size_t seq_ws_bytes = 0;

  // ---- ZeRO-1 (world > 1) ---------------------------------------------------
  int rank = 0, world = 1;
  void* comm = nullptr;            // ncclComm_t
  uint64_t shard_stride = 0;       // padded elements per rank (chunks_per_rank * 65,536)
  uint32_t chunks_per_rank = 0;
  void* d_recv = nullptr;          // world * shard_stride gradient elements
  size_t recv_bytes = 0;
  float* d_gsum = nullptr;         // rank-ordered f32 sums of this shard
  double* d_send = nullptr;        // chunks_per_rank partials + 1 flag
  double* d_gathered = nullptr;    // world * (chunks_per_rank + 1)
  uint32_t timeout_ms = 0;
  bool broken = false;             // a collective timed out and the comm was aborted
  // Peer-memory exchange (default when every rank could map every other
  // rank's buffers with CUDA IPC; otherwise the NCCL exchange above).
  int exchange = 0;                // SLM_ZERO1_NCCL or SLM_ZERO1_PEER
  void* d_gradbuf = nullptr;       // registered gradient buffer, P * 4 bytes, exported
  uint32_t* d_flags = nullptr;     // kFlagSlots * kMaxRanks arrival epochs, exported
  slmopt::PeerTable peers{};       // every rank's buffers as mapped here (own included)
  int grid_peer_update = 0;        // persistent grid of the peer-exchange update kernel
  void* opened[slmopt::kMaxRanks][4] = {};  // IPC mappings to close on destroy
  uint32_t epoch = 0;              // step counter shared (implicitly) by all ranks
  slmopt::PhaseTimer timer;

  bool sharded() const { return world > 1; }

  int err(int status, const std::string& msg) {
    last_error = msg;
    return slmopt::fail(status, msg);
  }
  int cuda(cudaError_t e, const char* what) {
    if (e == cudaSuccess) return SLM_OK;
    const int st = (e == cudaErrorMemoryAllocation) ? SLM_ERR_OUT_OF_MEMORY : SLM_ERR_CUDA;
    return err(st, std::string(what) + ": " + cudaGetErrorString(e));
  }
};

namespace slmopt {
// Phase timing: phase_begin starts a step (after folding in the previous
// complete one, which waits for it), phase_mark closes a phase, phase_end
// marks the step complete.  No-ops unless timing is enabled.
int phase_begin(slm_opt_handle* h, cudaStream_t s);
int phase_mark(slm_opt_handle* h, cudaStream_t s);
void phase_end(slm_opt_handle* h, int kind = kStepCall);
// Allocates the per-handle device state for [shard_begin, shard_begin+shard_len)
// with the bf16 buffer sized w16_elems; used by both create paths (api.cu).
int allocate_state(slm_opt_handle* h, uint64_t w16_elems);
// Validates the tensor table (non-empty, unique non-empty names) into h.
int build_table(slm_opt_handle* h, const slm_tensor_spec* table, uint32_t n_tensors);
int check_config(slm_opt_handle* h, const slm_step_config* cfg);
FinalizeParams finalize_params(const slm_opt_handle* h, const slm_step_config* cfg);
int read_state(slm_opt_handle* h, cudaStream_t s, DeviceStepState* out);
void fill_result(const DeviceStepState& s, slm_step_result* out);
// ZeRO-1 pieces (zero1.cu).
int zero1_step(slm_opt_handle* h, const void* grads, int dtype, int memory,
               const slm_step_config* cfg, cudaStream_t s);
int zero1_wait(slm_opt_handle* h, cudaStream_t s);
int zero1_gather(slm_opt_handle* h, const void* shard_src, size_t elem_bytes, void* dst_full,
                 cudaStream_t s);
int setup_peer_exchange(slm_opt_handle* h, cudaStream_t s);
void zero1_release(slm_opt_handle* h);
}  // namespace slmopt
