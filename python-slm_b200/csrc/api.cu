// C ABI of the optimizer step (include/slmopt.h): handle lifetime, state
// codec, the fused step, the strict apply_update drop-in, the state hash.
// The ZeRO-1 collectives live in zero1.cu.
#include "handle.h"
#include "hostcopy.h"
#include "sha256.h"

#include <algorithm>
#include <atomic>
#include <cstdio>
#include <cstdlib>
#include <memory>
#include <new>
#include <set>
#include <thread>

using namespace slmopt;

namespace slmopt {

thread_local std::string g_last_error = "no error";

// Rust f32::powi with a run-time exponent: LLVM lowers it to the
// compiler-builtins __powisf2 square-and-multiply loop (one f32 rounding per
// multiply, starting from the lowest exponent bit).  Computed once per step on
// the host; the kernels receive 1 - beta^t as a scalar.
float powi_f32(float base, int32_t exponent) {
  const bool recip = exponent < 0;
  uint32_t remaining = recip ? uint32_t(-int64_t(exponent)) : uint32_t(exponent);
  float product = 1.0f;
  for (;;) {
    if (remaining & 1u) product = product * base;
    remaining >>= 1;
    if (remaining == 0) break;
    base = base * base;
  }
  return recip ? 1.0f / product : product;
}

AdamwParams adamw_params(const slm_step_config* cfg) {
  AdamwParams p;
  p.lr = cfg->learning_rate;
  p.beta1 = cfg->beta1;
  p.beta2 = cfg->beta2;
  p.omb1 = 1.0f - cfg->beta1;
  p.omb2 = 1.0f - cfg->beta2;
  p.bc1 = 1.0f - powi_f32(cfg->beta1, int32_t(cfg->one_based_update));
  p.bc2 = 1.0f - powi_f32(cfg->beta2, int32_t(cfg->one_based_update));
  p.eps = cfg->epsilon;
  p.decay_weight = cfg->decay_weight;
  p.no_decay_weight = cfg->no_decay_weight;
  return p;
}

int check_config(slm_opt_handle* h, const slm_step_config* cfg) {
  if (!cfg) return h->err(SLM_ERR_INVALID_ARGUMENT, "cfg is NULL");
  // src/model/oracle.rs:519-531: a zero update index or non-finite lr/decay.
  if (cfg->one_based_update == 0 || cfg->one_based_update > 0x7fffffffu ||
      !finite_f32(cfg->learning_rate) || !finite_f32(cfg->decay_weight) ||
      !finite_f32(cfg->no_decay_weight))
    return h->err(SLM_ERR_MODEL_OPTIMIZER_INPUT_INVALID,
                  "OPT-001 requires finite state and a one-based update index");
  if (!finite_f32(cfg->beta1) || !finite_f32(cfg->beta2) || !finite_f32(cfg->epsilon) ||
      !(cfg->max_grad_norm > 0.0f) || !finite_f32(cfg->max_grad_norm) ||
      !finite_f32(cfg->min_clip_accept))
    return h->err(SLM_ERR_INVALID_ARGUMENT, "non-finite or non-positive hyperparameter");
  if (cfg->nonfinite_policy != SLM_NONFINITE_SKIP && cfg->nonfinite_policy != SLM_NONFINITE_ERROR)
    return h->err(SLM_ERR_INVALID_ARGUMENT, "unknown non-finite policy");
  if (cfg->loss_scale_mode == SLM_SCALE_STATIC) {
    if (!(cfg->static_loss_scale > 0.0f) || !finite_f32(cfg->static_loss_scale))
      return h->err(SLM_ERR_INVALID_ARGUMENT, "the static loss scale must be positive and finite");
  } else if (cfg->loss_scale_mode == SLM_SCALE_DYNAMIC) {
    if (cfg->growth_interval == 0)
      return h->err(SLM_ERR_INVALID_ARGUMENT, "the growth interval must be at least 1");
  } else {
    return h->err(SLM_ERR_INVALID_ARGUMENT, "unknown loss-scale mode");
  }
  return SLM_OK;
}

FinalizeParams finalize_params(const slm_opt_handle* h, const slm_step_config* cfg) {
  FinalizeParams fp;
  fp.max_grad_norm = cfg->max_grad_norm;
  fp.min_clip_accept = cfg->min_clip_accept;
  fp.apply_clip = cfg->apply_clip ? 1 : 0;
  fp.nonfinite_policy = cfg->nonfinite_policy;
  fp.dynamic = cfg->loss_scale_mode == SLM_SCALE_DYNAMIC ? 1 : 0;
  fp.growth_interval = cfg->growth_interval;
  fp.static_scale = cfg->static_loss_scale;
  fp.total_chunks = h->sharded() ? uint32_t(h->world) * h->chunks_per_rank : h->n_chunks;
  return fp;
}

void fill_result(const DeviceStepState& s, slm_step_result* out) {
  out->sum_squares = s.sum_squares;
  out->grad_norm = s.grad_norm;
  out->clip_scale = s.clip_scale;
  out->loss_scale_used = s.loss_scale_used;
  out->next_loss_scale = s.next_loss_scale;
  out->skipped = s.skipped;
  out->nonfinite = s.nonfinite;
  out->result_nonfinite = s.result_nonfinite;
  out->rejected = s.rejected;
  out->good_steps = s.good_steps;
  out->status = s.status != 0 ? s.status
                              : (s.result_nonfinite ? SLM_ERR_MODEL_OPTIMIZER_RESULT_NONFINITE
                                                    : SLM_OK);
  // A bounded in-kernel wait gave up: a peer never arrived (2) or a copy
  // pipeline stalled (1).
  if (s.kernel_error) out->status = (s.kernel_error & 2u) ? SLM_ERR_TIMEOUT : SLM_ERR_INTERNAL;
}

int read_state(slm_opt_handle* h, cudaStream_t s, DeviceStepState* out) {
  int st = h->cuda(cudaMemcpyAsync(h->h_state, h->d_state, sizeof(DeviceStepState),
                                   cudaMemcpyDeviceToHost, s),
                   "result copy");
  if (st) return st;
  if (h->sharded()) {
    if ((st = zero1_wait(h, s))) return st;
  } else if ((st = h->cuda(cudaStreamSynchronize(s), "step sync"))) {
    return st;
  }
  *out = *h->h_state;
  return SLM_OK;
}

int allocate_state(slm_opt_handle* h, uint64_t w16_elems) {
  const uint64_t L = h->shard_len;
  const uint64_t chunks = (h->P + kChunkElems - 1) / kChunkElems;
  if (chunks > 0xffffffffull)
    return h->err(SLM_ERR_SIZE_LIMIT, "parameter count exceeds the chunk index range");
  h->n_chunks = uint32_t(chunks);
  const uint64_t tiles = (L + kTileElems - 1) / kTileElems;
  std::vector<uint32_t> tile_first(tiles ? tiles : 1, 0);
  {
    uint32_t k = 0;
    for (uint64_t t = 0; t < tiles; ++t) {
      const uint64_t e = h->shard_begin + t * kTileElems;
      while (e >= h->offsets[k + 1]) ++k;
      tile_first[t] = k;
    }
  }
  const uint64_t Ls = L ? L : 1;  // keep every pointer valid for an empty shard
  int st;
#define SLM_TRY(expr, what) \
  if ((st = h->cuda((expr), what)) != SLM_OK) return st
  SLM_TRY(cudaMalloc(&h->master, Ls * sizeof(float)), "cudaMalloc master");
  SLM_TRY(cudaMalloc(&h->m1, Ls * sizeof(float)), "cudaMalloc m1");
  SLM_TRY(cudaMalloc(&h->m2, Ls * sizeof(float)), "cudaMalloc m2");
  SLM_TRY(cudaMalloc(&h->w16, w16_elems * sizeof(uint16_t)), "cudaMalloc bf16");
  SLM_TRY(cudaMalloc(&h->d_offsets, h->offsets.size() * sizeof(uint64_t)), "cudaMalloc offsets");
  SLM_TRY(cudaMalloc(&h->d_decay, h->decay.size()), "cudaMalloc decay");
  SLM_TRY(cudaMalloc(&h->d_tile_first, tile_first.size() * sizeof(uint32_t)), "cudaMalloc tiles");
  SLM_TRY(cudaMalloc(&h->d_partials, chunks * sizeof(double)), "cudaMalloc partials");
  SLM_TRY(cudaMalloc(&h->d_state, sizeof(DeviceStepState)), "cudaMalloc state");
  SLM_TRY(cudaMalloc(&h->d_scaler, sizeof(DeviceScaler)), "cudaMalloc scaler");
  SLM_TRY(cudaMalloc(&h->d_flag, sizeof(uint32_t)), "cudaMalloc flag");
  SLM_TRY(cudaMalloc(&h->d_seq_carry, sizeof(SeqCarry)), "cudaMalloc clip carry");
  h->seq_ws_bytes = seq_clip_workspace_bytes(h->P);
  SLM_TRY(cudaMalloc(&h->d_seq_ws, h->seq_ws_bytes), "cudaMalloc clip workspace");
  SLM_TRY(cudaMallocHost(&h->h_state, sizeof(DeviceStepState)), "cudaMallocHost state");
  SLM_TRY(cudaMemset(h->master, 0, Ls * sizeof(float)), "memset master");
  SLM_TRY(cudaMemset(h->m1, 0, Ls * sizeof(float)), "memset m1");
  SLM_TRY(cudaMemset(h->m2, 0, Ls * sizeof(float)), "memset m2");
  SLM_TRY(cudaMemset(h->w16, 0, w16_elems * sizeof(uint16_t)), "memset bf16");
  SLM_TRY(cudaMemset(h->d_state, 0, sizeof(DeviceStepState)), "memset state");
  SLM_TRY(cudaMemset(h->d_partials, 0, chunks * sizeof(double)), "memset partials");
  SLM_TRY(cudaMemcpy(h->d_offsets, h->offsets.data(), h->offsets.size() * sizeof(uint64_t),
                     cudaMemcpyHostToDevice),
          "upload offsets");
  SLM_TRY(cudaMemcpy(h->d_decay, h->decay.data(), h->decay.size(), cudaMemcpyHostToDevice),
          "upload decay");
  SLM_TRY(cudaMemcpy(h->d_tile_first, tile_first.data(), tile_first.size() * sizeof(uint32_t),
                     cudaMemcpyHostToDevice),
          "upload tile table");
  const DeviceScaler sc{65536.0f, 0u};
  SLM_TRY(cudaMemcpy(h->d_scaler, &sc, sizeof(sc), cudaMemcpyHostToDevice), "upload scaler");
#undef SLM_TRY
  h->grid_norm = norm_partials_grid(h->device);
  h->grid_norm_bulk = norm_bulk_grid(h->device);
  h->grid_update[0] = adamw_update_grid(h->device, 0);
  h->grid_update[1] = adamw_update_grid(h->device, 1);
  return SLM_OK;
}

int build_table(slm_opt_handle* h, const slm_tensor_spec* table, uint32_t n_tensors) {
  if (!table || n_tensors == 0)
    return fail(SLM_ERR_P12_OPTIMIZER_STATE_INVALID, "the AdamW state contains no parameters");
  std::set<std::string> seen;
  h->offsets.assign(1, 0);
  for (uint32_t k = 0; k < n_tensors; ++k) {
    const char* name = table[k].name;
    if (!name || !*name || table[k].elements == 0)
      return fail(SLM_ERR_P12_OPTIMIZER_STATE_INVALID,
                  "an AdamW parameter has an empty name or no elements");
    if (!seen.insert(name).second)
      return fail(SLM_ERR_P12_OPTIMIZER_PARAMETER_DUPLICATE,
                  std::string("duplicate stable parameter name: ") + name);
    h->names.emplace_back(name);
    h->decay.push_back(table[k].weight_decay ? 1 : 0);
    h->offsets.push_back(h->offsets.back() + table[k].elements);
  }
  h->P = h->offsets.back();
  return SLM_OK;
}

}  // namespace slmopt

namespace {

int role_info(slm_opt_handle* h, int role, void** ptr, uint64_t* full_bytes,
              uint64_t* shard_bytes) {
  switch (role) {
    case SLM_ROLE_PARAMETERS_BF16:
      *ptr = h->w16;
      *full_bytes = *shard_bytes = h->P * 2;
      return SLM_OK;
    case SLM_ROLE_MASTER_F32:
      *ptr = h->master;
      break;
    case SLM_ROLE_MOMENT1_F32:
      *ptr = h->m1;
      break;
    case SLM_ROLE_MOMENT2_F32:
      *ptr = h->m2;
      break;
    default:
      return h->err(SLM_ERR_INVALID_ARGUMENT, "unknown artifact role");
  }
  *full_bytes = h->P * 4;
  *shard_bytes = h->shard_len * 4;
  return SLM_OK;
}

// ---- host gradients in pageable memory ------------------------------------------
// A cudaMemcpyAsync from pageable memory goes through the driver's own bounce
// buffer, one buffer at a time, at ~11 GB/s (49 ms for the 541 MB f32
// gradient the reference hands apply_update).  stage_pageable instead lets
// several host threads copy consecutive 32 MB slices of the source into a
// ring of pinned slots while the previous slice's DMA runs on the handle's
// copy stream, so the host copy and the PCIe transfer overlap.  After each
// slice's DMA is enqueued, on_slice(offset, bytes, landed) runs on the host
// with `landed` recorded behind that DMA, so device work on the slice can
// start while later slices are still on their way.
bool is_pageable(const void* p) {
  cudaPointerAttributes a;
  if (cudaPointerGetAttributes(&a, p) != cudaSuccess) {
    cudaGetLastError();
    return true;
  }
  return a.type == cudaMemoryTypeUnregistered;
}

int ensure_staging(slm_opt_handle* h, size_t bytes) {
  if (h->staging_bytes >= bytes) return SLM_OK;
  cudaFree(h->d_staging);
  h->d_staging = nullptr;
  h->staging_bytes = 0;
  const int st = h->cuda(cudaMalloc(&h->d_staging, bytes), "cudaMalloc gradient staging");
  if (st == SLM_OK) h->staging_bytes = bytes;
  return st;
}

template <typename OnSlice>
int stage_pageable(slm_opt_handle* h, void* dst, const void* src, size_t bytes,
                   cudaStream_t compute, OnSlice on_slice) {
  using Ring = slm_opt_handle::PinnedRing;
  int st;
  if (!h->copy_stream &&
      (st = h->cuda(cudaStreamCreateWithFlags(&h->copy_stream, cudaStreamNonBlocking),
                    "copy stream")))
    return st;
  for (int k = 0; k < Ring::kSlots; ++k) {
    if (!h->ring.slot[k] &&
        (st = h->cuda(cudaMallocHost(&h->ring.slot[k], Ring::kSlotBytes), "pinned staging ring")))
      return st;
    if (!h->ring.drained[k] &&
        (st = h->cuda(cudaEventCreateWithFlags(&h->ring.drained[k], cudaEventDisableTiming),
                      "staging event")))
      return st;
  }
  // The device buffer may still be read by work enqueued earlier on the
  // compute stream: the copies wait for it.
  cudaEvent_t before = nullptr;
  if ((st = h->cuda(cudaEventCreateWithFlags(&before, cudaEventDisableTiming), "staging event")))
    return st;
  st = h->cuda(cudaEventRecord(before, compute), "staging event");
  if (!st) st = h->cuda(cudaStreamWaitEvent(h->copy_stream, before, 0), "staging wait");
  cudaEventDestroy(before);
  if (st) return st;

  const size_t n_slices = (bytes + Ring::kSlotBytes - 1) / Ring::kSlotBytes;
  // Host threads filling the ring: half the host's hardware threads, at most
  // 8, unless SLM_STAGING_THREADS (1..64) says otherwise.
  const unsigned hw = std::thread::hardware_concurrency();
  size_t T = std::min<size_t>(8, std::max<size_t>(1, hw / 2));
  if (const char* env = std::getenv("SLM_STAGING_THREADS")) {
    const long v = std::strtol(env, nullptr, 10);
    if (v >= 1 && v <= 64) T = size_t(v);
  }
  std::unique_ptr<std::atomic<size_t>[]> parts(new std::atomic<size_t>[n_slices]);
  for (size_t c = 0; c < n_slices; ++c) parts[c].store(0);
  std::atomic<size_t> go{0};  // slices whose slot is free to be filled
  std::atomic<bool> stop{false};
  auto fill = [&](size_t w) {
    for (size_t c = 0; c < n_slices; ++c) {
      while (go.load(std::memory_order_acquire) <= c) {
        if (stop.load(std::memory_order_acquire)) return;
        std::this_thread::yield();
      }
      const size_t off = c * Ring::kSlotBytes;
      const size_t len = std::min(Ring::kSlotBytes, bytes - off);
      const size_t part = (len + T - 1) / T;
      const size_t lo = std::min(len, w * part), hi = std::min(len, lo + part);
      if (lo < hi)
        stream_copy(static_cast<uint8_t*>(h->ring.slot[c % Ring::kSlots]) + lo,
                    static_cast<const uint8_t*>(src) + off + lo, hi - lo);
      parts[c].fetch_add(1, std::memory_order_acq_rel);
    }
  };
  std::vector<std::thread> pool;
  for (size_t w = 0; w < T; ++w) pool.emplace_back(fill, w);
  for (size_t c = 0; c < n_slices && st == SLM_OK; ++c) {
    const int k = int(c % Ring::kSlots);
    if (h->ring.used[k] &&
        (st = h->cuda(cudaEventSynchronize(h->ring.drained[k]), "staging slot wait")))
      break;
    go.store(c + 1, std::memory_order_release);
    while (parts[c].load(std::memory_order_acquire) < T) std::this_thread::yield();
    const size_t off = c * Ring::kSlotBytes;
    const size_t len = std::min(Ring::kSlotBytes, bytes - off);
    st = h->cuda(cudaMemcpyAsync(static_cast<uint8_t*>(dst) + off, h->ring.slot[k], len,
                                 cudaMemcpyHostToDevice, h->copy_stream),
                 "gradient upload");
    if (!st) st = h->cuda(cudaEventRecord(h->ring.drained[k], h->copy_stream), "staging event");
    if (st) break;
    h->ring.used[k] = true;
    st = on_slice(off, len, h->ring.drained[k]);
  }
  stop.store(true, std::memory_order_release);
  for (auto& th : pool) th.join();
  return st;
}

// Stage the gradient: device pointers are used in place (16-byte alignment
// required for the vector loads), host pointers are copied into a staging
// buffer ahead of the step's work on its stream (pinned memory with one
// asynchronous copy, pageable memory through stage_pageable).
int stage_grads(slm_opt_handle* h, const void* grads, int dtype, int memory, cudaStream_t s,
                const void** dev_grads) {
  const size_t esize = dtype == SLM_DTYPE_F32 ? 4 : 2;
  const size_t bytes = h->P * esize;
  if (memory == SLM_MEMORY_DEVICE) {
    if (reinterpret_cast<uintptr_t>(grads) % 16 != 0)
      return h->err(SLM_ERR_INVALID_ARGUMENT, "device gradients must be 16-byte aligned");
    *dev_grads = grads;
    return SLM_OK;
  }
  if (memory != SLM_MEMORY_HOST) return h->err(SLM_ERR_INVALID_ARGUMENT, "unknown memory kind");
  int st = ensure_staging(h, bytes);
  if (st) return st;
  if (is_pageable(grads) && bytes > slm_opt_handle::PinnedRing::kSlotBytes) {
    st = stage_pageable(h, h->d_staging, grads, bytes, s,
                        [&](size_t, size_t, cudaEvent_t landed) {
                          return h->cuda(cudaStreamWaitEvent(s, landed, 0), "upload wait");
                        });
  } else {
    st = h->cuda(cudaMemcpyAsync(h->d_staging, grads, bytes, cudaMemcpyHostToDevice, s),
                 "gradient upload");
  }
  if (st) return st;
  *dev_grads = h->d_staging;
  return SLM_OK;
}

int enqueue_norm(slm_opt_handle* h, const void* dev_grads, int dtype, const slm_step_config* cfg,
                 cudaStream_t s) {
  const FinalizeParams fp = finalize_params(h, cfg);
  return h->cuda(launch_norm_partials(dtype, dev_grads, h->P, 0, h->n_chunks, h->d_scaler,
                                      h->d_partials, h->d_state, fp, h->grid_norm_bulk, s),
                 "norm kernel");
}

int enqueue_update(slm_opt_handle* h, const void* dev_grads, int dtype,
                   const slm_step_config* cfg, cudaStream_t s) {
  const AdamwParams p = adamw_params(cfg);
  return h->cuda(launch_adamw_update(dtype, dev_grads, h->P, 0, h->master, h->m1, h->m2, h->w16,
                                     h->d_offsets, h->d_decay, h->d_tile_first, p, h->d_state,
                                     h->grid_update[dtype == SLM_DTYPE_F32 ? 0 : 1], s),
                 "update kernel");
}

// Folds the last complete step's phase intervals into the sums (waits for it).
int phase_harvest(slm_opt_handle* h) {
  PhaseTimer& t = h->timer;
  const int n = t.finished;
  t.finished = 0;
  if (n < 2) return SLM_OK;
  int st = h->cuda(cudaEventSynchronize(t.ev[n - 1]), "phase timing");
  if (st) return st;
  if (t.finished_kind != t.kind) {  // another entry point's phases: start the sums afresh
    for (double& a : t.acc) a = 0.0;
    t.steps = 0;
    t.kind = t.finished_kind;
  }
  for (int i = 0; i + 1 < n; ++i) {
    float ms = 0.0f;
    if ((st = h->cuda(cudaEventElapsedTime(&ms, t.ev[i], t.ev[i + 1]), "phase timing")))
      return st;
    t.acc[i] += ms;
  }
  t.phases = uint32_t(n - 1);
  ++t.steps;
  return SLM_OK;
}

int finish_result(slm_opt_handle* h, const DeviceStepState& ds, slm_step_result* out) {
  fill_result(ds, out);
  if (ds.kernel_error) h->broken = true;  // the ranks may be out of step: re-create the handle
  if (out->status != SLM_OK)
    return h->err(out->status, std::string("optimizer step failed: ") +
                                   slm_status_code_string(out->status));
  return SLM_OK;
}

// Full host copy of one role (gathered across ranks for a ZeRO-1 handle).
int download_role(slm_opt_handle* h, int role, void* dst, uint64_t bytes) {
  void* ptr = nullptr;
  uint64_t full = 0, shard = 0;
  int st = role_info(h, role, &ptr, &full, &shard);
  if (st) return st;
  if (bytes != full)
    return h->err(SLM_ERR_E1_STATE_ARTIFACT_INVALID,
                  "a checkpoint artifact does not cover the exact parameter layout");
  if (h->sharded() && role != SLM_ROLE_PARAMETERS_BF16)
    return zero1_gather(h, ptr, 4, dst, nullptr);
  return h->cuda(cudaMemcpy(dst, ptr, bytes, cudaMemcpyDeviceToHost), "snapshot copy");
}

}  // namespace

int slmopt::phase_begin(slm_opt_handle* h, cudaStream_t s) {
  PhaseTimer& t = h->timer;
  if (!t.enabled) return SLM_OK;
  t.marks = 0;  // drops the events of a step that failed part-way
  if (int st = phase_harvest(h)) return st;
  return phase_mark(h, s);
}

int slmopt::phase_mark(slm_opt_handle* h, cudaStream_t s) {
  PhaseTimer& t = h->timer;
  if (!t.enabled || t.marks >= PhaseTimer::kMaxMarks) return SLM_OK;
  return h->cuda(cudaEventRecord(t.ev[t.marks++], s), "phase timing");
}

void slmopt::phase_end(slm_opt_handle* h, int kind) {
  PhaseTimer& t = h->timer;
  if (!t.enabled) return;
  t.finished = t.marks;
  t.finished_kind = kind;
  t.marks = 0;
}

extern "C" {

int slm_abi_version(void) { return SLMOPT_ABI_VERSION; }

const char* slm_last_error_message(void) { return g_last_error.c_str(); }

const char* slm_status_code_string(int status) {
  switch (status) {
    case SLM_OK: return "OK";
    case SLM_ERR_MODEL_GRADIENT_NONFINITE: return "MODEL_GRADIENT_NONFINITE";
    case SLM_ERR_MODEL_GRADIENT_NORM_NONFINITE: return "MODEL_GRADIENT_NORM_NONFINITE";
    case SLM_ERR_MODEL_OPTIMIZER_INPUT_INVALID: return "MODEL_OPTIMIZER_INPUT_INVALID";
    case SLM_ERR_MODEL_OPTIMIZER_RESULT_NONFINITE: return "MODEL_OPTIMIZER_RESULT_NONFINITE";
    case SLM_ERR_P12_OPTIMIZER_GRADIENT_INVALID: return "P12_OPTIMIZER_GRADIENT_INVALID";
    case SLM_ERR_P12_SCHEDULER_STATE_MISMATCH: return "P12_SCHEDULER_STATE_MISMATCH";
    case SLM_ERR_P12_OPTIMIZER_STATE_INVALID: return "P12_OPTIMIZER_STATE_INVALID";
    case SLM_ERR_P12_UPDATE_INDEX_INVALID: return "P12_UPDATE_INDEX_INVALID";
    case SLM_ERR_P12_SCHEDULE_INDEX_INVALID: return "P12_SCHEDULE_INDEX_INVALID";
    case SLM_ERR_E1_PARAMETER_LAYOUT_MISMATCH: return "E1_PARAMETER_LAYOUT_MISMATCH";
    case SLM_ERR_E1_STATE_ARTIFACT_INVALID: return "E1_STATE_ARTIFACT_INVALID";
    case SLM_ERR_P12_OPTIMIZER_PARAMETER_DUPLICATE: return "P12_OPTIMIZER_PARAMETER_DUPLICATE";
    case SLM_ERR_INVALID_ARGUMENT: return "SLM_INVALID_ARGUMENT";
    case SLM_ERR_SIZE_LIMIT: return "SLM_SIZE_LIMIT";
    case SLM_ERR_CUDA: return "SLM_CUDA_ERROR";
    case SLM_ERR_OUT_OF_MEMORY: return "SLM_OUT_OF_MEMORY";
    case SLM_ERR_NCCL: return "SLM_NCCL_ERROR";
    case SLM_ERR_TIMEOUT: return "SLM_TIMEOUT";
    case SLM_ERR_NO_DEVICE: return "SLM_NO_DEVICE";
    case SLM_ERR_INTERNAL: return "SLM_INTERNAL_ERROR";
    default: return "SLM_UNKNOWN_STATUS";
  }
}

int slm_status_category(int status) {
  if (status == SLM_OK) return 0;
  if (status >= 10 && status < 20) return 5;  // Gate
  if (status >= 20 && status < 30) return 3;  // Integrity
  if (status >= 30 && status < 40) return 2;  // Usage
  if (status >= 40 && status < 50) return 4;  // Environment
  return 1;                                   // Internal
}

void slm_step_config_default(slm_step_config* cfg) {
  if (!cfg) return;
  // OPT-001, src/model/oracle.rs:469-484; decay 0.1 / 0.0 by group, trainer.rs:276.
  cfg->learning_rate = 3.0e-4f;
  cfg->one_based_update = 1;
  cfg->beta1 = 0.9f;
  cfg->beta2 = 0.95f;
  cfg->epsilon = 1.0e-8f;
  cfg->decay_weight = 0.1f;
  cfg->no_decay_weight = 0.0f;
  cfg->max_grad_norm = 1.0f;
  cfg->apply_clip = 1;
  cfg->min_clip_accept = 0.0f;
  cfg->nonfinite_policy = SLM_NONFINITE_SKIP;
  cfg->loss_scale_mode = SLM_SCALE_STATIC;
  cfg->static_loss_scale = 1.0f;
  cfg->growth_interval = 2000;
}

int slm_schedule_learning_rate(uint64_t t, float peak, float minimum, uint64_t warmup,
                               uint64_t total, float* out) {
  if (!out) return fail(SLM_ERR_INVALID_ARGUMENT, "out is NULL");
  if (t < 1 || t > total || warmup >= total)
    return fail(SLM_ERR_P12_SCHEDULE_INDEX_INVALID,
                "the scheduler index is outside the optimizer-update range");
  if (t <= warmup) {
    *out = peak * float(t) / float(warmup);
    return SLM_OK;
  }
  const double progress = double(t - warmup) / double(total - warmup);
  const double lr = double(minimum) + 0.5 * double(peak - minimum) *
                                          (1.0 + std::cos(3.14159265358979323846 * progress));
  *out = float(lr);
  return SLM_OK;
}

int slm_canonical_learning_rate(uint64_t t, float* out) {
  // src/train/trainer.rs:16-22 constants: 30,518 updates, 1,000 warmup,
  // peak 0.0025, minimum 0.00025.
  return slm_schedule_learning_rate(t, 0.0025f, 0.00025f, 1000u, 30518u, out);
}

int slm_opt_create(const slm_tensor_spec* table, uint32_t n_tensors, int device,
                   slm_opt_handle** out) {
  if (!out) return fail(SLM_ERR_INVALID_ARGUMENT, "out is NULL");
  *out = nullptr;
  slm_opt_handle* h = new (std::nothrow) slm_opt_handle();
  if (!h) return fail(SLM_ERR_OUT_OF_MEMORY, "host allocation failed");
  int st = build_table(h, table, n_tensors);
  if (st) {
    delete h;
    return st;
  }
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) {
    delete h;
    return fail(SLM_ERR_NO_DEVICE, "no CUDA device is visible");
  }
  if (device < 0 || device >= count) {
    delete h;
    return fail(SLM_ERR_INVALID_ARGUMENT, "device ordinal out of range");
  }
  h->device = device;
  h->shard_begin = 0;
  h->shard_len = h->P;
  DeviceGuard guard(device);
  if (!guard.ok) {
    delete h;
    return fail(SLM_ERR_CUDA, "cudaSetDevice failed");
  }
  if ((st = allocate_state(h, h->P))) {
    slm_opt_destroy(h);
    return st;
  }
  *out = h;
  return SLM_OK;
}

int slm_opt_destroy(slm_opt_handle* h) {
  if (!h) return SLM_OK;
  DeviceGuard guard(h->device);
  // Work this handle enqueued (on any stream) finishes before its buffers and
  // peer mappings go away; every kernel's waits are bounded.
  cudaDeviceSynchronize();
  zero1_release(h);
  if (h->timer.created)
    for (cudaEvent_t e : h->timer.ev) cudaEventDestroy(e);
  cudaFree(h->master);
  cudaFree(h->m1);
  cudaFree(h->m2);
  cudaFree(h->w16);
  cudaFree(h->d_offsets);
  cudaFree(h->d_decay);
  cudaFree(h->d_tile_first);
  cudaFree(h->d_partials);
  cudaFree(h->d_state);
  cudaFree(h->d_scaler);
  cudaFree(h->d_flag);
  cudaFree(h->d_seq_carry);
  cudaFree(h->d_seq_ws);
  cudaFree(h->d_staging);
  for (int k = 0; k < slm_opt_handle::PinnedRing::kSlots; ++k) {
    if (h->ring.drained[k]) {
      cudaEventSynchronize(h->ring.drained[k]);
      cudaEventDestroy(h->ring.drained[k]);
    }
    if (h->ring.slot[k]) cudaFreeHost(h->ring.slot[k]);
  }
  if (h->copy_stream) {
    cudaStreamSynchronize(h->copy_stream);
    cudaStreamDestroy(h->copy_stream);
  }
  for (auto& u : h->up) {
    if (u.consumed_recorded) cudaEventSynchronize(u.consumed);
    cudaFree(u.dev);
    if (u.uploaded) cudaEventDestroy(u.uploaded);
    if (u.consumed) cudaEventDestroy(u.consumed);
  }
  if (h->h_state) cudaFreeHost(h->h_state);
  delete h;
  return SLM_OK;
}

uint64_t slm_opt_parameter_count(const slm_opt_handle* h) { return h ? h->P : 0; }

const char* slm_opt_last_error(const slm_opt_handle* h) {
  return h ? h->last_error.c_str() : g_last_error.c_str();
}

int slm_opt_device_buffer(slm_opt_handle* h, int role, void** out_device_ptr) {
  if (!h || !out_device_ptr) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL argument");
  uint64_t full = 0, shard = 0;
  return role_info(h, role, out_device_ptr, &full, &shard);
}

int slm_opt_init_master(slm_opt_handle* h, const float* master_host, void* stream) {
  if (!h || !master_host) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL argument");
  DeviceGuard guard(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  int st = h->cuda(cudaMemcpyAsync(h->master, master_host + h->shard_begin,
                                   h->shard_len * sizeof(float), cudaMemcpyHostToDevice, s),
                   "upload master");
  if (st) return st;
  if (h->shard_len) {
    st = h->cuda(launch_init_from_master(h->master, h->m1, h->m2, h->w16 + h->shard_begin,
                                         h->shard_len, s),
                 "init kernel");
    if (st) return st;
  }
  if ((st = h->cuda(cudaStreamSynchronize(s), "init sync"))) return st;
  if (h->sharded())  // every rank needs every shard's bf16 weights
    return zero1_gather(h, h->w16 + h->shard_begin, 2, nullptr, s);
  return SLM_OK;
}

int slm_opt_snapshot(slm_opt_handle* h, int role, void* host_dst, uint64_t bytes) {
  if (!h || !host_dst) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL argument");
  void* ptr = nullptr;
  uint64_t full = 0, shard = 0;
  int st = role_info(h, role, &ptr, &full, &shard);
  if (st) return st;
  DeviceGuard guard(h->device);
  if (h->sharded() && bytes == shard && bytes != full)
    return h->cuda(cudaMemcpy(host_dst, ptr, bytes, cudaMemcpyDeviceToHost), "shard copy");
  return download_role(h, role, host_dst, bytes);
}

int slm_opt_restore(slm_opt_handle* h, int role, const void* host_src, uint64_t bytes) {
  if (!h || !host_src) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL argument");
  void* ptr = nullptr;
  uint64_t full = 0, shard = 0;
  int st = role_info(h, role, &ptr, &full, &shard);
  if (st) return st;
  if (bytes != full)
    return h->err(SLM_ERR_E1_STATE_ARTIFACT_INVALID,
                  "a checkpoint artifact does not cover the exact parameter layout");
  DeviceGuard guard(h->device);
  if (role == SLM_ROLE_PARAMETERS_BF16)
    return h->cuda(cudaMemcpy(ptr, host_src, bytes, cudaMemcpyHostToDevice), "restore copy");
  const uint8_t* src = static_cast<const uint8_t*>(host_src) + h->shard_begin * 4;
  return h->cuda(cudaMemcpy(ptr, src, shard, cudaMemcpyHostToDevice), "restore copy");
}

int slm_opt_validate_state(slm_opt_handle* h) {
  if (!h) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL handle");
  DeviceGuard guard(h->device);
  int st = h->cuda(cudaMemset(h->d_flag, 0, sizeof(uint32_t)), "validate memset");
  if (st) return st;
  if (h->shard_len) {
    st = h->cuda(launch_validate_state(h->master, h->m1, h->m2, h->w16 + h->shard_begin,
                                       h->shard_len, h->d_flag, nullptr),
                 "validate kernel");
    if (st) return st;
  }
  uint32_t bad = 0;
  st = h->cuda(cudaMemcpy(&bad, h->d_flag, sizeof(bad), cudaMemcpyDeviceToHost), "validate read");
  if (st) return st;
  if (bad)
    return h->err(SLM_ERR_P12_OPTIMIZER_STATE_INVALID,
                  "an AdamW parameter has mismatched or nonfinite state");
  return SLM_OK;
}

int slm_opt_set_loss_scale(slm_opt_handle* h, float scale, uint32_t good_steps) {
  if (!h) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL handle");
  if (!(scale > 0.0f) || !finite_f32(scale))
    return h->err(SLM_ERR_INVALID_ARGUMENT, "the loss scale must be positive and finite");
  DeviceGuard guard(h->device);
  const DeviceScaler sc{scale, good_steps};
  return h->cuda(cudaMemcpy(h->d_scaler, &sc, sizeof(sc), cudaMemcpyHostToDevice), "set scale");
}

int slm_opt_get_loss_scale(slm_opt_handle* h, float* scale, uint32_t* good_steps) {
  if (!h || !scale || !good_steps) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL argument");
  DeviceGuard guard(h->device);
  DeviceScaler sc{};
  int st = h->cuda(cudaMemcpy(&sc, h->d_scaler, sizeof(sc), cudaMemcpyDeviceToHost), "get scale");
  if (st) return st;
  *scale = sc.scale;
  *good_steps = sc.good_steps;
  return SLM_OK;
}

int slm_opt_norm_pass(slm_opt_handle* h, const void* grads, int dtype, int memory,
                      const slm_step_config* cfg, void* stream) {
  if (!h || !grads) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL argument");
  if (dtype != SLM_DTYPE_F32 && dtype != SLM_DTYPE_BF16)
    return h->err(SLM_ERR_INVALID_ARGUMENT, "unknown gradient dtype");
  int st = check_config(h, cfg);
  if (st) return st;
  if (h->sharded())
    return h->err(SLM_ERR_INVALID_ARGUMENT, "a ZeRO-1 handle runs whole steps (slm_opt_step)");
  DeviceGuard guard(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const void* dev = nullptr;
  h->pass_grads = nullptr;
  if ((st = stage_grads(h, grads, dtype, memory, s, &dev))) return st;
  if ((st = enqueue_norm(h, dev, dtype, cfg, s))) return st;
  h->pass_grads = dev;
  h->pass_dtype = dtype;
  h->pending = true;
  h->pending_stream = s;
  return SLM_OK;
}

int slm_grad_accumulate(float* acc_device, const void* micro_device, int dtype, uint64_t n,
                        int overwrite, void* stream) {
  if (!acc_device || !micro_device) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL argument");
  if (dtype != SLM_DTYPE_F32 && dtype != SLM_DTYPE_BF16)
    return fail(SLM_ERR_INVALID_ARGUMENT, "unknown gradient dtype");
  if (reinterpret_cast<uintptr_t>(acc_device) % 16 != 0 ||
      reinterpret_cast<uintptr_t>(micro_device) % 16 != 0)
    return fail(SLM_ERR_INVALID_ARGUMENT, "accumulator and gradients must be 16-byte aligned");
  const cudaError_t e = launch_accumulate(dtype, acc_device, micro_device, n, overwrite,
                                          static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess)
    return fail(SLM_ERR_CUDA, std::string("accumulate kernel: ") + cudaGetErrorString(e));
  return SLM_OK;
}

uint64_t slm_gradient_clip_workspace_bytes(uint64_t n) { return seq_clip_workspace_bytes(n); }

int slm_gradient_clip_scale(const float* grads_device, uint64_t n, slm_clip_result* out_device,
                            void* stream) {
  return slm_gradient_clip_scale_ws(grads_device, n, nullptr, 0, out_device, stream);
}

int slm_gradient_clip_scale_ws(const float* grads_device, uint64_t n, void* workspace_device,
                               uint64_t workspace_bytes, slm_clip_result* out_device,
                               void* stream) {
  if ((!grads_device && n) || !out_device) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL argument");
  if (workspace_device) {
    if (reinterpret_cast<uintptr_t>(workspace_device) % 16 != 0)
      return fail(SLM_ERR_INVALID_ARGUMENT, "the workspace must be 16-byte aligned");
    if (workspace_bytes < seq_clip_workspace_bytes(n))
      return fail(SLM_ERR_INVALID_ARGUMENT,
                  "the workspace is smaller than slm_gradient_clip_workspace_bytes(n)");
  }
  if (reinterpret_cast<uintptr_t>(grads_device) % 16 != 0)
    return fail(SLM_ERR_INVALID_ARGUMENT, "gradients must be 16-byte aligned");
  if (reinterpret_cast<uintptr_t>(out_device) % alignof(slm_clip_result) != 0)
    return fail(SLM_ERR_INVALID_ARGUMENT, "out_device must be 4-byte aligned");
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t e = cudaMemsetAsync(&out_device->kernel_error, 0, sizeof(uint32_t), s);
  if (e == cudaSuccess) {
    const SeqClipOut out{nullptr, &out_device->sum_squares, &out_device->clip_scale,
                         &out_device->status};
    e = launch_sequential_clip(grads_device, n, out, &out_device->kernel_error, s, nullptr,
                               false, true, workspace_device, size_t(workspace_bytes));
  }
  if (e != cudaSuccess)
    return fail(SLM_ERR_CUDA, std::string("clip scale kernel: ") + cudaGetErrorString(e));
  return SLM_OK;
}

int slm_opt_norm_pass_accumulate(slm_opt_handle* h, float* acc_device, const void* micro,
                                 int dtype, int memory, int overwrite,
                                 const slm_step_config* cfg, void* stream) {
  if (!h || !acc_device || !micro) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL argument");
  if (dtype != SLM_DTYPE_F32 && dtype != SLM_DTYPE_BF16)
    return h->err(SLM_ERR_INVALID_ARGUMENT, "unknown gradient dtype");
  if (h->sharded())
    return h->err(SLM_ERR_INVALID_ARGUMENT, "a ZeRO-1 handle runs whole steps (slm_opt_step)");
  if (reinterpret_cast<uintptr_t>(acc_device) % 16 != 0)
    return h->err(SLM_ERR_INVALID_ARGUMENT, "the accumulator must be 16-byte aligned");
  int st = check_config(h, cfg);
  if (st) return st;
  DeviceGuard guard(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const void* dev = nullptr;
  h->pass_grads = nullptr;
  if ((st = stage_grads(h, micro, dtype, memory, s, &dev))) return st;
  const FinalizeParams fp = finalize_params(h, cfg);
  if ((st = h->cuda(launch_accumulate_norm(dtype, acc_device, dev, h->P, overwrite, h->n_chunks,
                                           h->d_scaler, h->d_partials, h->d_state, fp, s),
                    "accumulate + norm kernel")))
    return st;
  h->pass_grads = acc_device;
  h->pass_dtype = SLM_DTYPE_F32;
  h->pending = true;
  h->pending_stream = s;
  return SLM_OK;
}

int slm_opt_update_pass(slm_opt_handle* h, const slm_step_config* cfg, void* stream) {
  if (!h) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL handle");
  if (!h->pass_grads)
    return h->err(SLM_ERR_INVALID_ARGUMENT, "slm_opt_update_pass needs a preceding norm pass");
  int st = check_config(h, cfg);
  if (st) return st;
  DeviceGuard guard(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = enqueue_update(h, h->pass_grads, h->pass_dtype, cfg, s);
  h->pass_grads = nullptr;
  h->pending = true;
  h->pending_stream = s;
  return st;
}

namespace {

// Enqueues one whole step on s (both passes, or the ZeRO-1 step); waits for
// and returns the result when out != NULL.
int run_step(slm_opt_handle* h, const void* grads, int dtype, int memory,
             const slm_step_config* cfg, slm_step_result* out, cudaStream_t s) {
  int st = SLM_OK;
  if (h->sharded()) {
    if ((st = zero1_step(h, grads, dtype, memory, cfg, s))) return st;
  } else {
    const void* dev = nullptr;
    if ((st = stage_grads(h, grads, dtype, memory, s, &dev))) return st;
    if ((st = phase_begin(h, s))) return st;
    if ((st = enqueue_norm(h, dev, dtype, cfg, s))) return st;
    if ((st = phase_mark(h, s))) return st;
    if ((st = enqueue_update(h, dev, dtype, cfg, s))) return st;
    if ((st = phase_mark(h, s))) return st;
  }
  phase_end(h);
  h->pending = true;
  h->pending_stream = s;
  if (!out) return SLM_OK;
  DeviceStepState ds;
  if ((st = read_state(h, s, &ds))) return st;
  h->pending = false;
  return finish_result(h, ds, out);
}

int release_slot(slm_opt_handle* h, slm_opt_handle::UploadSlot* slot, cudaStream_t s) {
  slot->filled = false;
  slot->consumed_recorded = true;
  return h->cuda(cudaEventRecord(slot->consumed, s), "upload slot release");
}

}  // namespace

int slm_opt_step(slm_opt_handle* h, const void* grads, int dtype, int memory,
                 const slm_step_config* cfg, slm_step_result* out, void* stream) {
  if (!h || !grads) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL argument");
  if (dtype != SLM_DTYPE_F32 && dtype != SLM_DTYPE_BF16)
    return h->err(SLM_ERR_INVALID_ARGUMENT, "unknown gradient dtype");
  int st = check_config(h, cfg);
  if (st) return st;
  if (h->broken)
    return h->err(SLM_ERR_TIMEOUT, "a previous collective timed out; the communicator is closed");
  DeviceGuard guard(h->device);
  return run_step(h, grads, dtype, memory, cfg, out, static_cast<cudaStream_t>(stream));
}

int slm_opt_upload_gradients(slm_opt_handle* h, const void* grads_host, int dtype,
                             int* slot_out) {
  if (!h || !grads_host || !slot_out) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL argument");
  if (dtype != SLM_DTYPE_F32 && dtype != SLM_DTYPE_BF16)
    return h->err(SLM_ERR_INVALID_ARGUMENT, "unknown gradient dtype");
  DeviceGuard guard(h->device);
  int st;
  if (!h->copy_stream &&
      (st = h->cuda(cudaStreamCreateWithFlags(&h->copy_stream, cudaStreamNonBlocking),
                    "copy stream")))
    return st;
  const int k = h->next_up;
  slm_opt_handle::UploadSlot& u = h->up[k];
  if (u.filled)
    return h->err(SLM_ERR_INVALID_ARGUMENT,
                  "both upload slots hold gradients that no step has used yet");
  if (!u.uploaded) {
    if ((st = h->cuda(cudaEventCreateWithFlags(&u.uploaded, cudaEventDisableTiming), "event")) ||
        (st = h->cuda(cudaEventCreateWithFlags(&u.consumed, cudaEventDisableTiming), "event")))
      return st;
  }
  // The slot is rewritten only after the last step that read it has run; the
  // host waits for that, so when this returns nothing on the device still
  // refers to the host buffer of the slot's previous upload.
  if (u.consumed_recorded &&
      (st = h->cuda(cudaEventSynchronize(u.consumed), "upload slot wait")))
    return st;
  const size_t bytes = h->P * (dtype == SLM_DTYPE_F32 ? 4 : 2);
  if (u.bytes < bytes) {
    cudaFree(u.dev);
    u.dev = nullptr;
    u.bytes = 0;
    if ((st = h->cuda(cudaMalloc(&u.dev, bytes), "cudaMalloc upload slot"))) return st;
    u.bytes = bytes;
  }
  if ((st = h->cuda(cudaMemcpyAsync(u.dev, grads_host, bytes, cudaMemcpyHostToDevice,
                                    h->copy_stream),
                    "gradient upload")) ||
      (st = h->cuda(cudaEventRecord(u.uploaded, h->copy_stream), "gradient upload")))
    return st;
  u.filled = true;
  u.dtype = dtype;
  h->next_up ^= 1;
  *slot_out = k;
  return SLM_OK;
}

int slm_opt_step_uploaded(slm_opt_handle* h, int slot, const slm_step_config* cfg,
                          slm_step_result* out, void* stream) {
  if (!h) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL handle");
  if (slot != 0 && slot != 1) return h->err(SLM_ERR_INVALID_ARGUMENT, "upload slot must be 0 or 1");
  slm_opt_handle::UploadSlot& u = h->up[slot];
  if (!u.filled)
    return h->err(SLM_ERR_INVALID_ARGUMENT, "the upload slot holds no gradients to step on");
  int st = check_config(h, cfg);
  if (st) return st;
  if (h->broken)
    return h->err(SLM_ERR_TIMEOUT, "a previous collective timed out; the communicator is closed");
  DeviceGuard guard(h->device);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if ((st = h->cuda(cudaStreamWaitEvent(s, u.uploaded, 0), "upload wait"))) return st;
  // Enqueue, then mark the slot read (even if the enqueue failed part-way, so
  // that the next upload into it waits for whatever did get enqueued), then
  // collect the result.
  st = run_step(h, u.dev, u.dtype, SLM_MEMORY_DEVICE, cfg, nullptr, s);
  const int rel = release_slot(h, &u, s);
  if (st) return st;
  if (rel) return rel;
  if (!out) return SLM_OK;
  DeviceStepState ds;
  if ((st = read_state(h, s, &ds))) return st;
  h->pending = false;
  return finish_result(h, ds, out);
}

int slm_opt_read_result(slm_opt_handle* h, slm_step_result* out) {
  if (!h || !out) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL argument");
  DeviceGuard guard(h->device);
  DeviceStepState ds;
  int st = read_state(h, h->pending ? h->pending_stream : nullptr, &ds);
  if (st) return st;
  h->pending = false;
  return finish_result(h, ds, out);
}

int slm_opt_export_weights_f32(slm_opt_handle* h, float* dst_device, uint64_t n, void* stream) {
  if (!h || !dst_device) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL argument");
  if (n != h->P)
    return h->err(SLM_ERR_INVALID_ARGUMENT, "the f32 weight buffer must hold every parameter");
  if (reinterpret_cast<uintptr_t>(dst_device) % 16 != 0)
    return h->err(SLM_ERR_INVALID_ARGUMENT, "the f32 weight buffer must be 16-byte aligned");
  DeviceGuard guard(h->device);
  return h->cuda(launch_export_f32(h->w16, dst_device, h->P, static_cast<cudaStream_t>(stream)),
                 "weight export kernel");
}

int slm_opt_phase_timing(slm_opt_handle* h, int enable) {
  if (!h) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL handle");
  DeviceGuard guard(h->device);
  PhaseTimer& t = h->timer;
  if (enable && !t.created) {
    for (int i = 0; i < PhaseTimer::kMaxMarks; ++i) {
      const int st = h->cuda(cudaEventCreate(&t.ev[i]), "cudaEventCreate");
      if (st) {
        for (int j = 0; j < i; ++j) cudaEventDestroy(t.ev[j]);
        return st;
      }
    }
    t.created = true;
  }
  t.enabled = enable != 0;
  t.marks = 0;
  t.finished = 0;
  t.steps = 0;
  t.phases = 0;
  t.kind = t.finished_kind = kStepCall;
  for (double& a : t.acc) a = 0.0;
  return SLM_OK;
}

int slm_opt_phase_times(slm_opt_handle* h, double* mean_ms, uint32_t capacity,
                        uint32_t* n_phases, uint64_t* steps) {
  if (!h || !n_phases || !steps || (capacity && !mean_ms))
    return fail(SLM_ERR_INVALID_ARGUMENT, "NULL argument");
  DeviceGuard guard(h->device);
  if (int st = phase_harvest(h)) return st;
  const PhaseTimer& t = h->timer;
  *n_phases = t.phases;
  *steps = t.steps;
  for (uint32_t i = 0; i < capacity && i < t.phases; ++i)
    mean_ms[i] = t.steps ? t.acc[i] / double(t.steps) : 0.0;
  return SLM_OK;
}

const char* slm_opt_phase_name(const slm_opt_handle* h, uint32_t phase) {
  static const char* const kSingle[] = {"norm pass", "update"};
  static const char* const kApply[] = {"gradient upload + sequential clip check", "update"};
  static const char* const kPeer[] = {"gradient barrier + peer reduce",
                                      "finalize + update + weight stores + weight barrier"};
  static const char* const kNccl[] = {"gradient all-to-all", "reduce", "partials all-gather",
                                      "finalize", "update", "weight all-gather"};
  if (!h) return nullptr;
  if (h->timer.kind == kApplyUpdateCall) return phase < 2 ? kApply[phase] : nullptr;
  if (!h->sharded()) return phase < 2 ? kSingle[phase] : nullptr;
  if (h->exchange == SLM_ZERO1_PEER) return phase < 2 ? kPeer[phase] : nullptr;
  return phase < 6 ? kNccl[phase] : nullptr;
}

int slm_opt_apply_update(slm_opt_handle* h, const float* grads_host, uint64_t n,
                         float learning_rate, uint64_t one_based_update,
                         uint64_t valid_targets, char* out_sha256_hex65) {
  (void)valid_targets;  // unused by the reference's CUDA backend (cuda_backend.rs:245)
  if (!h || !grads_host) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL argument");
  if (h->sharded())
    return h->err(SLM_ERR_INVALID_ARGUMENT,
                  "apply_update is the single-replica drop-in; use slm_opt_step for ZeRO-1");
  // trainer.rs:235-249: one FP32 gradient per parameter.
  if (n != h->P) {
    char msg[192];
    std::snprintf(msg, sizeof(msg),
                  "AdamW requires one FP32 gradient per parameter: update %llu supplied %llu "
                  "for %llu parameters",
                  (unsigned long long)one_based_update, (unsigned long long)n,
                  (unsigned long long)h->P);
    return h->err(SLM_ERR_P12_OPTIMIZER_GRADIENT_INVALID, msg);
  }
  slm_step_config cfg;
  slm_step_config_default(&cfg);
  cfg.learning_rate = finite_f32(learning_rate) ? learning_rate : 0.0f;
  cfg.one_based_update = one_based_update >= 1 && one_based_update <= 0x7fffffffu
                             ? uint32_t(one_based_update)
                             : 1u;
  cfg.apply_clip = 0;  // the input is already clipped
  cfg.nonfinite_policy = SLM_NONFINITE_ERROR;
  cfg.loss_scale_mode = SLM_SCALE_STATIC;
  cfg.static_loss_scale = 1.0f;

  DeviceGuard guard(h->device);
  cudaStream_t s = nullptr;
  const void* dev = nullptr;
  int st = phase_begin(h, s);
  if (st) return st;
  // Re-verification first (trainer.rs:250-260), with the reference's own
  // sequential f32 clip scale so that the accept / reject decision is the
  // reference's; nothing is written on failure.  From pageable memory the
  // check runs slice by slice as the slices land, overlapping the upload.
  const size_t bytes = h->P * sizeof(float);
  if (is_pageable(grads_host) && bytes > slm_opt_handle::PinnedRing::kSlotBytes) {
    if ((st = ensure_staging(h, bytes))) return st;
    float* staged = static_cast<float*>(h->d_staging);
    const SeqClipOut out{h->d_state, nullptr, nullptr, nullptr};
    st = stage_pageable(h, staged, grads_host, bytes, s,
                        [&](size_t off, size_t len, cudaEvent_t landed) {
                          int r = h->cuda(cudaStreamWaitEvent(s, landed, 0), "upload wait");
                          if (r) return r;
                          const uint64_t e0 = off / sizeof(float), ne = len / sizeof(float);
                          return h->cuda(launch_sequential_clip(staged + e0, ne, out,
                                                                &h->d_state->kernel_error, s,
                                                                h->d_seq_carry, e0 != 0,
                                                                e0 + ne == h->P, h->d_seq_ws,
                                                                h->seq_ws_bytes),
                                         "clip check kernel");
                        });
    if (st) return st;
    dev = staged;
  } else {
    if ((st = stage_grads(h, grads_host, SLM_DTYPE_F32, SLM_MEMORY_HOST, s, &dev))) return st;
    if ((st = h->cuda(launch_reference_clip(static_cast<const float*>(dev), h->P, h->d_state, s,
                                            h->d_seq_ws, h->seq_ws_bytes),
                      "clip check kernel")))
      return st;
  }
  if ((st = phase_mark(h, s))) return st;
  DeviceStepState ds;
  if ((st = read_state(h, s, &ds))) return st;
  if (ds.kernel_error) return h->err(SLM_ERR_INTERNAL, "the clip check's copy pipeline stalled");
  if (ds.status == SLM_ERR_MODEL_GRADIENT_NONFINITE)
    return h->err(ds.status, "OPT-001 rejects non-finite unscaled gradients");
  if (ds.status == SLM_ERR_MODEL_GRADIENT_NORM_NONFINITE)
    return h->err(ds.status, "OPT-001 global gradient norm is non-finite");
  if (ds.status != SLM_OK) return h->err(SLM_ERR_INTERNAL, "unexpected clip check status");
  const float tolerance = 0.05f;  // CLIP_VERIFICATION_TOLERANCE, trainer.rs:161
  if (ds.clip_scale < 1.0f - tolerance) {
    char msg[192];
    std::snprintf(msg, sizeof(msg),
                  "AdamW requires globally clipped FP32 gradients: update %llu re-measured a "
                  "clip scale of %e, outside the 0.05 verification tolerance of 1.0",
                  (unsigned long long)one_based_update, double(ds.clip_scale));
    return h->err(SLM_ERR_P12_OPTIMIZER_GRADIENT_INVALID, msg);
  }
  // trainer.rs:262-273: u32 index, then the frozen schedule's exact lr bits.
  if (one_based_update > 0xffffffffull)
    return h->err(SLM_ERR_P12_UPDATE_INDEX_INVALID,
                  "the optimizer update index cannot be represented canonically");
  float expected = 0.0f;
  if ((st = slm_canonical_learning_rate(one_based_update, &expected)))
    return h->err(st, g_last_error);
  if (f32_bits(learning_rate) != f32_bits(expected))
    return h->err(SLM_ERR_P12_SCHEDULER_STATE_MISMATCH,
                  "AdamW received a learning rate that differs from the frozen schedule");
  cfg.learning_rate = learning_rate;
  cfg.one_based_update = uint32_t(one_based_update);
  if ((st = enqueue_update(h, dev, SLM_DTYPE_F32, &cfg, s))) return st;
  if ((st = phase_mark(h, s))) return st;
  phase_end(h, kApplyUpdateCall);
  if ((st = read_state(h, s, &ds))) return st;
  if (ds.result_nonfinite)
    return h->err(SLM_ERR_MODEL_OPTIMIZER_RESULT_NONFINITE, "OPT-001 produced non-finite state");
  if (out_sha256_hex65) return slm_opt_state_sha256(h, out_sha256_hex65);
  return SLM_OK;
}

int slm_opt_state_sha256(slm_opt_handle* h, char out_hex[65]) {
  if (!h || !out_hex) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL argument");
  int st = slm_opt_validate_state(h);
  if (st) return st;
  DeviceGuard guard(h->device);
  // Full host copies (gathered for a ZeRO-1 handle: collective).
  std::vector<float> master(h->P), m1(h->P), m2(h->P);
  std::vector<uint16_t> w16(h->P);
  if ((st = download_role(h, SLM_ROLE_MASTER_F32, master.data(), h->P * 4))) return st;
  if ((st = download_role(h, SLM_ROLE_MOMENT1_F32, m1.data(), h->P * 4))) return st;
  if ((st = download_role(h, SLM_ROLE_MOMENT2_F32, m2.data(), h->P * 4))) return st;
  if ((st = download_role(h, SLM_ROLE_PARAMETERS_BF16, w16.data(), h->P * 2))) return st;
  // trainer.rs:297-320: tag (with NUL), then per tensor: name length (u64 LE),
  // name, decay byte, element count (u64 LE), master, bf16, m, v (LE bytes;
  // x86-64 and the device are little-endian, so the arrays hash as stored).
  Sha256 sha;
  static const char tag[] = "python-slm/adamw-state/v1";
  sha.update(tag, sizeof(tag));
  for (size_t k = 0; k < h->names.size(); ++k) {
    const uint64_t lo = h->offsets[k], count = h->offsets[k + 1] - lo;
    uint8_t le[8];
    const uint64_t name_len = h->names[k].size();
    for (int b = 0; b < 8; ++b) le[b] = uint8_t(name_len >> (8 * b));
    sha.update(le, 8);
    sha.update(h->names[k].data(), name_len);
    const uint8_t d = h->decay[k];
    sha.update(&d, 1);
    for (int b = 0; b < 8; ++b) le[b] = uint8_t(count >> (8 * b));
    sha.update(le, 8);
    sha.update(master.data() + lo, count * 4);
    sha.update(w16.data() + lo, count * 2);
    sha.update(m1.data() + lo, count * 4);
    sha.update(m2.data() + lo, count * 4);
  }
  uint8_t digest[32];
  sha.final(digest);
  Sha256::hex(digest, out_hex);
  return SLM_OK;
}

}  // extern "C"
