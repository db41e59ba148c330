/*
 * slmopt.h -- C ABI of the B200 optimizer step for python-slm's gqa-135m-v1.
 *
 * One opaque handle owns the optimizer state of one model replica (or one
 * ZeRO-1 shard of it) in HBM, in the reference's PARAM-001 flat order:
 *   master weights f32[P], first moments f32[P], second moments f32[P],
 *   bf16 weight storage u16[P], and the tensor table {name, elements, decay}.
 * Gradients are borrowed for the duration of a call (device pointer, or a host
 * pointer that the call copies in).  All device work is issued on the stream
 * the caller passes (NULL = the legacy default stream).  No exception crosses
 * this boundary; every entry point returns an slm_status.
 *
 * Citations are to the dhilipsiva/python-slm sources (path:line) whose
 * interface each entry point replaces.  No torch type appears here.
 */
#ifndef SLMOPT_H
#define SLMOPT_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define SLMOPT_ABI_VERSION 1

/* Status codes.  Each maps 1:1 onto a reference ProductError code
 * (src/error.rs:16-93) and its category / process exit code (error.rs:85-93):
 * Internal=1, Usage=2, Integrity=3, Environment=4, Gate=5. */
typedef enum slm_status {
    SLM_OK = 0,
    /* Gate (5): src/model/oracle.rs:489-494, :499-503, :519-531, :544-552 */
    SLM_ERR_MODEL_GRADIENT_NONFINITE = 10,
    SLM_ERR_MODEL_GRADIENT_NORM_NONFINITE = 11,
    SLM_ERR_MODEL_OPTIMIZER_INPUT_INVALID = 12,
    SLM_ERR_MODEL_OPTIMIZER_RESULT_NONFINITE = 13,
    /* Integrity (3): src/train/trainer.rs:240-273, :163-189, :102-119 */
    SLM_ERR_P12_OPTIMIZER_GRADIENT_INVALID = 20,
    SLM_ERR_P12_SCHEDULER_STATE_MISMATCH = 21,
    SLM_ERR_P12_OPTIMIZER_STATE_INVALID = 22,
    SLM_ERR_P12_UPDATE_INDEX_INVALID = 23,
    SLM_ERR_P12_SCHEDULE_INDEX_INVALID = 24,
    SLM_ERR_E1_PARAMETER_LAYOUT_MISMATCH = 25,       /* full_state.rs:218-236 */
    SLM_ERR_E1_STATE_ARTIFACT_INVALID = 26,          /* full_state.rs:467-480 */
    SLM_ERR_P12_OPTIMIZER_PARAMETER_DUPLICATE = 27,  /* trainer.rs:199-206 */
    /* Usage (2) */
    SLM_ERR_INVALID_ARGUMENT = 30,
    SLM_ERR_SIZE_LIMIT = 31,
    /* Environment (4) */
    SLM_ERR_CUDA = 40,
    SLM_ERR_OUT_OF_MEMORY = 41,
    SLM_ERR_NCCL = 42,
    SLM_ERR_TIMEOUT = 43,
    SLM_ERR_NO_DEVICE = 44,
    /* Internal (1) */
    SLM_ERR_INTERNAL = 50
} slm_status;

/* The reference's ProductError.code string for a status, e.g.
 * "MODEL_GRADIENT_NONFINITE"; "OK" for SLM_OK. */
const char* slm_status_code_string(int status);
/* The reference's exit code of the status's category (src/error.rs:85-93); 0 for SLM_OK. */
int slm_status_category(int status);
/* Human-readable detail of the last failure on this thread (never NULL). */
const char* slm_last_error_message(void);
int slm_abi_version(void);

typedef struct slm_opt_handle slm_opt_handle;

/* One row of the PARAM-001 tensor table (src/model/oracle.rs:177-275,
 * src/train/full_state.rs:113-154).  weight_decay follows weight_decay_for
 * (full_state.rs:179-181): 0 exactly for names ending in "norm.weight". */
typedef struct slm_tensor_spec {
    const char* name;
    uint64_t elements;
    uint32_t weight_decay;
} slm_tensor_spec;

/* Artifact roles of the five-artifact checkpoint (src/train/full_state.rs:27-36);
 * the runtime JSON stays with the host. */
typedef enum slm_role {
    SLM_ROLE_PARAMETERS_BF16 = 0, /* model/parameters.bf16, u16 LE */
    SLM_ROLE_MASTER_F32 = 1,      /* optimizer/master.f32 */
    SLM_ROLE_MOMENT1_F32 = 2,     /* optimizer/adamw-m1.f32 */
    SLM_ROLE_MOMENT2_F32 = 3      /* optimizer/adamw-m2.f32 */
} slm_role;

typedef enum slm_dtype { SLM_DTYPE_F32 = 0, SLM_DTYPE_BF16 = 1 } slm_dtype;
typedef enum slm_memory { SLM_MEMORY_DEVICE = 0, SLM_MEMORY_HOST = 1 } slm_memory;
typedef enum slm_nonfinite_policy {
    SLM_NONFINITE_SKIP = 0,  /* skip the update, state bit-unchanged, halve a dynamic scale */
    SLM_NONFINITE_ERROR = 1  /* reference behaviour: MODEL_GRADIENT_NONFINITE, state unchanged */
} slm_nonfinite_policy;
typedef enum slm_scale_mode {
    SLM_SCALE_STATIC = 0,  /* divide by static_loss_scale (1 for plain fp32 gradients) */
    SLM_SCALE_DYNAMIC = 1  /* divide by the handle's device-resident dynamic loss scale */
} slm_scale_mode;

/* Hyperparameters of one step.  The reference freezes them as constants
 * (src/model/oracle.rs:469-484, src/train/trainer.rs:276); here they are
 * explicit.  slm_step_config_default() fills OPT-001's values. */
typedef struct slm_step_config {
    float learning_rate;
    uint32_t one_based_update;  /* t >= 1; bias corrections use f32 powi(beta, t) */
    float beta1, beta2, epsilon;
    float decay_weight;         /* for tensors with weight_decay=1 (0.1) */
    float no_decay_weight;      /* for the RMSNorm scales (0.0) */
    float max_grad_norm;        /* global L2 clip (1.0) */
    int32_t apply_clip;         /* 1: g *= clip; 0: measure only (pre-clipped input) */
    float min_clip_accept;      /* >0: reject (no update) when clip < this (0.95 verification) */
    int32_t nonfinite_policy;   /* slm_nonfinite_policy */
    int32_t loss_scale_mode;    /* slm_scale_mode */
    float static_loss_scale;    /* divisor under SLM_SCALE_STATIC */
    uint32_t growth_interval;   /* dynamic scale doubles after this many applied steps */
} slm_step_config;

typedef struct slm_step_result {
    double sum_squares;        /* fixed-tree f64 sum of the unscaled gradients' squares */
    double grad_norm;          /* sqrt(sum_squares) */
    float clip_scale;          /* min(max_norm / sqrtf((float)sum), 1); 1 when the sum is 0 */
    float loss_scale_used;
    float next_loss_scale;
    uint32_t skipped;          /* 1: no state was written */
    uint32_t nonfinite;        /* 1: an unscaled gradient was inf/nan */
    uint32_t result_nonfinite; /* 1: AdamW produced non-finite state */
    uint32_t rejected;         /* 1: clip verification failed */
    uint32_t good_steps;       /* dynamic scaler's consecutive applied steps */
    int32_t status;            /* slm_status of the step */
} slm_step_result;

void slm_step_config_default(slm_step_config* cfg);

/* ---- lifetime ------------------------------------------------------------- */

/* Allocate the state for the tensor table on `device`; every buffer zeroed.
 * Replaces CudaTrainerBackend::from_state / FullModelState::new
 * (src/train/cuda_backend.rs:56-73, src/train/full_state.rs:206-245).
 * Rejects empty tables, empty or duplicate names. */
int slm_opt_create(const slm_tensor_spec* table, uint32_t n_tensors, int device,
                   slm_opt_handle** out);
/* Waits for the device's outstanding work, then frees the handle. */
int slm_opt_destroy(slm_opt_handle* h);
uint64_t slm_opt_parameter_count(const slm_opt_handle* h);
/* Human-readable detail of the handle's last failure (never NULL). */
const char* slm_opt_last_error(const slm_opt_handle* h);

/* Masters from host f32[P]; bf16 = RNE(master), moments zero, as
 * FullModelState::initialize_canonical does (src/train/full_state.rs:259-291). */
int slm_opt_init_master(slm_opt_handle* h, const float* master_host, void* stream);

/* ---- checkpoint codec (src/train/full_state.rs:387-520) --------------------- */

/* Copy one artifact out (D2H, little-endian flat bytes in PARAM-001 order).
 * `bytes` must equal the artifact size (2P or 4P).  Synchronous. */
int slm_opt_snapshot(slm_opt_handle* h, int role, void* host_dst, uint64_t bytes);
/* Copy one artifact in (H2D).  Call slm_opt_validate_state after the last one. */
int slm_opt_restore(slm_opt_handle* h, int role, const void* host_src, uint64_t bytes);
/* AdamwParameterState::validate (src/train/trainer.rs:163-189) on the device:
 * all master/m/v finite and bf16 == RNE(master), else
 * SLM_ERR_P12_OPTIMIZER_STATE_INVALID.  Synchronous. */
int slm_opt_validate_state(slm_opt_handle* h);
/* Device address of one state buffer (for in-place use of the bf16 weights). */
int slm_opt_device_buffer(slm_opt_handle* h, int role, void** out_device_ptr);

/* CanonicalAdamw::state_sha256 (src/train/trainer.rs:297-320): validates, then
 * SHA-256 over tag, name, decay, count, master, bf16, m, v per tensor.
 * Synchronous; downloads the whole state.  Not on the step's timed path. */
int slm_opt_state_sha256(slm_opt_handle* h, char out_hex[65]);

/* ---- the step --------------------------------------------------------------- */

/* Fused mixed-precision step: unscale -> non-finite check -> fixed-tree f64
 * norm -> clip -> AdamW (fp32 master/m/v) -> bf16 weight copy, and the loss
 * scaler.  Subsumes src/train/trainer.rs:884-904 plus
 * CudaTrainerBackend::apply_update (src/train/cuda_backend.rs:240-258).
 * `grads` holds P elements of `dtype` in `memory`.  If `out` is non-NULL the
 * call waits for the stream and fills it (status included); if NULL the call
 * only enqueues, and slm_opt_read_result() collects the result later.
 * The skip path (non-finite gradient under SLM_NONFINITE_SKIP) is a success. */
int slm_opt_step(slm_opt_handle* h, const void* grads, int dtype, int memory,
                 const slm_step_config* cfg, slm_step_result* out, void* stream);
/* Wait for the handle's last enqueued step on its stream and return its result. */
int slm_opt_read_result(slm_opt_handle* h, slm_step_result* out);

/* Pipelined host gradients (the reference hands apply_update a host slice
 * every update, src/train/trainer.rs:902-904).  slm_opt_step with host memory
 * uploads on the step's own stream, so the PCIe copy and the step's kernels
 * run one after the other.  slm_opt_upload_gradients instead copies P
 * gradients of `dtype` from host memory (pinned for an asynchronous copy)
 * into one of two device slots on the handle's own copy stream and returns
 * the slot; slm_opt_step_uploaded(slot) then runs the step on `stream` once
 * that copy has landed.  Uploading the next update's gradients before
 * stepping on the current ones overlaps the copy with the step.  The copy
 * does not wait for earlier work on any caller stream: the host buffer must
 * hold its final contents when the upload is called and stay valid until the
 * step that uses it has run.  Before reusing a slot the upload waits on the
 * host until the step that read it has run (so the buffer of that slot's
 * previous upload is free again when it returns); a third upload before
 * either slot was stepped on is rejected. */
int slm_opt_upload_gradients(slm_opt_handle* h, const void* grads_host, int dtype,
                             int* slot_out);
int slm_opt_step_uploaded(slm_opt_handle* h, int slot, const slm_step_config* cfg,
                          slm_step_result* out, void* stream);

/* The bf16 weights as f32 -- each value exactly bf16_bits_to_f32 of the bf16
 * copy, the values the reference reloads into its graph after every update
 * (CudaTrainerBackend::reload_graph, src/train/cuda_backend.rs:169-177 ->
 * FullModelGraph::load, src/model/accelerator/full_model.rs:212-251) -- written
 * on the device into dst_device (n == P floats, 16-byte aligned, PARAM-001
 * order; a [rows, columns] tensor is its row-major slice), enqueued on
 * `stream` after the step.  No host round trip; a ZeRO-1 handle exports its
 * full gathered copy. */
int slm_opt_export_weights_f32(slm_opt_handle* h, float* dst_device, uint64_t n, void* stream);

/* Per-phase device timing of slm_opt_step (diagnostics; no counterpart in the
 * reference, whose step is one host loop).  While enabled, every step records
 * CUDA events on its stream at its phase boundaries, and the next step first
 * waits for the previous one to fold its intervals into running sums, so
 * steps no longer overlap the host: keep it off in timed runs.  Enabling
 * (again) clears the sums.  slm_opt_phase_times writes up to `capacity` mean
 * phase durations in ms, the phase count and the number of steps timed;
 * slm_opt_phase_name names phase i for this handle's mode (NULL past the end):
 *   one GPU:         norm pass, update
 *   ZeRO-1 peer:     gradient barrier + peer reduce,
 *                    finalize + update + weight stores + weight barrier
 *   ZeRO-1 NCCL:     gradient all-to-all, reduce, partials all-gather,
 *                    finalize, update, weight all-gather
 *   slm_opt_apply_update: gradient upload + sequential clip check (overlapped
 *                    slice by slice for pageable host memory), update
 * A host gradient's upload is not part of any slm_opt_step phase.  The sums
 * describe one entry point: a timed call of the other (slm_opt_step versus
 * slm_opt_apply_update) starts them afresh. */
int slm_opt_phase_timing(slm_opt_handle* h, int enable);
int slm_opt_phase_times(slm_opt_handle* h, double* mean_ms, uint32_t capacity,
                        uint32_t* n_phases, uint64_t* steps);
const char* slm_opt_phase_name(const slm_opt_handle* h, uint32_t phase);

/* slm_opt_step split in its two device passes, both enqueue-only:
 *   slm_opt_norm_pass   -- stage (host) gradients, unscale, non-finite check,
 *                          fixed-tree norm, clip / skip decision, scaler update
 *                          (the reference's trainer.rs:884-901);
 *   slm_opt_update_pass -- AdamW + bf16 weight write over the gradients the
 *                          norm pass saw (CanonicalAdamw's loop, trainer.rs:274-293).
 * The gradient buffer must stay valid until the update pass has run; cfg must
 * be the same for both.  Lets a caller overlap the norm pass with other work
 * or time each pass with its own events. */
int slm_opt_norm_pass(slm_opt_handle* h, const void* grads, int dtype, int memory,
                      const slm_step_config* cfg, void* stream);
int slm_opt_update_pass(slm_opt_handle* h, const slm_step_config* cfg, void* stream);

/* The strict drop-in for TrainerBackend::apply_update (src/train/trainer.rs:512-518)
 * as CudaTrainerBackend implements it (src/train/cuda_backend.rs:240-258 ->
 * CanonicalAdamw::apply_normalized_clipped_gradients, trainer.rs:222-295):
 * n must equal P (else P12_OPTIMIZER_GRADIENT_INVALID); non-finite gradients
 * fail with MODEL_GRADIENT_NONFINITE; the clip is re-verified (tolerance 0.05,
 * trainer.rs:161) with the reference's own sequential f32 clip scale
 * (gradient_clip_scale, src/model/oracle.rs:486-507, reproduced bit for bit
 * on the device, so the accept / reject decision is the reference's even where
 * that sum drifts from the exact one; see slm_gradient_clip_scale); from
 * pageable host memory the gradients travel through a pinned ring of three
 * 32 MB slots filled by host threads with streaming stores (half the host's
 * hardware threads, at most 8; the environment variable SLM_STAGING_THREADS,
 * 1..64, overrides), and the check runs slice by slice as they land; the lr
 * must bit-equal canonical_learning_rate(t) (P12_SCHEDULER_STATE_MISMATCH);
 * AdamW runs with
 * OPT-001's constants and no further clip.  `grads_host` is host f32[n].
 * valid_targets is accepted and unused, as in the reference.  If out_sha256
 * is non-NULL it receives the post-update state SHA-256 (slow, off-path). */
int slm_opt_apply_update(slm_opt_handle* h, const float* grads_host, uint64_t n,
                         float learning_rate, uint64_t one_based_update,
                         uint64_t valid_targets, char* out_sha256_hex65);

/* The reference's gradient_clip_scale (src/model/oracle.rs:486-507), which the
 * trainer applies to the normalised gradients (src/train/trainer.rs:897) and
 * CanonicalAdamw re-checks (trainer.rs:250-260), on the device and bit for
 * bit: the sequential f32 sum of squares s <- fl(s + fl(g * g)) over
 * g[0..n), then min(1 / sqrtf(s), 1), or 1 when s == 0.  It is computed in
 * parallel by an exact method (while s stays in one binade each add is an
 * integer number of ulps; only the terms where s changes binade or an add
 * ties are added one at a time), about 2,000x faster than adding 135M terms
 * in order.  grads_device: n f32 in device memory, 16-byte aligned.  The
 * result is written to out_device (device memory, stream-ordered on
 * `stream`): status 0, MODEL_GRADIENT_NONFINITE (a gradient is inf or NaN;
 * takes precedence, as in the reference) or MODEL_GRADIENT_NORM_NONFINITE
 * (the sum overflowed); kernel_error 1 if the kernel's copy pipeline stalled
 * (never expected).  Allocates nothing; one CTA streams the n terms
 * (about 0.25 ms per million).  slm_gradient_clip_scale_ws gives the same
 * bits with every SM: workspace_device (device memory, 16-byte aligned, at
 * least slm_gradient_clip_workspace_bytes(n) bytes -- 29 per 8,192 gradients,
 * rounded up to 16) receives per-window summaries computed in parallel (the
 * window's exact f64 sum and, for the few binades the running sum can be in
 * there, its integer ulp total and whether an add ties), which one CTA then
 * chains in order, adding a window term by term only where no summary fits.
 * A workspace that is too small or misaligned is INVALID_ARGUMENT; NULL
 * selects the single-CTA form. */
typedef struct slm_clip_result {
    float sum_squares;     /* the reference's sequential f32 sum */
    float clip_scale;
    int32_t status;
    uint32_t kernel_error;
} slm_clip_result;
int slm_gradient_clip_scale(const float* grads_device, uint64_t n, slm_clip_result* out_device,
                            void* stream);
uint64_t slm_gradient_clip_workspace_bytes(uint64_t n);
int slm_gradient_clip_scale_ws(const float* grads_device, uint64_t n, void* workspace_device,
                               uint64_t workspace_bytes, slm_clip_result* out_device,
                               void* stream);

/* ---- micro-batch accumulation ---------------------------------------------------
 * The reference sums each micro-batch's fp32 gradient into a host accumulator
 * (src/train/trainer.rs:856-877, `total += value`) and normalises by the
 * update's target count (:884).  On the device: slm_grad_accumulate adds
 * `micro` (n elements of dtype, device memory) into the f32 accumulator in the
 * same per-element order (overwrite=1 starts an update: acc = micro).  The last
 * micro-batch of an update can instead go through slm_opt_norm_pass_accumulate,
 * which accumulates and runs the norm pass over the sums in one read (unscale
 * by cfg's loss scale -- the target count for the reference's normalisation
 * -- non-finite check, fixed-tree norm, clip / skip); follow it with
 * slm_opt_update_pass(h, cfg, stream), which reads `acc` as f32 gradients.
 * A non-finite sum is caught by the norm pass (the reference stops at the
 * micro-batch that produced it; the outcome -- no update -- is the same). */
int slm_grad_accumulate(float* acc_device, const void* micro_device, int dtype, uint64_t n,
                        int overwrite, void* stream);
int slm_opt_norm_pass_accumulate(slm_opt_handle* h, float* acc_device, const void* micro,
                                 int dtype, int memory, int overwrite,
                                 const slm_step_config* cfg, void* stream);

/* ---- ZeRO-1 data parallel (no counterpart in the reference, which runs one
 * device per process, src/train/cuda_backend.rs:56-73) ---------------------------
 * One handle per rank and GPU.  The flat buffer is cut into 65,536-element
 * chunks, the chunk count padded to a multiple of `world`; rank r owns the
 * chunk-aligned element range slm_opt_shard_range() reports and keeps master /
 * m / v for it, plus the full bf16 weights.  slm_opt_step() on such a handle
 * takes this rank's full local gradient (P elements) and runs: all-to-all of
 * gradient slices, f32 sum in rank order 0..N-1 fused with the unscale and the
 * norm partials, all-gather of the partials, the same fixed-tree finalize on
 * every rank, AdamW on the shard, in-place all-gather of the bf16 weights.
 * The result equals a single replica's step on the rank-ordered f32 sum of the
 * gradients, bit for bit.  Collective entry points (every rank calls them in
 * the same order): slm_opt_create_zero1, slm_opt_step, slm_opt_init_master,
 * slm_opt_snapshot of a full f32 role, slm_opt_state_sha256.  Waits are
 * bounded by timeout_ms (0 = 300 s); on expiry the communicator is aborted and
 * the call returns SLM_ERR_TIMEOUT.  With the peer-memory exchange (the
 * default when every rank can map every other rank's memory) each device-side
 * wait is bounded by min(timeout_ms, 10 s); a rank that gives up reports
 * SLM_ERR_TIMEOUT from the step and its handle refuses further steps.
 * Teardown: the ranks read and write each other's buffers during a step, so
 * after a failed step every rank should return from its own step (each is
 * bounded) and the ranks should agree on the host before any of them calls
 * slm_opt_destroy, which frees the buffers the others have mapped. */

/* A fresh NCCL unique id (128 bytes) for rank 0 to share with the others. */
int slm_zero1_unique_id(uint8_t out[128]);
int slm_opt_create_zero1(const slm_tensor_spec* table, uint32_t n_tensors, int device, int rank,
                         int world, const uint8_t unique_id[128], uint32_t timeout_ms,
                         slm_opt_handle** out);
/* This rank's element range [begin, begin + len) of the flat buffer. */
int slm_opt_shard_range(const slm_opt_handle* h, uint64_t* begin, uint64_t* len);

/* How a ZeRO-1 step moves data between ranks.  SLM_ZERO1_PEER (the default
 * when every rank could map every other rank's buffers with CUDA IPC at
 * creation): the reduce kernel reads the other ranks' gradient slices over
 * NVLink directly from their registered gradient buffers, the update kernel
 * stores its bf16 results straight into every rank's weights, and ranks meet
 * at bounded device-side flag barriers.  SLM_ZERO1_NCCL: NCCL send/recv and
 * all-gathers with a staging buffer.  Both give bit-identical results. */
typedef enum slm_zero1_exchange { SLM_ZERO1_NCCL = 0, SLM_ZERO1_PEER = 1 } slm_zero1_exchange;
/* Collective: every rank must select the same exchange before its next step.
 * SLM_ZERO1_PEER fails with SLM_ERR_INVALID_ARGUMENT if it was not set up. */
int slm_opt_zero1_set_exchange(slm_opt_handle* h, int exchange);
int slm_opt_zero1_exchange(const slm_opt_handle* h);
/* The rank's registered gradient buffer (bytes = 4P; holds P bf16 or P f32
 * gradients).  A step given this pointer reads it in place (the other ranks
 * read their slices of it); any other gradient pointer is first copied into
 * it.  Do not overwrite it while a step that reads it is in flight. */
int slm_opt_gradient_buffer(slm_opt_handle* h, void** out_device_ptr, uint64_t* bytes);

/* ---- gradient norm without allocation -----------------------------------------
 * No counterpart in the reference.  For callers that cannot call cudaMalloc
 * where they need the norm (another allocator owns the HBM budget, a latency-
 * critical loop must not take cudaMalloc's device-wide synchronisation, or all
 * memory is reserved up front): the fixed-tree f64 norm, clip scale and
 * non-finite flag of `n` gradients of `dtype` on the current device, divided by
 * `loss_scale` -- the same values an optimizer handle's norm pass computes.
 * Its scratch is a fixed file-scope device array (about 33 KB on every GPU that
 * loads the library, held until exit), so nothing is allocated; n above
 * SLM_NOALLOC_MAX_ELEMENTS is rejected with SLM_ERR_SIZE_LIMIT.  The result is
 * written to the caller's device memory `out_device` (8-byte aligned),
 * stream-ordered on `stream`; `grads` must be aligned to its element size.
 * The first call on a device looks up the array's device address and caches
 * it, so make that first call before any stream capture, and do not call this
 * entry point on a device after cudaDeviceReset (the reset unloads the array).
 * All calls on a device share the array: calls whose work overlaps on the GPU
 * race. */
#define SLM_NOALLOC_MAX_ELEMENTS 268435456ull /* 2^28 elements = 4,096 chunks */
typedef struct slm_norm_result {
    double sum_squares;  /* fixed-tree f64 sum of (g / loss_scale)^2 */
    double grad_norm;    /* sqrt(sum_squares) */
    float clip_scale;    /* min(max_grad_norm / sqrtf((float)sum), 1); 1 when the sum is 0 */
    uint32_t nonfinite;  /* 1 when a gradient or the f32 sum is inf/nan (clip_scale is then 0) */
} slm_norm_result;
int slm_grad_norm_noalloc(const void* grads, int dtype, uint64_t n, float loss_scale,
                          float max_grad_norm, slm_norm_result* out_device, void* stream);

/* ---- loss scaler ------------------------------------------------------------- */
int slm_opt_set_loss_scale(slm_opt_handle* h, float scale, uint32_t good_steps);
int slm_opt_get_loss_scale(slm_opt_handle* h, float* scale, uint32_t* good_steps);

/* ---- lr schedule (host, scalar) ---------------------------------------------- */

/* src/train/trainer.rs:102-119 canonical_learning_rate: bit-exact f32 result. */
int slm_canonical_learning_rate(uint64_t one_based_update, float* out);
/* The same warmup + cosine form over explicit constants. */
int slm_schedule_learning_rate(uint64_t one_based_update, float peak, float minimum,
                               uint64_t warmup, uint64_t total, float* out);

#ifdef __cplusplus
}
#endif
#endif /* SLMOPT_H */
