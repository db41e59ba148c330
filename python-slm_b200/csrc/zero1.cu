// ZeRO-1 data-parallel optimizer step over NVLink 5 / NVSwitch: peer memory
// (default) or NCCL.
//
// Partition: the flat PARAM-001 buffer is cut into 65,536-element chunks; the
// chunk count is padded to a multiple of the world size and rank r owns
// chunks [r*Cr, (r+1)*Cr), i.e. elements [r*S, r*S + S) with S = Cr * 65,536
// (clipped to P).  Shards are chunk-aligned, so every norm partial is formed
// from exactly the same elements, in the same order, as on a single replica.
//
// Peer-memory step (every rank maps every other rank's gradient buffer,
// partials area, flags and bf16 weights with CUDA IPC), two kernels on the
// caller's stream:
//   1. zero1_peer_reduce_kernel: gradient barrier, then this shard's slices of
//      every rank's gradient buffer pulled with bulk copies (NVLink for the
//      peers), f32 sum in rank order 0..N-1, unscale, chunk partials pushed to
//      every rank, partials flag;
//   2. zero1_peer_update_kernel: every block waits for all ranks' partials and
//      reduces them with the single-replica tree (same decision everywhere),
//      AdamW on the shard with each bf16 tile bulk-stored to every rank, and
//      the last block's weight barrier.
//
// NCCL step, all on the caller's stream:
//   1. all-to-all of gradient slices (grouped ncclSend/ncclRecv): rank r
//      receives slice r of every rank's gradient;
//   2. zero1_reduce_kernel: f32 sum in rank order 0..N-1, unscale, chunk
//      partials, non-finite flag;
//   3. ncclAllGather of the partials + flag (a few KB);
//   4. zero1_finalize_kernel: every rank reduces all partials in global chunk
//      order -> the same norm / clip / skip bits as one GPU;
//   5. adamw_update_kernel on the shard (fp32 master/m/v), writing its bf16 slice;
//   6. in-place ncclAllGather of the bf16 weights.
// NCCL's own reduce-scatter would add in bf16 in an algorithm-dependent order;
// moving the slices and summing them locally keeps the result deterministic.
//
// The communicator is non-blocking; every wait on it (init, group end, the
// step's stream) is bounded by the handle's timeout, after which the
// communicator is aborted and the call returns SLM_ERR_TIMEOUT.
#include "handle.h"

#include <nccl.h>

#include <algorithm>
#include <chrono>
#include <new>
#include <thread>
#include <vector>

using namespace slmopt;

namespace {

using Clock = std::chrono::steady_clock;

ncclComm_t comm_of(const slm_opt_handle* h) { return static_cast<ncclComm_t>(h->comm); }

double elapsed_ms(Clock::time_point t0) {
  return std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
}

void abort_comm(slm_opt_handle* h) {
  if (h->comm) ncclCommAbort(comm_of(h));
  h->comm = nullptr;
  h->broken = true;
}

int nccl_fail(slm_opt_handle* h, ncclResult_t r, const char* what) {
  std::string msg = std::string(what) + ": " + ncclGetErrorString(r);
  if (h->comm) {
    const char* last = ncclGetLastError(comm_of(h));
    if (last && *last) msg += std::string(" (") + last + ")";
  }
  abort_comm(h);
  return h->err(SLM_ERR_NCCL, msg);
}

// Wait until the communicator has no call in progress, bounded by the timeout.
int settle(slm_opt_handle* h, ncclResult_t issued, const char* what) {
  if (issued != ncclSuccess && issued != ncclInProgress) return nccl_fail(h, issued, what);
  const auto t0 = Clock::now();
  for (;;) {
    ncclResult_t state = ncclSuccess;
    const ncclResult_t q = ncclCommGetAsyncError(comm_of(h), &state);
    if (q != ncclSuccess) return nccl_fail(h, q, what);
    if (state == ncclSuccess) return SLM_OK;
    if (state != ncclInProgress) return nccl_fail(h, state, what);
    if (elapsed_ms(t0) > h->timeout_ms) {
      abort_comm(h);
      return h->err(SLM_ERR_TIMEOUT, std::string(what) + ": timed out waiting for the other ranks");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(20));
  }
}

ncclDataType_t elem_type(size_t bytes) {
  return bytes == 4 ? ncclFloat32 : (bytes == 8 ? ncclFloat64 : ncclBfloat16);
}

}  // namespace

namespace slmopt {

// Bound of each device-side wait of the peer exchange: the handle's timeout,
// at most 10 s.
uint64_t peer_wait_ms(const slm_opt_handle* h) {
  return h->timeout_ms < 10000u ? h->timeout_ms : 10000u;
}

int zero1_wait(slm_opt_handle* h, cudaStream_t s) {
  const auto t0 = Clock::now();
  // Over peer memory every device wait of a step is bounded (the gradient
  // barrier, the wait for every rank's partials and the weight barrier, each
  // by barrier_timeout_ns), so the host allows for all of them: a missing rank
  // is then reported by the device and the stream has drained when this
  // returns.
  const uint64_t limit_ms =
      h->exchange == SLM_ZERO1_PEER ? uint64_t(h->timeout_ms) + 3ull * peer_wait_ms(h)
                                    : uint64_t(h->timeout_ms);
  for (;;) {
    const cudaError_t e = cudaStreamQuery(s);
    if (e == cudaSuccess) return SLM_OK;
    if (e != cudaErrorNotReady) return h->cuda(e, "step sync");
    if (h->comm) {
      ncclResult_t state = ncclSuccess;
      ncclCommGetAsyncError(comm_of(h), &state);
      if (state != ncclSuccess && state != ncclInProgress)
        return nccl_fail(h, state, "collective failed");
    }
    if (elapsed_ms(t0) > limit_ms) {
      abort_comm(h);
      return h->err(SLM_ERR_TIMEOUT, "the step did not complete within the timeout; a rank "
                                     "stopped participating");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(10));
  }
}

void zero1_release(slm_opt_handle* h) {
  if (h->comm) {
    if (h->broken)
      ncclCommAbort(comm_of(h));
    else
      ncclCommDestroy(comm_of(h));
    h->comm = nullptr;
  }
  for (int q = 0; q < kMaxRanks; ++q)
    for (int b = 0; b < 4; ++b)
      if (h->opened[q][b]) {
        cudaIpcCloseMemHandle(h->opened[q][b]);
        h->opened[q][b] = nullptr;
      }
  cudaFree(h->d_recv);
  cudaFree(h->d_gsum);
  cudaFree(h->d_send);
  cudaFree(h->d_gathered);
  cudaFree(h->d_gradbuf);
  cudaFree(h->d_flags);
  h->d_recv = nullptr;
  h->d_gsum = nullptr;
  h->d_send = nullptr;
  h->d_gathered = nullptr;
  h->d_gradbuf = nullptr;
  h->d_flags = nullptr;
}

int zero1_gather(slm_opt_handle* h, const void* shard_src, size_t elem_bytes, void* dst_full,
                 cudaStream_t s) {
  if (!h->sharded()) return h->err(SLM_ERR_INTERNAL, "gather on a single-replica handle");
  if (h->broken) return h->err(SLM_ERR_TIMEOUT, "the communicator was aborted");
  const uint64_t S = h->shard_stride;
  int st;
  if (dst_full == nullptr) {  // in place on the bf16 weights
    st = settle(h, ncclAllGather(static_cast<const uint16_t*>(shard_src), h->w16, S,
                                 ncclBfloat16, comm_of(h), s),
                "bf16 all-gather");
    if (st) return st;
    return zero1_wait(h, s);
  }
  void* tmp = nullptr;
  if ((st = h->cuda(cudaMalloc(&tmp, uint64_t(h->world) * S * elem_bytes), "gather buffer")))
    return st;
  uint8_t* slot = static_cast<uint8_t*>(tmp) + uint64_t(h->rank) * S * elem_bytes;
  st = h->cuda(cudaMemsetAsync(slot, 0, S * elem_bytes, s), "gather memset");
  if (!st && h->shard_len)
    st = h->cuda(cudaMemcpyAsync(slot, shard_src, h->shard_len * elem_bytes,
                                 cudaMemcpyDeviceToDevice, s),
                 "gather stage");
  if (!st)
    st = settle(h, ncclAllGather(slot, tmp, S, elem_type(elem_bytes), comm_of(h), s),
                "state all-gather");
  if (!st) st = zero1_wait(h, s);
  if (!st)
    st = h->cuda(cudaMemcpy(dst_full, tmp, h->P * elem_bytes, cudaMemcpyDeviceToHost),
                 "gather download");
  cudaFree(tmp);
  return st;
}

// Collective set-up of the peer-memory exchange: every rank exports its
// gradient buffer, gathered-partials area, flag array and bf16 weights with
// CUDA IPC, the 4 x 64-byte handles are all-gathered over NCCL, and each rank
// maps the others'.  The ranks then agree (NCCL min) whether all of them
// succeeded; if any did not, all use the NCCL exchange.
int setup_peer_exchange(slm_opt_handle* h, cudaStream_t s) {
  const int N = h->world;
  h->exchange = SLM_ZERO1_NCCL;
  if (N > kMaxRanks) return SLM_OK;
  int st;
  if ((st = h->cuda(cudaMalloc(&h->d_gradbuf, h->P * 4), "cudaMalloc gradient buffer"))) return st;
  if ((st = h->cuda(cudaMalloc(&h->d_flags, kFlagSlots * kMaxRanks * sizeof(uint32_t)),
                    "cudaMalloc flags")))
    return st;
  if ((st = h->cuda(cudaMemset(h->d_flags, 0, kFlagSlots * kMaxRanks * sizeof(uint32_t)),
                    "memset flags")))
    return st;
  void* mine[4] = {h->d_gradbuf, h->d_gathered, h->d_flags, h->w16};
  std::vector<cudaIpcMemHandle_t> handles(size_t(N) * 4);
  int ok = 1;
  for (int b = 0; b < 4; ++b)
    if (cudaIpcGetMemHandle(&handles[size_t(h->rank) * 4 + b], mine[b]) != cudaSuccess) ok = 0;
  cudaGetLastError();  // a refused export only selects the NCCL exchange
  uint8_t* d_handles = nullptr;
  int32_t* d_ok = nullptr;
  const size_t hbytes = handles.size() * sizeof(cudaIpcMemHandle_t);
  if ((st = h->cuda(cudaMalloc(&d_handles, hbytes), "cudaMalloc handle buffer"))) return st;
  if ((st = h->cuda(cudaMalloc(&d_ok, sizeof(int32_t)), "cudaMalloc agreement"))) {
    cudaFree(d_handles);
    return st;
  }
  const size_t each = 4 * sizeof(cudaIpcMemHandle_t);
  st = h->cuda(cudaMemcpy(d_handles + size_t(h->rank) * each, &handles[size_t(h->rank) * 4], each,
                          cudaMemcpyHostToDevice),
               "stage handles");
  if (!st)
    st = settle(h, ncclAllGather(d_handles + size_t(h->rank) * each, d_handles, each, ncclUint8,
                                 comm_of(h), s),
                "handle all-gather");
  if (!st) st = zero1_wait(h, s);
  if (!st)
    st = h->cuda(cudaMemcpy(handles.data(), d_handles, hbytes, cudaMemcpyDeviceToHost),
                 "fetch handles");
  if (!st && ok) {
    for (int q = 0; q < N && ok; ++q) {
      if (q == h->rank) continue;
      for (int b = 0; b < 4 && ok; ++b) {
        void* ptr = nullptr;
        if (cudaIpcOpenMemHandle(&ptr, handles[size_t(q) * 4 + b],
                                 cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
          cudaGetLastError();
          ok = 0;
        } else {
          h->opened[q][b] = ptr;
        }
      }
    }
  }
  if (!st && ok) {
    // The peer kernels' shared-memory limits; a failure here also selects NCCL.
    h->grid_peer_update = prepare_peer_kernels(h->device, N);
    if (h->grid_peer_update <= 0) {
      cudaGetLastError();
      ok = 0;
    }
  }
  if (!st) {
    const int32_t v = ok;
    st = h->cuda(cudaMemcpy(d_ok, &v, sizeof(v), cudaMemcpyHostToDevice), "stage agreement");
  }
  if (!st)
    st = settle(h, ncclAllReduce(d_ok, d_ok, 1, ncclInt32, ncclMin, comm_of(h), s),
                "agreement all-reduce");
  if (!st) st = zero1_wait(h, s);
  int32_t all_ok = 0;
  if (!st) st = h->cuda(cudaMemcpy(&all_ok, d_ok, sizeof(all_ok), cudaMemcpyDeviceToHost), "agree");
  cudaFree(d_handles);
  cudaFree(d_ok);
  if (st) return st;
  if (all_ok) {
    for (int q = 0; q < N; ++q) {
      void* const* src = q == h->rank ? mine : h->opened[q];
      h->peers.grads[q] = src[0];
      h->peers.gathered[q] = static_cast<double*>(src[1]);
      h->peers.flags[q] = static_cast<uint32_t*>(src[2]);
      h->peers.w16[q] = static_cast<uint16_t*>(src[3]);
    }
    h->exchange = SLM_ZERO1_PEER;
  } else {
    for (int q = 0; q < kMaxRanks; ++q)
      for (int b = 0; b < 4; ++b)
        if (h->opened[q][b]) {
          cudaIpcCloseMemHandle(h->opened[q][b]);
          h->opened[q][b] = nullptr;
        }
  }
  return SLM_OK;
}

namespace {

uint64_t barrier_timeout_ns(const slm_opt_handle* h) { return peer_wait_ms(h) * 1000000ull; }

// One ZeRO-1 step over peer memory, all on stream s: two kernels, the reduce
// (gradient barrier in its prologue) and the update (finalize in its prologue,
// weight barrier in its epilogue).  See slm_opt_zero1_set_exchange.
int peer_step(slm_opt_handle* h, int dtype, const slm_step_config* cfg, cudaStream_t s) {
  const uint32_t epoch = ++h->epoch;
  const uint64_t tmo = barrier_timeout_ns(h);
  const FinalizeParams fp = finalize_params(h, cfg);
  int st;
  if ((st = phase_begin(h, s))) return st;
  if ((st = h->cuda(launch_zero1_peer_reduce(dtype, h->peers, h->rank, h->world, h->shard_begin,
                                             h->shard_len, h->chunks_per_rank, h->d_scaler, fp,
                                             h->d_gsum, epoch, h->d_state, tmo, s),
                    "peer reduce kernel")))
    return st;
  if ((st = phase_mark(h, s))) return st;
  PeerStores ps{};
  for (int q = 0; q < h->world; ++q)
    if (q != h->rank) ps.w16[ps.count++] = h->peers.w16[q] + h->shard_begin;
  const AdamwParams p = adamw_params(cfg);
  if ((st = h->cuda(launch_zero1_peer_update(h->d_gsum, h->shard_len, h->shard_begin, h->master,
                                             h->m1, h->m2, h->w16 + h->shard_begin, h->d_offsets,
                                             h->d_decay, h->d_tile_first, p, h->d_state,
                                             h->d_scaler, h->peers, ps, h->rank, h->world,
                                             h->chunks_per_rank, epoch, fp, tmo,
                                             h->grid_peer_update, s),
                    "peer update kernel")))
    return st;
  return phase_mark(h, s);
}

}  // namespace

int zero1_step(slm_opt_handle* h, const void* grads, int dtype, int memory,
               const slm_step_config* cfg, cudaStream_t s) {
  if (h->broken || !h->comm)
    return h->err(SLM_ERR_TIMEOUT, "the communicator was aborted after a timeout");
  const size_t esize = dtype == SLM_DTYPE_F32 ? 4 : 2;
  const uint64_t S = h->shard_stride;
  const int N = h->world;
  int st;
  if (memory != SLM_MEMORY_HOST && memory != SLM_MEMORY_DEVICE)
    return h->err(SLM_ERR_INVALID_ARGUMENT, "unknown memory kind");
  if (memory == SLM_MEMORY_DEVICE && reinterpret_cast<uintptr_t>(grads) % 16 != 0)
    return h->err(SLM_ERR_INVALID_ARGUMENT, "device gradients must be 16-byte aligned");
  if (h->exchange == SLM_ZERO1_PEER) {
    // The other ranks read this rank's slices from its registered buffer.
    if (grads != h->d_gradbuf) {
      const cudaMemcpyKind kind =
          memory == SLM_MEMORY_HOST ? cudaMemcpyHostToDevice : cudaMemcpyDeviceToDevice;
      if ((st = h->cuda(cudaMemcpyAsync(h->d_gradbuf, grads, h->P * esize, kind, s),
                        "gradient to registered buffer")))
        return st;
    }
    return peer_step(h, dtype, cfg, s);
  }
  // Stage host gradients on the device first.
  const void* dev = grads;
  if (memory == SLM_MEMORY_HOST) {
    const size_t bytes = h->P * esize;
    if (h->staging_bytes < bytes) {
      cudaFree(h->d_staging);
      h->d_staging = nullptr;
      h->staging_bytes = 0;
      if ((st = h->cuda(cudaMalloc(&h->d_staging, bytes), "cudaMalloc gradient staging")))
        return st;
      h->staging_bytes = bytes;
    }
    if ((st = h->cuda(cudaMemcpyAsync(h->d_staging, grads, bytes, cudaMemcpyHostToDevice, s),
                      "gradient upload")))
      return st;
    dev = h->d_staging;
  }
  const size_t need = size_t(N) * S * esize;
  if (h->recv_bytes < need) {
    cudaFree(h->d_recv);
    h->d_recv = nullptr;
    h->recv_bytes = 0;
    if ((st = h->cuda(cudaMalloc(&h->d_recv, need), "cudaMalloc receive buffer"))) return st;
    h->recv_bytes = need;
  }
  const ncclDataType_t type = elem_type(esize);
  if ((st = phase_begin(h, s))) return st;
  // 1. slice q of this rank's gradient goes to rank q; slice r of every rank arrives here.
  ncclGroupStart();
  for (int q = 0; q < N; ++q) {
    const uint64_t begin_q = uint64_t(q) * S;
    const uint64_t len_q = begin_q >= h->P ? 0 : std::min<uint64_t>(S, h->P - begin_q);
    if (len_q)
      ncclSend(static_cast<const uint8_t*>(dev) + begin_q * esize, len_q, type, q, comm_of(h), s);
    if (h->shard_len)
      ncclRecv(static_cast<uint8_t*>(h->d_recv) + uint64_t(q) * S * esize, h->shard_len, type, q,
               comm_of(h), s);
  }
  if ((st = settle(h, ncclGroupEnd(), "gradient all-to-all"))) return st;
  if ((st = phase_mark(h, s))) return st;
  // 2. rank-ordered sum + unscale + partials.
  const FinalizeParams fp = finalize_params(h, cfg);
  if ((st = h->cuda(launch_zero1_reduce(dtype, h->d_recv, uint32_t(N), S, h->shard_len,
                                        h->chunks_per_rank, h->d_scaler, fp, h->d_gsum,
                                        h->d_send, h->d_state, h->grid_norm, s),
                    "zero1 reduce kernel")))
    return st;
  if ((st = phase_mark(h, s))) return st;
  // 3. partials of every rank, 4. identical finalize everywhere.
  if ((st = settle(h, ncclAllGather(h->d_send, h->d_gathered, h->chunks_per_rank + 1,
                                    ncclFloat64, comm_of(h), s),
                   "partials all-gather")))
    return st;
  if ((st = phase_mark(h, s))) return st;
  if ((st = h->cuda(launch_zero1_finalize(h->d_gathered, uint32_t(N), h->chunks_per_rank,
                                          h->d_scaler, h->d_state, fp, s),
                    "zero1 finalize kernel")))
    return st;
  if ((st = phase_mark(h, s))) return st;
  // 5. AdamW on the shard over the raw f32 sums (unscaled inside, as on one GPU).
  const AdamwParams p = adamw_params(cfg);
  if ((st = h->cuda(launch_adamw_update(SLM_DTYPE_F32, h->d_gsum, h->shard_len, h->shard_begin,
                                        h->master, h->m1, h->m2, h->w16 + h->shard_begin,
                                        h->d_offsets, h->d_decay, h->d_tile_first, p, h->d_state,
                                        h->grid_update[0], s),
                    "update kernel")))
    return st;
  if ((st = phase_mark(h, s))) return st;
  // 6. bf16 weights of every shard on every rank.
  if ((st = settle(h, ncclAllGather(h->w16 + uint64_t(h->rank) * S, h->w16, S, ncclBfloat16,
                                    comm_of(h), s),
                   "bf16 all-gather")))
    return st;
  return phase_mark(h, s);
}

}  // namespace slmopt

extern "C" {

int slm_zero1_unique_id(uint8_t out[128]) {
  if (!out) return fail(SLM_ERR_INVALID_ARGUMENT, "out is NULL");
  ncclUniqueId id;
  const ncclResult_t r = ncclGetUniqueId(&id);
  if (r != ncclSuccess) return fail(SLM_ERR_NCCL, std::string("ncclGetUniqueId: ") +
                                                      ncclGetErrorString(r));
  static_assert(sizeof(id.internal) == 128, "NCCL unique id is 128 bytes");
  std::memcpy(out, id.internal, 128);
  return SLM_OK;
}

int slm_opt_create_zero1(const slm_tensor_spec* table, uint32_t n_tensors, int device, int rank,
                         int world, const uint8_t unique_id[128], uint32_t timeout_ms,
                         slm_opt_handle** out) {
  if (!out || !unique_id) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL argument");
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world)
    return fail(SLM_ERR_INVALID_ARGUMENT, "rank must lie in [0, world)");
  if (world == 1) return slm_opt_create(table, n_tensors, device, out);
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
  h->rank = rank;
  h->world = world;
  h->timeout_ms = timeout_ms ? timeout_ms : 300000u;
  const uint64_t chunks = (h->P + kChunkElems - 1) / kChunkElems;
  const uint64_t per_rank = (chunks + world - 1) / world;
  h->chunks_per_rank = uint32_t(per_rank);
  h->shard_stride = per_rank * kChunkElems;
  h->shard_begin = uint64_t(rank) * h->shard_stride;
  h->shard_len = h->shard_begin >= h->P ? 0
                                        : std::min<uint64_t>(h->shard_stride,
                                                             h->P - h->shard_begin);
  DeviceGuard guard(device);
  if (!guard.ok) {
    delete h;
    return fail(SLM_ERR_CUDA, "cudaSetDevice failed");
  }
  if ((st = allocate_state(h, uint64_t(world) * h->shard_stride))) {
    slm_opt_destroy(h);
    return st;
  }
  if ((st = h->cuda(cudaMalloc(&h->d_gsum, std::max<uint64_t>(h->shard_len, 1) * sizeof(float)),
                    "cudaMalloc shard sums")) ||
      (st = h->cuda(cudaMalloc(&h->d_send, (per_rank + 1) * sizeof(double)), "cudaMalloc send")) ||
      (st = h->cuda(cudaMalloc(&h->d_gathered, uint64_t(world) * (per_rank + 1) * sizeof(double)),
                    "cudaMalloc gathered"))) {
    slm_opt_destroy(h);
    return st;
  }
  ncclUniqueId id;
  std::memcpy(id.internal, unique_id, 128);
  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;
  ncclComm_t comm = nullptr;
  const ncclResult_t r = ncclCommInitRankConfig(&comm, world, id, rank, &config);
  h->comm = comm;
  if ((st = settle(h, r, "ncclCommInitRankConfig")) || (st = setup_peer_exchange(h, nullptr))) {
    const std::string msg = h->last_error;
    slm_opt_destroy(h);
    return fail(st, msg);
  }
  *out = h;
  return SLM_OK;
}

int slm_opt_zero1_set_exchange(slm_opt_handle* h, int exchange) {
  if (!h) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL handle");
  if (!h->sharded()) return h->err(SLM_ERR_INVALID_ARGUMENT, "not a ZeRO-1 handle");
  if (exchange == SLM_ZERO1_NCCL) {
    h->exchange = SLM_ZERO1_NCCL;
    return SLM_OK;
  }
  if (exchange == SLM_ZERO1_PEER && h->peers.flags[h->rank] != nullptr) {
    h->exchange = SLM_ZERO1_PEER;
    return SLM_OK;
  }
  return h->err(SLM_ERR_INVALID_ARGUMENT, "the peer-memory exchange is not available");
}

int slm_opt_zero1_exchange(const slm_opt_handle* h) {
  return h && h->sharded() ? h->exchange : -1;
}

int slm_opt_gradient_buffer(slm_opt_handle* h, void** out_device_ptr, uint64_t* bytes) {
  if (!h || !out_device_ptr || !bytes) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL argument");
  if (!h->d_gradbuf)
    return h->err(SLM_ERR_INVALID_ARGUMENT, "this handle has no registered gradient buffer");
  *out_device_ptr = h->d_gradbuf;
  *bytes = h->P * 4;
  return SLM_OK;
}

int slm_opt_shard_range(const slm_opt_handle* h, uint64_t* begin, uint64_t* len) {
  if (!h || !begin || !len) return fail(SLM_ERR_INVALID_ARGUMENT, "NULL argument");
  *begin = h->shard_begin;
  *len = h->shard_len;
  return SLM_OK;
}

}  // extern "C"
