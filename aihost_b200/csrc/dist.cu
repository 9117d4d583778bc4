// dist.cu — KV-head-sharded execution across GPUs behind the C ABI (one process per GPU).
//
// Heads are independent: rank r of N computes KV heads [r*Hkv/N, (r+1)*Hkv/N) and their query
// heads from a local cache that holds only those heads, then one NCCL all-gather over NVLink
// assembles every rank's head outputs, rank-major. The reference splits layers across GPUs and
// stages activations through the host (Inference/MultiGPUTransformer.cs:48-183); this shards
// one layer's attention instead.
//
// NCCL is resolved at run time (dlopen of libnccl.so.2, preferring a copy the process has
// already loaded), so the library loads and runs single-GPU without it. No kernel of this file
// waits on another rank: the only cross-GPU step is the NCCL collective on the caller's stream.
//
// Every NCCL wait is bounded on the host. Communicators are created nonblocking
// (ncclCommInitRankConfig with blocking = 0) and polled with ncclCommGetAsyncError; a set-up
// that does not finish within the limit (a rank that never joins) is aborted with ncclCommAbort
// and reported as AIHOST_ETIMEOUT, so the ranks that did join are not left waiting forever.
// aihost_attn_dist_sync waits the same way for a stream's collectives and aborts the
// communicator when they do not finish. The reference's waits have no bound at all
// (ICompute/Vulkan/VulkanComputeCommandQueue.cs:287 waits on its fence with UInt64.MaxValue).
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <chrono>
#include <mutex>
#include <stdlib.h>
#include <thread>

#include "../../include/aihost_attn.h"
#include "common.cuh"
#include "kernels.h"

namespace aihost {
aihost_status api_fail(aihost_status st, const char* fmt, ...);
int32_t ctx_device(const aihost_attn_ctx* ctx);  // api.cu
}  // namespace aihost

using namespace aihost;

namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank_config)(ncclComm_t*, int, ncclUniqueId, int, ncclConfig_t*) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_abort)(ncclComm_t) = nullptr;
  ncclResult_t (*comm_get_async_error)(ncclComm_t, ncclResult_t*) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static std::once_flag once;
  static NcclApi api;
  std::call_once(once, [] {
    void* h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return;
    api.get_unique_id = reinterpret_cast<decltype(api.get_unique_id)>(dlsym(h, "ncclGetUniqueId"));
    api.comm_init_rank_config = reinterpret_cast<decltype(api.comm_init_rank_config)>(dlsym(h, "ncclCommInitRankConfig"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.comm_abort = reinterpret_cast<decltype(api.comm_abort)>(dlsym(h, "ncclCommAbort"));
    api.comm_get_async_error = reinterpret_cast<decltype(api.comm_get_async_error)>(dlsym(h, "ncclCommGetAsyncError"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank_config && api.comm_destroy && api.comm_abort &&
             api.comm_get_async_error && api.all_gather && api.error_string;
  });
  return api;
}

aihost_status nccl_fail(ncclResult_t r, const char* what) {
  return api_fail(AIHOST_ENCCL, "%s: %s", what, nccl().error_string ? nccl().error_string(r) : "NCCL error");
}

// The limit of aihost_attn_dist_init: AIHOST_NCCL_TIMEOUT_MS from the environment, else 300 s.
int32_t default_timeout_ms() {
  const char* v = getenv("AIHOST_NCCL_TIMEOUT_MS");
  if (v && *v) {
    const long ms = strtol(v, nullptr, 10);
    if (ms > 0 && ms < INT32_MAX) return static_cast<int32_t>(ms);
  }
  return 300000;
}

using Clock = std::chrono::steady_clock;

double elapsed_ms(Clock::time_point t0) {
  return std::chrono::duration<double, std::milli>(Clock::now() - t0).count();
}

int64_t elem_bytes(int32_t dtype) { return dtype == AIHOST_F32 ? 4 : 2; }

}  // namespace

struct aihost_attn_dist {
  int32_t world = 1, rank = 0, device = 0;
  ncclComm_t comm = nullptr;
  bool aborted = false;
};

namespace {

// Aborts the communicator (ends its in-flight collectives and its set-up) and marks `d` unusable.
void abort_comm(aihost_attn_dist* d) {
  if (d->comm) nccl().comm_abort(d->comm);
  d->comm = nullptr;
  d->aborted = true;
}

// Polls a nonblocking communicator until its pending NCCL call has finished (not ncclInProgress),
// at most timeout_ms. On expiry or an asynchronous error the communicator is aborted.
aihost_status wait_comm(aihost_attn_dist* d, int32_t timeout_ms, const char* what) {
  const Clock::time_point t0 = Clock::now();
  for (;;) {
    ncclResult_t st = ncclSuccess;
    const ncclResult_t r = nccl().comm_get_async_error(d->comm, &st);
    if (r != ncclSuccess) {
      abort_comm(d);
      return nccl_fail(r, "ncclCommGetAsyncError");
    }
    if (st == ncclSuccess) return AIHOST_OK;
    if (st != ncclInProgress) {
      abort_comm(d);
      return nccl_fail(st, what);
    }
    const double ms = elapsed_ms(t0);
    if (ms > timeout_ms) {
      abort_comm(d);
      return api_fail(AIHOST_ETIMEOUT, "%s did not finish within %d ms (a rank missing?); communicator aborted", what,
                      timeout_ms);
    }
    // a collective's enqueue normally finishes within microseconds: spin (yielding) for the first
    // 2 ms so the stream gets its work at once, then poll every 100 us (set-up, a slow peer)
    if (ms < 2.0) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
}

}  // namespace

extern "C" {

aihost_status aihost_attn_dist_unique_id(void* out_id) {
  if (!out_id) return api_fail(AIHOST_EINVAL, "out_id is NULL");
  const NcclApi& api = nccl();
  if (!api.ok) return api_fail(AIHOST_EUNSUPPORTED, "libnccl.so.2 could not be loaded");
  ncclUniqueId id;
  const ncclResult_t r = api.get_unique_id(&id);
  if (r != ncclSuccess) return nccl_fail(r, "ncclGetUniqueId");
  memcpy(out_id, id.internal, NCCL_UNIQUE_ID_BYTES);
  return AIHOST_OK;
}

aihost_status aihost_attn_dist_init_bounded(int32_t world, int32_t rank, const void* nccl_id, int32_t device,
                                            int32_t timeout_ms, aihost_attn_dist** out) {
  if (!out || !nccl_id) return api_fail(AIHOST_EINVAL, "out and nccl_id must be non-NULL");
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world)
    return api_fail(AIHOST_EINVAL, "rank %d outside a world of %d", rank, world);
  if (timeout_ms < 1) return api_fail(AIHOST_EINVAL, "timeout_ms (%d) must be >= 1", timeout_ms);
  const NcclApi& api = nccl();
  if (!api.ok) return api_fail(AIHOST_EUNSUPPORTED, "libnccl.so.2 could not be loaded");
  int prev = 0;
  cudaGetDevice(&prev);
  cudaError_t e = cudaSetDevice(device);
  if (e != cudaSuccess) return api_fail(AIHOST_ECUDA, "cudaSetDevice(%d): %s", device, cudaGetErrorString(e));
  ncclUniqueId id;
  memcpy(id.internal, nccl_id, NCCL_UNIQUE_ID_BYTES);
  auto* d = new aihost_attn_dist();
  d->world = world;
  d->rank = rank;
  d->device = device;
  ncclConfig_t config = NCCL_CONFIG_INITIALIZER;
  config.blocking = 0;  // set-up runs in the background; polled below with a limit
  const ncclResult_t r = api.comm_init_rank_config(&d->comm, world, id, rank, &config);
  aihost_status s = AIHOST_OK;
  if (r != ncclSuccess && r != ncclInProgress) {
    if (d->comm) api.comm_abort(d->comm);
    s = nccl_fail(r, "ncclCommInitRankConfig");
  } else {
    s = wait_comm(d, timeout_ms, "ncclCommInitRankConfig");
  }
  cudaSetDevice(prev);
  if (s != AIHOST_OK) {
    delete d;
    return s;
  }
  *out = d;
  return AIHOST_OK;
}

aihost_status aihost_attn_dist_init(int32_t world, int32_t rank, const void* nccl_id, int32_t device,
                                    aihost_attn_dist** out) {
  return aihost_attn_dist_init_bounded(world, rank, nccl_id, device, default_timeout_ms(), out);
}

aihost_status aihost_attn_dist_destroy(aihost_attn_dist* d) {
  if (!d) return AIHOST_OK;
  if (d->comm && nccl().ok) nccl().comm_destroy(d->comm);
  delete d;
  return AIHOST_OK;
}

aihost_status aihost_attn_dist_sync(aihost_attn_dist* d, void* stream, int32_t timeout_ms) {
  if (!d) return api_fail(AIHOST_EINVAL, "dist is NULL");
  if (timeout_ms < 1) return api_fail(AIHOST_EINVAL, "timeout_ms (%d) must be >= 1", timeout_ms);
  if (d->aborted) return api_fail(AIHOST_ENCCL, "the communicator was aborted after an earlier failure");
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(d->device);
  const Clock::time_point t0 = Clock::now();
  aihost_status s = AIHOST_OK;
  for (;;) {
    const cudaError_t q = cudaStreamQuery(static_cast<cudaStream_t>(stream));
    if (q == cudaSuccess) break;
    if (q != cudaErrorNotReady) {
      s = api_fail(AIHOST_ECUDA, "cudaStreamQuery: %s", cudaGetErrorString(q));
      break;
    }
    ncclResult_t st = ncclSuccess;
    if (d->comm && d->world > 1) {
      nccl().comm_get_async_error(d->comm, &st);
      if (st != ncclSuccess && st != ncclInProgress) {
        abort_comm(d);
        s = nccl_fail(st, "collective");
        break;
      }
    }
    const double ms = elapsed_ms(t0);
    if (ms > timeout_ms) {
      if (d->world > 1) abort_comm(d);
      s = api_fail(AIHOST_ETIMEOUT, "the stream's work did not finish within %d ms%s", timeout_ms,
                   d->world > 1 ? "; communicator aborted" : "");
      break;
    }
    if (ms < 2.0) std::this_thread::yield();
    else std::this_thread::sleep_for(std::chrono::microseconds(100));
  }
  cudaSetDevice(prev);
  return s;
}

aihost_status aihost_attn_forward_sharded(aihost_attn_dist* dist, aihost_attn_ctx* ctx, const aihost_attn_desc* local,
                                          int32_t batch, int32_t n_new, const void* q, const void* k_new,
                                          const void* v_new, void* k_cache, void* v_cache, const int32_t* seq_len,
                                          const int32_t* h_seq_len, void* out_gathered, void* stream) {
  if (!dist || !ctx || !local || !out_gathered)
    return api_fail(AIHOST_EINVAL, "dist, ctx, desc and out_gathered must be non-NULL");
  if (dist->aborted) return api_fail(AIHOST_ENCCL, "the communicator was aborted after an earlier failure");
  if (ctx_device(ctx) != dist->device)
    return api_fail(AIHOST_EINVAL, "the context is on device %d and the communicator on device %d", ctx_device(ctx),
                    dist->device);
  if (local->out_dtype != AIHOST_F32 && local->out_dtype != AIHOST_F16)
    return api_fail(AIHOST_EINVAL, "out_dtype %d must be F32 (0) or F16 (1)", local->out_dtype);
  const int64_t chunk_bytes = static_cast<int64_t>(batch) * n_new * local->n_q_heads * local->head_dim *
                              elem_bytes(local->out_dtype);
  uint8_t* mine = static_cast<uint8_t*>(out_gathered) + dist->rank * chunk_bytes;
  aihost_status s = aihost_attn_forward(ctx, local, batch, n_new, q, k_new, v_new, k_cache, v_cache, seq_len,
                                        h_seq_len, mine, stream);
  if (s != AIHOST_OK) return s;
  if (dist->world == 1) return AIHOST_OK;
  int prev = 0;
  cudaGetDevice(&prev);
  cudaSetDevice(dist->device);
  // in place: every rank's slot of the rank-major buffer is its send buffer
  const ncclResult_t r =
      nccl().all_gather(mine, out_gathered, static_cast<size_t>(chunk_bytes), ncclUint8, dist->comm,
                        static_cast<cudaStream_t>(stream));
  // a nonblocking communicator may still be enqueuing: bounded poll until the call is issued
  if (r == ncclInProgress) s = wait_comm(dist, default_timeout_ms(), "ncclAllGather");
  else if (r != ncclSuccess) s = nccl_fail(r, "ncclAllGather");
  cudaSetDevice(prev);
  return s;
}

}  // extern "C"
