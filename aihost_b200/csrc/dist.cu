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
#include <dlfcn.h>
#include <nccl.h>
#include <string.h>

#include <mutex>

#include "../../include/aihost_attn.h"
#include "common.cuh"
#include "kernels.h"

namespace aihost {
aihost_status api_fail(aihost_status st, const char* fmt, ...);
}  // namespace aihost

using namespace aihost;

namespace {

struct NcclApi {
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
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
    api.comm_init_rank = reinterpret_cast<decltype(api.comm_init_rank)>(dlsym(h, "ncclCommInitRank"));
    api.comm_destroy = reinterpret_cast<decltype(api.comm_destroy)>(dlsym(h, "ncclCommDestroy"));
    api.all_gather = reinterpret_cast<decltype(api.all_gather)>(dlsym(h, "ncclAllGather"));
    api.error_string = reinterpret_cast<decltype(api.error_string)>(dlsym(h, "ncclGetErrorString"));
    api.ok = api.get_unique_id && api.comm_init_rank && api.comm_destroy && api.all_gather && api.error_string;
  });
  return api;
}

aihost_status nccl_fail(ncclResult_t r, const char* what) {
  return api_fail(AIHOST_ENCCL, "%s: %s", what, nccl().error_string ? nccl().error_string(r) : "NCCL error");
}

int64_t elem_bytes(int32_t dtype) { return dtype == AIHOST_F32 ? 4 : 2; }

}  // namespace

struct aihost_attn_dist {
  int32_t world = 1, rank = 0, device = 0;
  ncclComm_t comm = nullptr;
};

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

aihost_status aihost_attn_dist_init(int32_t world, int32_t rank, const void* nccl_id, int32_t device,
                                    aihost_attn_dist** out) {
  if (!out || !nccl_id) return api_fail(AIHOST_EINVAL, "out and nccl_id must be non-NULL");
  *out = nullptr;
  if (world < 1 || rank < 0 || rank >= world)
    return api_fail(AIHOST_EINVAL, "rank %d outside a world of %d", rank, world);
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
  const ncclResult_t r = api.comm_init_rank(&d->comm, world, id, rank);
  cudaSetDevice(prev);
  if (r != ncclSuccess) {
    delete d;
    return nccl_fail(r, "ncclCommInitRank");
  }
  *out = d;
  return AIHOST_OK;
}

aihost_status aihost_attn_dist_destroy(aihost_attn_dist* d) {
  if (!d) return AIHOST_OK;
  if (d->comm && nccl().ok) nccl().comm_destroy(d->comm);
  delete d;
  return AIHOST_OK;
}

aihost_status aihost_attn_forward_sharded(aihost_attn_dist* dist, aihost_attn_ctx* ctx, const aihost_attn_desc* local,
                                          int32_t batch, int32_t n_new, const void* q, const void* k_new,
                                          const void* v_new, void* k_cache, void* v_cache, const int32_t* seq_len,
                                          const int32_t* h_seq_len, void* out_gathered, void* stream) {
  if (!dist || !local || !out_gathered) return api_fail(AIHOST_EINVAL, "dist, desc and out_gathered must be non-NULL");
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
  cudaSetDevice(prev);
  if (r != ncclSuccess) return nccl_fail(r, "ncclAllGather");
  return AIHOST_OK;
}

}  // extern "C"
