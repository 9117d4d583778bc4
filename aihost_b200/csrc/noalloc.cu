// noalloc.cu — decode entry point that allocates no device memory.
//
// Some hosts of this library cannot call cudaMalloc at the point where they decode. Examples:
// an engine whose device memory is fully carved up by its own pool before inference starts; a
// sandboxed or driver-level host whose allocator lock must not be taken on the token path; code
// running while another component holds the GPU's allocation budget. aihost_attn_forward needs
// a context (one cudaMalloc for its status word) and split scratch sized by
// aihost_attn_reserve (another cudaMalloc). aihost_attn_decode_noalloc does the same
// decode step (RoPE, KV append, split-K attention, split merge) with the split scratch and the
// merge counters in
// g_noalloc_scratch below: a fixed array that the CUDA runtime places in every device's
// memory when the library's module is loaded, and that stays there until the process exits.
//
// Limits and rules of use:
//   - scratch = batch * n_q_heads * max_splits * (head_dim + 2) * 4 bytes must fit in
//     kNoAllocScratchBytes (8 MiB); larger requests are refused with AIHOST_ENOMEM before
//     anything is enqueued;
//   - the first call on each device looks up the array's device address
//     (cudaGetSymbolAddress, which loads the module there); make that first call before any
//     stream capture;
//   - all calls share the one array: calls whose kernels overlap on the GPU (different streams,
//     different host threads) race on it. Serialise them, e.g. one stream per device;
//   - the array keeps the last call's contents. Two fields must start at zero: the device
//     status word and the split-merge arrival counters, both zero when the module loads. The
//     status word then collects the error bits of every call (a device-side length past
//     kv_capacity, a bounded wait that ran out) until aihost_attn_noalloc_sync_status reads and
//     clears it, so an error is never lost to a later call. The counters are tagged with a
//     per-device call epoch, so stale counts of earlier calls are never mistaken for this call's.
#include <string.h>

#include <mutex>

#include "../../include/aihost_attn.h"
#include "common.cuh"
#include "kernels.h"

namespace aihost {
// Defined in api.cu: the thread-local error message of aihost_attn_last_error(), and the
// validation / split plan / RoPE table shared with aihost_attn_forward (none allocates).
aihost_status api_fail(aihost_status st, const char* fmt, ...);
aihost_status noalloc_prepare(const aihost_attn_desc* desc, int32_t batch, KvLayout* kv, float* scale,
                              int32_t* chunk, int32_t* max_splits, RopeFreqs* freqs, int32_t num_sms);
size_t noalloc_need_bytes(const aihost_attn_desc* desc, int32_t batch, int32_t num_sms, size_t have, bool* use_sk);

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(8) << 20;
constexpr size_t kStatusBytes = 256;  // status word, kept at the front
constexpr size_t kCounterBytes = kMaxSplitCounters * sizeof(unsigned long long);  // then the counters
constexpr int kMaxDevices = 64;

__device__ __align__(256) uint8_t g_noalloc_scratch[kStatusBytes + kCounterBytes + kNoAllocScratchBytes];

std::mutex g_mu;
void* g_dev_addr[kMaxDevices] = {};
uint32_t g_epoch[kMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once per device).
aihost_status scratch_address(int dev, uint8_t** out) {
  std::lock_guard<std::mutex> lk(g_mu);
  if (!g_dev_addr[dev]) {
    void* p = nullptr;
    cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess)
      return api_fail(AIHOST_ECUDA, "cudaGetSymbolAddress(g_noalloc_scratch) on device %d: %s", dev,
                   cudaGetErrorString(e));
    g_dev_addr[dev] = p;
  }
  *out = static_cast<uint8_t*>(g_dev_addr[dev]);
  return AIHOST_OK;
}

uint32_t next_epoch(int dev) {
  std::lock_guard<std::mutex> lk(g_mu);
  return g_epoch[dev]++;
}

}  // namespace

}  // namespace aihost

using namespace aihost;

extern "C" aihost_status aihost_attn_decode_noalloc(const aihost_attn_desc* desc, int32_t batch, const void* q,
                                                    const void* k_new, const void* v_new, void* k_cache,
                                                    void* v_cache, const int32_t* seq_len, const int32_t* h_seq_len,
                                                    void* out, void* stream) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return api_fail(AIHOST_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return api_fail(AIHOST_EUNSUPPORTED, "device index %d >= %d", dev, kMaxDevices);
  int sms = 0;
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess || sms < 1)
    return api_fail(AIHOST_ECUDA, "cudaDeviceGetAttribute(multiprocessor count) on device %d: %s", dev,
                    cudaGetErrorString(e));
  KvLayout kv;
  float scale;
  int32_t chunk, max_splits;
  RopeFreqs freqs;
  aihost_status s = noalloc_prepare(desc, batch, &kv, &scale, &chunk, &max_splits, &freqs, sms);
  if (s != AIHOST_OK) return s;
  // the size check depends on the description alone and comes before the pointer checks
  bool use_sk = false;
  const size_t need = noalloc_need_bytes(desc, batch, sms, kNoAllocScratchBytes, &use_sk);
  if (need > kNoAllocScratchBytes)
    return api_fail(AIHOST_ENOMEM,
                 "aihost_attn_decode_noalloc: this call needs %zu bytes of split scratch; the static array holds "
                 "%zu (8 MiB). Use aihost_attn_forward with a reserved context for larger batches or contexts",
                 need, kNoAllocScratchBytes);
  if (!q || !k_new || !v_new || !k_cache || !v_cache || !seq_len || !out)
    return api_fail(AIHOST_EINVAL, "q, k_new, v_new, k_cache, v_cache, seq_len and out must be non-NULL");
  for (const void* p : {q, k_new, v_new, static_cast<const void*>(k_cache), static_cast<const void*>(v_cache),
                        static_cast<const void*>(out)})
    if (reinterpret_cast<uintptr_t>(p) % 16)
      return api_fail(AIHOST_EINVAL, "tensor pointers must be 16-byte aligned");
  if (h_seq_len)
    for (int32_t b = 0; b < batch; ++b)
      if (h_seq_len[b] < 0 || static_cast<int64_t>(h_seq_len[b]) + 1 > desc->kv_capacity)
        return api_fail(AIHOST_EINVAL, "sequence %d: %d cached rows + 1 exceed kv_capacity %d", b, h_seq_len[b],
                     desc->kv_capacity);
  uint8_t* base = nullptr;
  s = scratch_address(dev, &base);
  if (s != AIHOST_OK) return s;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  // sticky: kernels only set bits; aihost_attn_noalloc_sync_status reads and clears them
  int32_t* status = reinterpret_cast<int32_t*>(base);

  DecodeArgs a;
  memset(&a, 0, sizeof(a));
  a.q = q;
  a.q_dtype = desc->q_dtype;
  a.k_cache = k_cache;
  a.v_cache = v_cache;
  a.kv = kv;
  a.seq_len = seq_len;
  a.len_offset = 1;
  a.batch = batch;
  a.n_q_heads = desc->n_q_heads;
  a.n_kv_heads = desc->n_kv_heads;
  a.head_dim = desc->head_dim;
  a.scale = scale;
  a.rope_mode = desc->rope_mode;
  a.freqs = freqs;
  a.chunk = chunk;
  a.max_splits = max_splits;
  float* part = reinterpret_cast<float*>(base + kStatusBytes + kCounterBytes);
  a.part_o = part;
  a.part_ml = part + static_cast<size_t>(batch) * desc->n_q_heads * max_splits * desc->head_dim;
  a.out = out;
  a.out_dtype = desc->out_dtype;
  a.status = status;
  a.k_new = k_new;  // appended by the decode kernel itself, or by the append kernel first
  a.v_new = v_new;
  a.new_dtype = desc->q_dtype;
  a.counters = reinterpret_cast<unsigned long long*>(base + kStatusBytes);
  a.epoch = next_epoch(dev);
  a.stream_k = use_sk ? 1 : 0;
  a.num_sms = sms;
  e = launch_decode_any(a, st, nullptr);
  if (e != cudaSuccess) return api_fail(AIHOST_ECUDA, "decode launch: %s", cudaGetErrorString(e));
  return AIHOST_OK;
}

extern "C" aihost_status aihost_attn_noalloc_sync_status(void* stream, int32_t* out_bits) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return api_fail(AIHOST_ECUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (dev < 0 || dev >= kMaxDevices) return api_fail(AIHOST_EUNSUPPORTED, "device index %d >= %d", dev, kMaxDevices);
  uint8_t* base = nullptr;
  aihost_status s = scratch_address(dev, &base);
  if (s != AIHOST_OK) return s;
  e = cudaStreamSynchronize(static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return api_fail(AIHOST_ECUDA, "cudaStreamSynchronize: %s", cudaGetErrorString(e));
  // a host int and the device word: plain synchronous copies, no allocation on either side
  int32_t bits = 0;
  const int32_t zero = 0;
  e = cudaMemcpy(&bits, base, sizeof(bits), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemcpy(base, &zero, sizeof(zero), cudaMemcpyHostToDevice);
  if (e != cudaSuccess) return api_fail(AIHOST_ECUDA, "reading the no-alloc status word: %s", cudaGetErrorString(e));
  if (out_bits) *out_bits = bits;
  if (bits & kStatusWaitTimeout)
    return api_fail(AIHOST_ETIMEOUT, "a no-alloc decode kernel's bounded wait expired (status 0x%x)", bits);
  if (bits & kStatusBadLength)
    return api_fail(AIHOST_EINVAL, "a no-alloc decode call got a device-side sequence length past kv_capacity");
  return AIHOST_OK;
}
