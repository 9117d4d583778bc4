// api.cu — the extern "C" boundary of libaihost_attn.so (declared in include/aihost_attn.h).
//
// Host-side work only: argument validation (each failure gets its own message and status, the
// way ICompute/CUDA/CudaApi.cs:CheckError turns error codes into exceptions on the C# side),
// the RoPE frequency table, cache-geometry resolution, TMA descriptor encoding and the choice
// of split size for decode. No allocation happens outside create / reserve.
#include <math.h>
#include <stdarg.h>
#include <stdio.h>
#include <string.h>

#include <algorithm>
#include <mutex>
#include <utility>
#include <vector>

#include "../../include/aihost_attn.h"
#include "common.cuh"
#include "kernels.h"

using namespace aihost;

// Per-kernel-kind device-time accumulator (events recorded around each launch while enabled).
struct ProfSlot {
  std::vector<std::pair<cudaEvent_t, cudaEvent_t>> pending;
  int64_t launches = 0;
  double total_ms = 0.0;
};

struct aihost_attn_ctx {
  int32_t device = 0;
  int32_t num_sms = 148;
  int32_t* d_status = nullptr;
  void* scratch = nullptr;
  size_t scratch_bytes = 0;
  unsigned long long* counters = nullptr;  // fused split merge: epoch-tagged arrival counts
  uint32_t epoch = 0;
  bool profiling = false;
  std::mutex prof_mu;
  ProfSlot prof[AIHOST_KERNEL_COUNT];
  std::vector<cudaEvent_t> event_pool;
};

namespace {
thread_local char g_err[512] = "";
}  // namespace

namespace aihost {
// Records the thread-local message returned by aihost_attn_last_error().
aihost_status api_fail(aihost_status st, const char* fmt, ...) {
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(g_err, sizeof(g_err), fmt, ap);
  va_end(ap);
  return st;
}
}  // namespace aihost

namespace {

#define fail api_fail

aihost_status cuda_fail(cudaError_t e, const char* what) {
  return fail(AIHOST_ECUDA, "%s: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
}

// Runs `f` with the context's device current and restores the caller's device afterwards.
class DeviceGuard {
 public:
  explicit DeviceGuard(int32_t dev) {
    ok_ = cudaGetDevice(&prev_) == cudaSuccess;
    if (ok_ && prev_ != dev) ok_ = cudaSetDevice(dev) == cudaSuccess;
  }
  ~DeviceGuard() {
    int cur = -1;
    if (cudaGetDevice(&cur) == cudaSuccess && cur != prev_) cudaSetDevice(prev_);
  }
  bool ok() const { return ok_; }

 private:
  int prev_ = 0;
  bool ok_ = false;
};

int64_t row_bytes(int32_t dtype, int32_t head_dim) {
  if (dtype == AIHOST_F32) return 4LL * head_dim;
  if (dtype == AIHOST_F16) return 2LL * head_dim;
  return 34LL * (head_dim / 32);
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// Validates the static description; fills the resolved cache layout and scale.
aihost_status check_desc(const aihost_attn_desc* d, KvLayout* kv, float* scale) {
  memset(kv, 0, sizeof(*kv));  // contiguous layout: no block table
  if (!d) return fail(AIHOST_EINVAL, "desc is NULL");
  if (d->n_q_heads < 1 || d->n_kv_heads < 1)
    return fail(AIHOST_EINVAL, "n_q_heads (%d) and n_kv_heads (%d) must be >= 1", d->n_q_heads, d->n_kv_heads);
  if (d->n_q_heads % d->n_kv_heads)
    return fail(AIHOST_EINVAL, "n_q_heads (%d) must be a multiple of n_kv_heads (%d)", d->n_q_heads, d->n_kv_heads);
  if (d->head_dim != 64 && d->head_dim != 128)
    return fail(AIHOST_EUNSUPPORTED, "head_dim %d is not supported (64 or 128)", d->head_dim);
  if (d->q_dtype != AIHOST_F32 && d->q_dtype != AIHOST_F16)
    return fail(AIHOST_EINVAL, "q_dtype %d must be F32 (0) or F16 (1)", d->q_dtype);
  if (d->out_dtype != AIHOST_F32 && d->out_dtype != AIHOST_F16)
    return fail(AIHOST_EINVAL, "out_dtype %d must be F32 (0) or F16 (1)", d->out_dtype);
  if (d->kv_dtype != AIHOST_F32 && d->kv_dtype != AIHOST_F16 && d->kv_dtype != AIHOST_Q8_0)
    return fail(AIHOST_EINVAL, "kv_dtype %d must be F32 (0), F16 (1) or Q8_0 (6)", d->kv_dtype);
  if (d->rope_mode < AIHOST_ROPE_INTERLEAVED || d->rope_mode > AIHOST_ROPE_NONE)
    return fail(AIHOST_EINVAL, "rope_mode %d is not a valid aihost_rope_mode", d->rope_mode);
  if (d->rope_mode != AIHOST_ROPE_NONE && !(d->rope_theta > 0.0f && isfinite(d->rope_theta)))
    return fail(AIHOST_EINVAL, "rope_theta must be a positive finite number");
  if (d->kv_capacity < 1) return fail(AIHOST_EINVAL, "kv_capacity must be >= 1");
  if (!(isfinite(d->scale) && d->scale >= 0.0f)) return fail(AIHOST_EINVAL, "scale must be >= 0 and finite");
  const int64_t rb = row_bytes(d->kv_dtype, d->head_dim);
  kv->head_stride = d->kv_head_stride ? d->kv_head_stride : rb;
  kv->token_stride = d->kv_token_stride ? d->kv_token_stride : kv->head_stride * d->n_kv_heads;
  kv->seq_stride = d->kv_seq_stride ? d->kv_seq_stride : kv->token_stride * d->kv_capacity;
  kv->capacity = d->kv_capacity;
  kv->dtype = d->kv_dtype;
  if (kv->head_stride < rb || kv->token_stride < rb || kv->seq_stride < 0)
    return fail(AIHOST_EINVAL, "kv strides smaller than one head row (%lld bytes)", static_cast<long long>(rb));
  const int64_t need_align = d->kv_dtype == AIHOST_Q8_0 ? 2 : 16;
  if (kv->head_stride % need_align || kv->token_stride % need_align || kv->seq_stride % need_align)
    return fail(AIHOST_EINVAL, "kv strides must be multiples of %lld bytes", static_cast<long long>(need_align));
  *scale = d->scale != 0.0f ? d->scale : 1.0f / sqrtf(static_cast<float>(d->head_dim));
  return AIHOST_OK;
}

RopeFreqs make_freqs(float theta, int32_t head_dim) {
  RopeFreqs f;
  memset(&f, 0, sizeof(f));
  for (int i = 0; i < head_dim / 2 && i < kMaxHeadDim / 2; ++i)
    f.f[i] = 1.0f / powf(theta, static_cast<float>(2 * i) / static_cast<float>(head_dim));
  return f;
}

// Decode split plan: rows per split chosen from the capacity (so the scratch size is a
// function of the description alone).
//  - fp16 / Q8_0 caches (tensor-core kernels, 2 CTAs per SM, one CTA per <= 16 query heads):
//    splits of at most 4096 rows, evenly sized, and enough of them for two CTAs per SM. Long
//    splits amortise each CTA's fixed work (Q rotation, pipeline fill, the four-warp merge).
//  - fp32 caches (CUDA-core kernel): ~8 resident CTAs per SM, 64..512 rows per split.
struct DecodePlan {
  int32_t chunk, max_splits;
};
DecodePlan plan_decode(const aihost_attn_desc* d, int32_t batch, int32_t num_sms) {
  const int32_t G = d->n_q_heads / d->n_kv_heads;
  DecodePlan p;
  if (d->kv_dtype == AIHOST_F16 || d->kv_dtype == AIHOST_Q8_0) {
    const int64_t units = static_cast<int64_t>(batch) * d->n_kv_heads * ((G + 15) / 16);
    const int64_t cap = d->kv_capacity;
    int64_t splits = (cap + 4095) / 4096;
    const int64_t fill = (2LL * num_sms + units - 1) / units;
    if (splits < fill) splits = fill;
    int64_t chunk = (cap + splits - 1) / splits;
    chunk = (chunk + 63) / 64 * 64;
    p.chunk = static_cast<int32_t>(chunk);
    p.max_splits = static_cast<int32_t>((cap + chunk - 1) / chunk);
    return p;
  }
  const int32_t gt = G >= 8 ? 8 : G >= 4 ? 4 : G >= 2 ? 2 : 1;
  const int64_t units = static_cast<int64_t>(batch) * d->n_kv_heads * ((G + gt - 1) / gt);
  const int64_t target = static_cast<int64_t>(num_sms) * 8;
  int64_t chunk = (static_cast<int64_t>(d->kv_capacity) * units + target - 1) / target;
  chunk = (chunk + 31) / 32 * 32;
  if (chunk < 64) chunk = 64;
  if (chunk > 512) chunk = 512;
  p.chunk = static_cast<int32_t>(chunk);
  p.max_splits = static_cast<int32_t>((d->kv_capacity + chunk - 1) / chunk);
  return p;
}

// The stream-K schedule of the Q8_0 decode (see decode_q8s_kernel) applies to head groups of
// up to 8 query heads and at most kQ8StreamKMaxUnits sequences.
bool q8_stream_k_eligible(const aihost_attn_desc* d, int32_t batch) {
  return d->kv_dtype == AIHOST_Q8_0 && d->n_q_heads / d->n_kv_heads <= 8 && batch <= kQ8StreamKMaxUnits &&
         d->n_kv_heads <= 64 && batch * static_cast<int64_t>(d->n_kv_heads) <= kMaxSplitCounters;
}

// Decode scratch of the split plan, and of the stream-K schedule where it applies (the larger
// of the two); *use_sk tells whether `have` bytes allow the stream-K schedule.
size_t decode_need_bytes(const aihost_attn_desc* d, int32_t batch, int32_t num_sms, size_t have = SIZE_MAX,
                         bool* use_sk = nullptr) {
  const DecodePlan p = plan_decode(d, batch, num_sms);
  const size_t split = decode_scratch_bytes(batch, d->n_q_heads, d->head_dim, p.max_splits);
  const size_t sk = q8_stream_k_eligible(d, batch) ? std::max(split, q8_stream_k_bytes(d->head_dim, num_sms)) : 0;
  const bool sk_ok = sk != 0 && sk <= have;
  if (use_sk) *use_sk = sk_ok;
  return sk_ok || have == SIZE_MAX ? std::max(split, sk) : split;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn get_encode_fn() {
  static std::once_flag once;
  static EncodeTiledFn fn = nullptr;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(p);
  });
  return fn;
}

// fp16 tensor [d3][d2][d1][d0 = head_dim] with byte strides s1, s2, s3; box {64, 1, box_rows, 1},
// 128-byte swizzle (the canonical tcgen05 K-major / MN-major operand layout).
aihost_status encode_f16_map(CUtensorMap* map, const void* base, int32_t d0, int64_t d1, int64_t d2, int64_t d3,
                             int64_t s1, int64_t s2, int64_t s3, const char* what, uint32_t box_rows = 128) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(AIHOST_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (!aligned(base, 16)) return fail(AIHOST_EINVAL, "%s must be 16-byte aligned", what);
  if (s1 % 16 || s2 % 16 || s3 % 16) return fail(AIHOST_EINVAL, "%s strides must be multiples of 16 bytes", what);
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(d0), static_cast<cuuint64_t>(d1), static_cast<cuuint64_t>(d2),
                        static_cast<cuuint64_t>(d3)};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(s1), static_cast<cuuint64_t>(s2), static_cast<cuuint64_t>(s3)};
  cuuint32_t box[4] = {64, 1, box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AIHOST_ECUDA, "cuTensorMapEncodeTiled(%s) failed with %d", what, static_cast<int>(r));
  return AIHOST_OK;
}

// Q8_0 cache viewed as 32-bit words: dims {words per token row, capacity, batch, 1}, box
// {box_words, 64 rows, 1, 1}, no swizzle. Needs 16-byte token/sequence strides and 4-byte heads.
aihost_status encode_q8_map(CUtensorMap* map, const void* base, const KvLayout& kv, int32_t batch,
                            uint32_t box_words) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(AIHOST_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  // a paged cache is one pool "sequence" of n_pages * page_rows rows
  const int64_t rows = kv.block_table ? static_cast<int64_t>(kv.n_pages) * kv.page_rows : kv.capacity;
  if (kv.block_table) batch = 1;
  const int64_t seq_stride =
      kv.block_table ? kv.token_stride * rows : (kv.seq_stride ? kv.seq_stride : kv.token_stride * kv.capacity);
  if (!aligned(base, 16) || kv.token_stride % 16 || seq_stride % 16 || kv.head_stride % 4)
    return fail(AIHOST_EINVAL, "Q8_0 cache strides are not TMA-compatible");
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(kv.token_stride / 4), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(batch), 1};
  cuuint64_t strides[3] = {static_cast<cuuint64_t>(kv.token_stride), static_cast<cuuint64_t>(seq_stride),
                           static_cast<cuuint64_t>(seq_stride) * static_cast<cuuint64_t>(batch)};
  cuuint32_t box[4] = {box_words, 64, 1, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 4, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AIHOST_ECUDA, "cuTensorMapEncodeTiled(q8 cache) failed with %d", static_cast<int>(r));
  return AIHOST_OK;
}

aihost_status check_ctx(aihost_attn_ctx* ctx) {
  if (!ctx) return fail(AIHOST_EINVAL, "ctx is NULL");
  return AIHOST_OK;
}

cudaEvent_t take_event(aihost_attn_ctx* ctx) {
  if (!ctx->event_pool.empty()) {
    cudaEvent_t e = ctx->event_pool.back();
    ctx->event_pool.pop_back();
    return e;
  }
  cudaEvent_t e = nullptr;
  if (cudaEventCreate(&e) != cudaSuccess) return nullptr;
  return e;
}

// Launch through `fn`, bracketed by timing events on `st` when the profiler is on.
template <class F>
cudaError_t timed_launch(aihost_attn_ctx* ctx, int kind, cudaStream_t st, F&& fn) {
  if (!ctx->profiling) return fn();
  std::lock_guard<std::mutex> lk(ctx->prof_mu);
  cudaEvent_t a = take_event(ctx), b = take_event(ctx);
  if (!a || !b) return cudaErrorMemoryAllocation;
  cudaError_t e = cudaEventRecord(a, st);
  if (e != cudaSuccess) return e;
  e = fn();
  if (e != cudaSuccess) return e;
  e = cudaEventRecord(b, st);
  if (e != cudaSuccess) return e;
  ctx->prof[kind].pending.emplace_back(a, b);
  return cudaSuccess;
}

// One-token attention over rows [0, start + len_offset). With k_new / v_new (forward decode) the
// new rows are appended at row seq_len[b] first (inside the decode kernel where it can).
aihost_status run_decode(aihost_attn_ctx* ctx, const aihost_attn_desc* d, const KvLayout& kv, float scale,
                         int32_t batch, const void* q, const void* kc, const void* vc, const int32_t* seq_len,
                         int32_t start_scalar, int32_t len_offset, int32_t rope_mode, void* out, cudaStream_t st,
                         const void* k_new = nullptr, const void* v_new = nullptr, const int32_t* q_pos = nullptr,
                         float* lse = nullptr) {
  DecodePlan plan = plan_decode(d, batch, ctx->num_sms);
  bool use_sk = false;
  const size_t need = decode_need_bytes(d, batch, ctx->num_sms, ctx->scratch_bytes, &use_sk);
  if (need > ctx->scratch_bytes)
    return fail(AIHOST_ENOMEM, "decode needs %zu bytes of scratch, context has %zu (call aihost_attn_reserve)", need,
                ctx->scratch_bytes);
  DecodeArgs a;
  memset(&a, 0, sizeof(a));
  a.q = q;
  a.q_dtype = d->q_dtype;
  a.k_cache = kc;
  a.v_cache = vc;
  a.kv = kv;
  a.seq_len = seq_len;
  a.start_scalar = start_scalar;
  a.len_offset = len_offset;
  a.rope_pos_offset = 0;
  a.batch = batch;
  a.n_q_heads = d->n_q_heads;
  a.n_kv_heads = d->n_kv_heads;
  a.head_dim = d->head_dim;
  a.scale = scale;
  a.rope_mode = rope_mode;
  if (rope_mode != AIHOST_ROPE_NONE) a.freqs = make_freqs(d->rope_theta, d->head_dim);
  a.chunk = plan.chunk;
  a.max_splits = plan.max_splits;
  float* scratch = static_cast<float*>(ctx->scratch);
  a.part_o = scratch;
  a.part_ml = scratch ? scratch + static_cast<size_t>(batch) * d->n_q_heads * plan.max_splits * d->head_dim : nullptr;
  a.out = out;
  a.out_dtype = d->out_dtype;
  a.status = ctx->d_status;
  a.k_new = k_new;
  a.v_new = v_new;
  a.new_dtype = d->q_dtype;
  a.q_pos = q_pos;
  a.lse = lse;
  a.stream_k = use_sk ? 1 : 0;
  a.num_sms = ctx->num_sms;
  cudaError_t e = launch_decode_any(a, st, ctx);
  if (e != cudaSuccess) return cuda_fail(e, "decode launch");
  return AIHOST_OK;
}

size_t round256(size_t x) { return (x + 255) / 256 * 256; }

// Scratch for the fp16 copies the prefill kernel reads when q is fp32 or the cache is fp32 /
// Q8_0 (zero for fp16 operands): q [batch][n_q][Hq][d], K and V [batch][kv_rows][Hkv][d].
size_t prefill_stage_bytes(const aihost_attn_desc* d, int32_t batch, int32_t n_q, int32_t kv_rows) {
  size_t bytes = 0;
  if (d->q_dtype != AIHOST_F16)
    bytes += round256(static_cast<size_t>(batch) * n_q * d->n_q_heads * d->head_dim * 2);
  if (d->kv_dtype != AIHOST_F16)
    bytes += 2 * round256(static_cast<size_t>(batch) * kv_rows * d->n_kv_heads * d->head_dim * 2);
  return bytes;
}

// Prefill of n_q query rows per sequence over cache rows [0, start_b + len_offset), where
// start_b = seq_len[b] (or start_scalar) and at most kv_rows rows are attended by any sequence.
// fp32 q and fp32 / Q8_0 caches are first converted to fp16 in the context's scratch (q rotated
// in fp32 on the way), then the same tensor-core kernel runs on the copies.
aihost_status run_prefill(aihost_attn_ctx* ctx, const aihost_attn_desc* d, const KvLayout& kv_in, float scale,
                          int32_t batch, int32_t n_q, const void* q, const void* kc, const void* vc,
                          const int32_t* seq_len, int32_t start_scalar, int32_t len_offset, int32_t kv_rows,
                          int32_t rope_mode, void* out, cudaStream_t st, bool after_append) {
  if (!prefill_supported(d->head_dim)) return fail(AIHOST_EUNSUPPORTED, "prefill head_dim %d", d->head_dim);
  KvLayout kv = kv_in;
  const bool q_staged = d->q_dtype != AIHOST_F16, kv_staged = d->kv_dtype != AIHOST_F16;
  if (q_staged || kv_staged) {
    const size_t need = prefill_stage_bytes(d, batch, n_q, kv_rows);
    if (need > ctx->scratch_bytes)
      return fail(AIHOST_ENOMEM,
                  "prefill with fp32 / Q8_0 operands needs %zu bytes of scratch, context has %zu "
                  "(call aihost_attn_reserve with aihost_attn_workspace_size)",
                  need, ctx->scratch_bytes);
    uint8_t* sp = static_cast<uint8_t*>(ctx->scratch);
    if (d->q_dtype != AIHOST_F16) {
      __half* qh = reinterpret_cast<__half*>(sp);
      sp += round256(static_cast<size_t>(batch) * n_q * d->n_q_heads * d->head_dim * 2);
      const RopeFreqs fr = make_freqs(rope_mode != AIHOST_ROPE_NONE ? d->rope_theta : 1.0f, d->head_dim);
      cudaError_t e = timed_launch(ctx, AIHOST_KERNEL_CONVERT, st, [&] {
        return launch_stage_q(static_cast<const float*>(q), qh, seq_len, start_scalar, batch, n_q, d->n_q_heads,
                              d->head_dim, rope_mode, fr, st);
      });
      if (e != cudaSuccess) return cuda_fail(e, "q staging launch");
      q = qh;
      rope_mode = AIHOST_ROPE_NONE;
    }
    if (d->kv_dtype != AIHOST_F16) {
      const size_t part = round256(static_cast<size_t>(batch) * kv_rows * d->n_kv_heads * d->head_dim * 2);
      __half* kh = reinterpret_cast<__half*>(sp);
      __half* vh = reinterpret_cast<__half*>(sp + part);
      cudaError_t e = timed_launch(ctx, AIHOST_KERNEL_CONVERT, st, [&] {
        return launch_stage_kv(kc, vc, kv, kh, vh, kv_rows, seq_len, start_scalar, len_offset, batch, d->n_kv_heads,
                               d->head_dim, st);
      });
      if (e != cudaSuccess) return cuda_fail(e, "cache staging launch");
      kc = kh;
      vc = vh;
      kv.head_stride = 2LL * d->head_dim;
      kv.token_stride = kv.head_stride * d->n_kv_heads;
      kv.seq_stride = kv.token_stride * kv_rows;
      kv.capacity = kv_rows;
      kv.dtype = AIHOST_F16;
      kv.block_table = nullptr;  // the staged copies are dense per sequence, whatever the cache was
    }
  }
  PrefillArgs a;
  memset(&a, 0, sizeof(a));
  const int64_t D = d->head_dim, Hq = d->n_q_heads;
  aihost_status s = encode_f16_map(&a.q_map, q, d->head_dim, Hq, n_q, batch, D * 2, Hq * D * 2,
                                   static_cast<int64_t>(n_q) * Hq * D * 2, "q");
  if (s != AIHOST_OK) return s;
  // a paged cache is one pool "sequence" of n_pages * page_rows rows; otherwise one per sequence
  const int64_t map_rows = kv.block_table ? static_cast<int64_t>(kv.n_pages) * kv.page_rows : kv.capacity;
  const int64_t map_seqs = kv.block_table ? 1 : batch;
  const int64_t map_seq_stride =
      kv.block_table ? kv.token_stride * map_rows : (kv.seq_stride ? kv.seq_stride : kv.token_stride * kv.capacity);
  s = encode_f16_map(&a.k_map, kc, d->head_dim, d->n_kv_heads, map_rows, map_seqs, kv.head_stride, kv.token_stride,
                     map_seq_stride, "k_cache");
  if (s != AIHOST_OK) return s;
  s = encode_f16_map(&a.v_map, vc, d->head_dim, d->n_kv_heads, map_rows, map_seqs, kv.head_stride, kv.token_stride,
                     map_seq_stride, "v_cache");
  if (s != AIHOST_OK) return s;
  a.block_table = kv.block_table;
  a.max_pages = kv.max_pages;
  a.page_rows = kv.page_rows;
  a.q = q;
  a.seq_len = seq_len;
  a.start_scalar = start_scalar;
  a.len_offset = len_offset;
  a.batch = batch;
  a.n_new = n_q;
  a.n_q_heads = d->n_q_heads;
  a.n_kv_heads = d->n_kv_heads;
  a.head_dim = d->head_dim;
  a.scale = scale;
  a.rope_mode = rope_mode;
  if (rope_mode != AIHOST_ROPE_NONE) a.freqs = make_freqs(d->rope_theta, d->head_dim);
  a.out = out;
  a.out_dtype = d->out_dtype;
  a.status = ctx->d_status;
  a.split_kv = prefill_split_kv(batch, n_q, d->n_q_heads, ctx->num_sms) ? 1 : 0;
  // The kernel launched just before the prefill: staging of the cache (q, if staged, was
  // written one launch earlier), else staging of q, else (forward) the append, which leaves q
  // alone, else (mha) the caller's own work, which may have produced q.
  a.q_early = kv_staged || (!q_staged && after_append) ? 1 : 0;
  cudaError_t e = timed_launch(ctx, AIHOST_KERNEL_PREFILL, st, [&] { return launch_prefill(a, st); });
  if (e != cudaSuccess) return cuda_fail(e, "prefill launch");
  return AIHOST_OK;
}

}  // namespace

namespace aihost {
cudaError_t launch_decode_any(DecodeArgs a, cudaStream_t st, aihost_attn_ctx* ctx) {
  auto run = [&](int kind, auto&& fn) -> cudaError_t { return ctx ? timed_launch(ctx, kind, st, fn) : fn(); };
  // Tensor-core path: TMA maps over the cache (fp16 tiles, or Q8_0 rows as 32-bit words).
  DecodeMmaArgs m;
  memset(&m, 0, sizeof(m));
  bool mma = false;
  char saved[sizeof(g_err)];
  memcpy(saved, g_err, sizeof(g_err));
  if (a.kv.dtype == AIHOST_F16) {
    // a paged cache is one pool "sequence" of n_pages * page_rows rows; otherwise one per sequence
    const int64_t rows = a.kv.block_table ? static_cast<int64_t>(a.kv.n_pages) * a.kv.page_rows : a.kv.capacity;
    const int64_t seqs = a.kv.block_table ? 1 : a.batch;
    const int64_t seq_stride = a.kv.block_table ? a.kv.token_stride * rows
                                                : (a.kv.seq_stride ? a.kv.seq_stride : a.kv.token_stride * a.kv.capacity);
    mma = encode_f16_map(&m.k_map, a.k_cache, a.head_dim, a.n_kv_heads, rows, seqs, a.kv.head_stride,
                         a.kv.token_stride, seq_stride, "k_cache", 64) == AIHOST_OK &&
          encode_f16_map(&m.v_map, a.v_cache, a.head_dim, a.n_kv_heads, rows, seqs, a.kv.head_stride,
                         a.kv.token_stride, seq_stride, "v_cache", 64) == AIHOST_OK;
  } else if (a.kv.dtype == AIHOST_Q8_0) {
    const uint32_t bw = q8_box_words(a.head_dim, a.kv.head_stride);
    mma = bw && encode_q8_map(&m.k_map, a.k_cache, a.kv, a.batch, bw) == AIHOST_OK &&
          encode_q8_map(&m.v_map, a.v_cache, a.kv, a.batch, bw) == AIHOST_OK;
  }
  if (!mma) memcpy(g_err, saved, sizeof(g_err));  // strides TMA cannot describe: CUDA-core kernel instead
  // One CTA per <= 16 query heads: with a single head group per KV head, the CTA of the last
  // split appends the new rows itself and the last split to finish merges the partials.
  // The CUDA-core kernel (fp32 caches, strides TMA cannot describe) fuses the append for fp32
  // caches (its shared copy of the new row is then exactly the stored row) and the merge for
  // any layout, with up to batch * n_q_heads counters (one per head group).
  const int32_t G = a.n_q_heads / a.n_kv_heads;
  const bool one_group = G <= 16;
  const int64_t n_counters = mma ? static_cast<int64_t>(a.batch) * a.n_kv_heads
                                 : static_cast<int64_t>(a.batch) * a.n_q_heads;
  a.fuse_append = a.k_new && ((mma && one_group) || (!mma && a.kv.dtype == AIHOST_F32)) ? 1 : 0;
  if (ctx) {
    a.counters = ctx->counters;
    a.epoch = ctx->epoch++;
  }
  if (!((mma ? one_group : true) && n_counters <= kMaxSplitCounters)) a.counters = nullptr;
  if (!mma || !a.counters) a.stream_k = 0;  // the stream-K schedule needs the tensor maps and counters
  cudaError_t e = cudaSuccess;
  if (a.k_new && !a.fuse_append) {
    e = run(AIHOST_KERNEL_APPEND, [&] {
      return launch_kv_append(a.k_new, a.v_new, a.new_dtype, const_cast<void*>(a.k_cache), const_cast<void*>(a.v_cache),
                              a.kv, a.seq_len, a.batch, 1, a.n_kv_heads, a.head_dim, a.rope_mode, a.freqs, a.status,
                              st, a.q_pos);
    });
    if (e != cudaSuccess) return e;
  }
  if (mma) {
    m.base = a;
    e = run(AIHOST_KERNEL_DECODE, [&] { return launch_decode_mma(m, st); });
  } else {
    e = run(AIHOST_KERNEL_DECODE, [&] { return launch_decode(a, st); });
  }
  if (e != cudaSuccess || a.max_splits <= 1 || a.counters) return e;
  return run(AIHOST_KERNEL_COMBINE, [&] { return launch_decode_combine(a, st); });
}

int32_t ctx_device(const aihost_attn_ctx* ctx) { return ctx ? ctx->device : -1; }

size_t noalloc_need_bytes(const aihost_attn_desc* desc, int32_t batch, int32_t num_sms, size_t have, bool* use_sk) {
  return decode_need_bytes(desc, batch, num_sms, have, use_sk);
}

// Validation, split plan and RoPE table of a one-token decode, for aihost_attn_decode_noalloc.
aihost_status noalloc_prepare(const aihost_attn_desc* desc, int32_t batch, KvLayout* kv, float* scale,
                              int32_t* chunk, int32_t* max_splits, RopeFreqs* freqs, int32_t num_sms) {
  aihost_status s = check_desc(desc, kv, scale);
  if (s != AIHOST_OK) return s;
  if (batch < 1) return fail(AIHOST_EINVAL, "batch (%d) must be >= 1", batch);
  const DecodePlan p = plan_decode(desc, batch, num_sms);
  *chunk = p.chunk;
  *max_splits = p.max_splits;
  *freqs = make_freqs(desc->rope_mode != AIHOST_ROPE_NONE ? desc->rope_theta : 1.0f, desc->head_dim);
  return AIHOST_OK;
}
}  // namespace aihost

extern "C" {

int32_t aihost_attn_abi_version(void) { return AIHOST_ATTN_ABI_VERSION; }

const char* aihost_attn_last_error(void) { return g_err; }

aihost_status aihost_attn_create(int32_t device, aihost_attn_ctx** out_ctx) {
  if (!out_ctx) return fail(AIHOST_EINVAL, "out_ctx is NULL");
  *out_ctx = nullptr;
  int n = 0;
  cudaError_t e = cudaGetDeviceCount(&n);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceCount");
  if (device < 0 || device >= n) return fail(AIHOST_EINVAL, "device %d out of range (%d devices)", device, n);
  DeviceGuard g(device);
  if (!g.ok()) return fail(AIHOST_ECUDA, "cudaSetDevice(%d) failed", device);
  cudaDeviceProp prop;
  e = cudaGetDeviceProperties(&prop, device);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDeviceProperties");
  if (prop.major != 10) return fail(AIHOST_EUNSUPPORTED, "device %d is sm_%d%d; this build targets sm_100a", device,
                                    prop.major, prop.minor);
  auto* ctx = new aihost_attn_ctx();
  ctx->device = device;
  ctx->num_sms = prop.multiProcessorCount;
  e = cudaMalloc(&ctx->d_status, sizeof(int32_t));
  if (e != cudaSuccess) {
    delete ctx;
    return cuda_fail(e, "cudaMalloc(status)");
  }
  e = cudaMemset(ctx->d_status, 0, sizeof(int32_t));
  if (e == cudaSuccess) e = cudaMalloc(&ctx->counters, kMaxSplitCounters * sizeof(unsigned long long));
  if (e == cudaSuccess) e = cudaMemset(ctx->counters, 0, kMaxSplitCounters * sizeof(unsigned long long));
  if (e != cudaSuccess) {
    cudaFree(ctx->counters);
    cudaFree(ctx->d_status);
    delete ctx;
    return cuda_fail(e, "context setup");
  }
  *out_ctx = ctx;
  return AIHOST_OK;
}

aihost_status aihost_attn_destroy(aihost_attn_ctx* ctx) {
  if (!ctx) return AIHOST_OK;
  DeviceGuard g(ctx->device);
  for (auto& slot : ctx->prof)
    for (auto& pr : slot.pending) {
      cudaEventDestroy(pr.first);
      cudaEventDestroy(pr.second);
    }
  for (cudaEvent_t e : ctx->event_pool) cudaEventDestroy(e);
  cudaFree(ctx->scratch);
  cudaFree(ctx->counters);
  cudaFree(ctx->d_status);
  delete ctx;
  return AIHOST_OK;
}

aihost_status aihost_attn_workspace_size(const aihost_attn_desc* desc, int32_t batch, int32_t n_new,
                                         size_t* out_bytes) {
  if (!out_bytes) return fail(AIHOST_EINVAL, "out_bytes is NULL");
  KvLayout kv;
  float scale;
  aihost_status s = check_desc(desc, &kv, &scale);
  if (s != AIHOST_OK) return s;
  if (batch < 1 || n_new < 1) return fail(AIHOST_EINVAL, "batch (%d) and n_new (%d) must be >= 1", batch, n_new);
  *out_bytes = prefill_stage_bytes(desc, batch, n_new, desc->kv_capacity);
  if (n_new == 1) {
    int sms = 148;
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    *out_bytes = decode_need_bytes(desc, batch, sms);
  }
  return AIHOST_OK;
}

aihost_status aihost_attn_reserve(aihost_attn_ctx* ctx, size_t bytes) {
  aihost_status s = check_ctx(ctx);
  if (s != AIHOST_OK) return s;
  if (bytes <= ctx->scratch_bytes) return AIHOST_OK;
  DeviceGuard g(ctx->device);
  if (ctx->scratch) {
    cudaError_t e = cudaDeviceSynchronize();
    if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize before scratch resize");
    cudaFree(ctx->scratch);
    ctx->scratch = nullptr;
    ctx->scratch_bytes = 0;
  }
  cudaError_t e = cudaMalloc(&ctx->scratch, bytes);
  if (e != cudaSuccess) {
    ctx->scratch = nullptr;
    return fail(AIHOST_ENOMEM, "cudaMalloc(%zu) for scratch failed: %s", bytes, cudaGetErrorString(e));
  }
  ctx->scratch_bytes = bytes;
  return AIHOST_OK;
}

// The fused op over a contiguous cache (paging NULL) or a paged fp16 pool (paging carries the
// block table and page geometry; validated by the caller).
static aihost_status forward_common(aihost_attn_ctx* ctx, const aihost_attn_desc* desc, const KvLayout* paging,
                                    int32_t batch, int32_t n_new, const void* q, const void* k_new, const void* v_new,
                                    void* k_cache, void* v_cache, const int32_t* seq_len, const int32_t* h_seq_len,
                                    void* out, void* stream) {
  aihost_status s = check_ctx(ctx);
  if (s != AIHOST_OK) return s;
  KvLayout kv;
  float scale;
  s = check_desc(desc, &kv, &scale);
  if (s != AIHOST_OK) return s;
  if (paging) {
    kv.block_table = paging->block_table;
    kv.max_pages = paging->max_pages;
    kv.page_rows = paging->page_rows;
    kv.n_pages = paging->n_pages;
    kv.seq_stride = 0;
    // the pools must be describable by the tensor maps the kernels read them through
    const int64_t rows = static_cast<int64_t>(kv.n_pages) * kv.page_rows;
    CUtensorMap probe;
    if (kv.dtype == AIHOST_F32) {
      // read row by row by the CUDA-core decode kernel and the prefill staging: no tensor map
    } else if (kv.dtype == AIHOST_F16) {
      s = encode_f16_map(&probe, k_cache, desc->head_dim, desc->n_kv_heads, rows, 1, kv.head_stride, kv.token_stride,
                         kv.token_stride * rows, "k_pool", 64);
      if (s == AIHOST_OK)
        s = encode_f16_map(&probe, v_cache, desc->head_dim, desc->n_kv_heads, rows, 1, kv.head_stride,
                           kv.token_stride, kv.token_stride * rows, "v_pool", 64);
    } else {
      const uint32_t bw = q8_box_words(desc->head_dim, kv.head_stride);
      s = bw ? encode_q8_map(&probe, k_cache, kv, 1, bw) : fail(AIHOST_EINVAL, "Q8_0 head stride is not TMA-compatible");
      if (s == AIHOST_OK) s = encode_q8_map(&probe, v_cache, kv, 1, bw);
    }
    if (s != AIHOST_OK) return s;
  }
  if (batch < 1 || n_new < 1) return fail(AIHOST_EINVAL, "batch (%d) and n_new (%d) must be >= 1", batch, n_new);
  if (!q || !k_new || !v_new || !k_cache || !v_cache || !seq_len || !out)
    return fail(AIHOST_EINVAL, "q, k_new, v_new, k_cache, v_cache, seq_len and out must be non-NULL");
  if (!aligned(q, 16) || !aligned(k_new, 16) || !aligned(v_new, 16) || !aligned(out, 16) || !aligned(k_cache, 16) ||
      !aligned(v_cache, 16) || !aligned(seq_len, 4))
    return fail(AIHOST_EINVAL, "tensor pointers must be 16-byte aligned");
  if (n_new > desc->kv_capacity) return fail(AIHOST_EINVAL, "n_new %d exceeds kv_capacity %d", n_new, desc->kv_capacity);
  if (h_seq_len)
    for (int32_t b = 0; b < batch; ++b)
      if (h_seq_len[b] < 0 || static_cast<int64_t>(h_seq_len[b]) + n_new > desc->kv_capacity)
        return fail(AIHOST_EINVAL, "sequence %d: %d cached + %d new rows exceed kv_capacity %d", b, h_seq_len[b],
                    n_new, desc->kv_capacity);
  DeviceGuard g(ctx->device);
  if (!g.ok()) return fail(AIHOST_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n_new == 1)  // append + attention (the append fused into the decode kernel where it can be)
    return run_decode(ctx, desc, kv, scale, batch, q, k_cache, v_cache, seq_len, 0, 1, desc->rope_mode, out, st,
                      k_new, v_new);
  const RopeFreqs freqs = make_freqs(desc->rope_mode != AIHOST_ROPE_NONE ? desc->rope_theta : 1.0f, desc->head_dim);
  cudaError_t e = timed_launch(ctx, AIHOST_KERNEL_APPEND, st, [&] {
    return launch_kv_append(k_new, v_new, desc->q_dtype, k_cache, v_cache, kv, seq_len, batch, n_new,
                            desc->n_kv_heads, desc->head_dim, desc->rope_mode, freqs, ctx->d_status, st);
  });
  if (e != cudaSuccess) return cuda_fail(e, "kv append launch");
  int32_t kv_rows = desc->kv_capacity;
  if (h_seq_len) {
    kv_rows = 0;
    for (int32_t b = 0; b < batch; ++b) kv_rows = h_seq_len[b] + n_new > kv_rows ? h_seq_len[b] + n_new : kv_rows;
  }
  return run_prefill(ctx, desc, kv, scale, batch, n_new, q, k_cache, v_cache, seq_len, 0, n_new, kv_rows,
                     desc->rope_mode, out, st, true);
}

aihost_status aihost_attn_forward(aihost_attn_ctx* ctx, const aihost_attn_desc* desc, int32_t batch,
                                  int32_t n_new, const void* q, const void* k_new, const void* v_new,
                                  void* k_cache, void* v_cache, const int32_t* seq_len,
                                  const int32_t* h_seq_len, void* out, void* stream) {
  return forward_common(ctx, desc, nullptr, batch, n_new, q, k_new, v_new, k_cache, v_cache, seq_len, h_seq_len, out,
                        stream);
}

aihost_status aihost_attn_forward_paged(aihost_attn_ctx* ctx, const aihost_attn_desc* desc, int32_t batch,
                                        int32_t n_new, const void* q, const void* k_new, const void* v_new,
                                        void* k_pool, void* v_pool, int32_t n_pages, int32_t page_rows,
                                        const int32_t* block_table, int32_t max_pages, const int32_t* seq_len,
                                        const int32_t* h_seq_len, void* out, void* stream) {
  if (!desc) return fail(AIHOST_EINVAL, "desc is NULL");
  if (desc->kv_dtype != AIHOST_F16 && desc->kv_dtype != AIHOST_Q8_0 && desc->kv_dtype != AIHOST_F32)
    return fail(AIHOST_EUNSUPPORTED, "kv_dtype %d cannot be paged", desc->kv_dtype);
  if (page_rows < 128 || page_rows % 128) return fail(AIHOST_EINVAL, "page_rows %d must be a positive multiple of 128",
                                                      page_rows);
  if (n_pages < 1 || max_pages < 1) return fail(AIHOST_EINVAL, "n_pages (%d) and max_pages (%d) must be >= 1", n_pages,
                                                max_pages);
  if (static_cast<int64_t>(n_pages) * page_rows > INT32_MAX)
    return fail(AIHOST_EINVAL, "the pool (%d pages of %d rows) exceeds 2^31 rows", n_pages, page_rows);
  if (desc->kv_capacity > static_cast<int64_t>(max_pages) * page_rows)
    return fail(AIHOST_EINVAL, "kv_capacity %d exceeds max_pages * page_rows = %lld", desc->kv_capacity,
                static_cast<long long>(max_pages) * page_rows);
  if (!block_table || !aligned(block_table, 4)) return fail(AIHOST_EINVAL, "block_table must be a non-NULL int32 array");
  KvLayout paging;
  memset(&paging, 0, sizeof(paging));
  paging.block_table = block_table;
  paging.max_pages = max_pages;
  paging.page_rows = page_rows;
  paging.n_pages = n_pages;
  return forward_common(ctx, desc, &paging, batch, n_new, q, k_new, v_new, k_pool, v_pool, seq_len, h_seq_len, out,
                        stream);
}

aihost_status aihost_attn_mha(aihost_attn_ctx* ctx, const aihost_attn_desc* desc, int32_t n_q, int32_t n_kv,
                              int32_t start_pos, const void* q, const void* k, const void* v, void* out,
                              void* stream) {
  aihost_status s = check_ctx(ctx);
  if (s != AIHOST_OK) return s;
  KvLayout kv;
  float scale;
  s = check_desc(desc, &kv, &scale);
  if (s != AIHOST_OK) return s;
  if (n_q < 1 || n_kv < 1) return fail(AIHOST_EINVAL, "n_q (%d) and n_kv (%d) must be >= 1", n_q, n_kv);
  if (n_kv > desc->kv_capacity) return fail(AIHOST_EINVAL, "n_kv %d exceeds kv_capacity %d", n_kv, desc->kv_capacity);
  if (start_pos < 0 || (n_q > 1 && start_pos >= n_kv))
    return fail(AIHOST_EINVAL, "start_pos %d outside [0, n_kv=%d)", start_pos, n_kv);
  if (!q || !k || !v || !out) return fail(AIHOST_EINVAL, "q, k, v and out must be non-NULL");
  if (!aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) || !aligned(out, 16))
    return fail(AIHOST_EINVAL, "tensor pointers must be 16-byte aligned");
  DeviceGuard g(ctx->device);
  if (!g.ok()) return fail(AIHOST_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (n_q == 1)  // FusedMHAGenerate: every row visible, no mask
    return run_decode(ctx, desc, kv, scale, 1, q, k, v, nullptr, 0, n_kv, AIHOST_ROPE_NONE, out, st);
  return run_prefill(ctx, desc, kv, scale, 1, n_q, q, k, v, nullptr, start_pos, n_kv - start_pos, n_kv,
                     AIHOST_ROPE_NONE, out, st, false);
}

aihost_status aihost_attn_decode_partial(aihost_attn_ctx* ctx, const aihost_attn_desc* desc, int32_t batch,
                                         const void* q, const void* k_new, const void* v_new, void* k_cache,
                                         void* v_cache, const int32_t* seq_len, const int32_t* q_pos, void* out,
                                         float* lse, void* stream) {
  aihost_status s = check_ctx(ctx);
  if (s != AIHOST_OK) return s;
  KvLayout kv;
  float scale;
  s = check_desc(desc, &kv, &scale);
  if (s != AIHOST_OK) return s;
  if (batch < 1) return fail(AIHOST_EINVAL, "batch (%d) must be >= 1", batch);
  if (!q || !k_cache || !v_cache || !seq_len || !out)
    return fail(AIHOST_EINVAL, "q, k_cache, v_cache, seq_len and out must be non-NULL");
  if (!k_new != !v_new) return fail(AIHOST_EINVAL, "k_new and v_new must both be given or both be NULL");
  if (k_new && !q_pos) return fail(AIHOST_EINVAL, "appending k_new needs q_pos (the new rows' global positions)");
  if (!aligned(q, 16) || !aligned(out, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16) ||
      !aligned(k_new, 16) || !aligned(v_new, 16) || !aligned(seq_len, 4) || !aligned(q_pos, 4) || !aligned(lse, 4))
    return fail(AIHOST_EINVAL, "tensor pointers must be 16-byte aligned (seq_len, q_pos and lse 4-byte)");
  DeviceGuard g(ctx->device);
  if (!g.ok()) return fail(AIHOST_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
  const int32_t rope = q_pos ? desc->rope_mode : AIHOST_ROPE_NONE;
  return run_decode(ctx, desc, kv, scale, batch, q, k_cache, v_cache, seq_len, 0, k_new ? 1 : 0, rope, out,
                    static_cast<cudaStream_t>(stream), k_new, v_new, q_pos, lse);
}

aihost_status aihost_attn_merge_partials(aihost_attn_ctx* ctx, int32_t n_parts, int32_t rows, int32_t head_dim,
                                         int32_t dtype, const void* o_parts, const float* lse_parts, void* out,
                                         float* lse_out, void* stream) {
  aihost_status s = check_ctx(ctx);
  if (s != AIHOST_OK) return s;
  if (n_parts < 1 || rows < 1) return fail(AIHOST_EINVAL, "n_parts (%d) and rows (%d) must be >= 1", n_parts, rows);
  if (head_dim < 1 || head_dim > kMaxHeadDim)
    return fail(AIHOST_EINVAL, "head_dim %d outside [1, %d]", head_dim, kMaxHeadDim);
  if (dtype != AIHOST_F32 && dtype != AIHOST_F16) return fail(AIHOST_EINVAL, "dtype must be F32 or F16");
  if (!o_parts || !lse_parts || !out) return fail(AIHOST_EINVAL, "o_parts, lse_parts and out must be non-NULL");
  DeviceGuard g(ctx->device);
  if (!g.ok()) return fail(AIHOST_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = timed_launch(ctx, AIHOST_KERNEL_COMBINE, st, [&] {
    return launch_merge_partials(n_parts, rows, head_dim, dtype, o_parts, lse_parts, out, lse_out, st);
  });
  if (e != cudaSuccess) return cuda_fail(e, "merge launch");
  return AIHOST_OK;
}

aihost_status aihost_rope_full(void* x, int32_t dtype, int32_t seq, int32_t n_heads, int32_t head_dim,
                               int32_t start_pos, float theta, int32_t rope_mode, void* stream) {
  if (!x) return fail(AIHOST_EINVAL, "x is NULL");
  if (dtype != AIHOST_F32 && dtype != AIHOST_F16) return fail(AIHOST_EINVAL, "dtype %d must be F32 or F16", dtype);
  if (seq < 0 || n_heads < 1 || head_dim < 2 || head_dim % 2 || head_dim > kMaxHeadDim)
    return fail(AIHOST_EINVAL, "bad shape seq=%d n_heads=%d head_dim=%d", seq, n_heads, head_dim);
  if (start_pos < 0) return fail(AIHOST_EINVAL, "start_pos must be >= 0");
  if (rope_mode == AIHOST_ROPE_NONE) return AIHOST_OK;
  if (rope_mode != AIHOST_ROPE_INTERLEAVED && rope_mode != AIHOST_ROPE_NEOX)
    return fail(AIHOST_EINVAL, "rope_mode %d is not a valid aihost_rope_mode", rope_mode);
  if (!(theta > 0.0f && isfinite(theta))) return fail(AIHOST_EINVAL, "theta must be a positive finite number");
  cudaError_t e = launch_rope_full(x, dtype, seq, n_heads, head_dim, start_pos, rope_mode, make_freqs(theta, head_dim),
                                   static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "rope launch");
  return AIHOST_OK;
}

aihost_status aihost_qk_norm_rope(void* x, int32_t dtype, int32_t seq, int32_t n_heads, int32_t head_dim,
                                  const float* weight, float eps, int32_t start_pos, float theta, int32_t rope_mode,
                                  void* stream) {
  if (!x || !weight) return fail(AIHOST_EINVAL, "x and weight must be non-NULL");
  if (dtype != AIHOST_F32 && dtype != AIHOST_F16) return fail(AIHOST_EINVAL, "dtype %d must be F32 or F16", dtype);
  if (seq < 0 || n_heads < 1 || head_dim < 2 || head_dim % 2 || head_dim > kMaxHeadDim)
    return fail(AIHOST_EINVAL, "bad shape seq=%d n_heads=%d head_dim=%d", seq, n_heads, head_dim);
  if (!aligned(x, dtype == AIHOST_F32 ? 4 : 2) || !aligned(weight, 4))
    return fail(AIHOST_EINVAL, "x and weight must be aligned to their element size");
  if (start_pos < 0) return fail(AIHOST_EINVAL, "start_pos must be >= 0");
  if (!(eps >= 0.0f && isfinite(eps))) return fail(AIHOST_EINVAL, "eps must be a non-negative finite number");
  if (rope_mode != AIHOST_ROPE_INTERLEAVED && rope_mode != AIHOST_ROPE_NEOX && rope_mode != AIHOST_ROPE_NONE)
    return fail(AIHOST_EINVAL, "rope_mode %d is not a valid aihost_rope_mode", rope_mode);
  if (rope_mode != AIHOST_ROPE_NONE && !(theta > 0.0f && isfinite(theta)))
    return fail(AIHOST_EINVAL, "theta must be a positive finite number");
  const RopeFreqs freqs = make_freqs(rope_mode != AIHOST_ROPE_NONE ? theta : 1.0f, head_dim);
  cudaError_t e = launch_qk_norm_rope(x, dtype, seq, n_heads, head_dim, weight, eps, start_pos, rope_mode, freqs,
                                      static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "qk norm + rope launch");
  return AIHOST_OK;
}

aihost_status aihost_kv_append(aihost_attn_ctx* ctx, const aihost_attn_desc* desc, int32_t batch, int32_t n_new,
                               const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                               const int32_t* seq_len, void* stream) {
  aihost_status s = check_ctx(ctx);
  if (s != AIHOST_OK) return s;
  KvLayout kv;
  float scale;
  s = check_desc(desc, &kv, &scale);
  if (s != AIHOST_OK) return s;
  if (batch < 1 || n_new < 1) return fail(AIHOST_EINVAL, "batch (%d) and n_new (%d) must be >= 1", batch, n_new);
  if (!k_new || !v_new || !k_cache || !v_cache || !seq_len)
    return fail(AIHOST_EINVAL, "k_new, v_new, k_cache, v_cache and seq_len must be non-NULL");
  if (!aligned(k_new, 16) || !aligned(v_new, 16) || !aligned(k_cache, 16) || !aligned(v_cache, 16))
    return fail(AIHOST_EINVAL, "tensor pointers must be 16-byte aligned");
  DeviceGuard g(ctx->device);
  if (!g.ok()) return fail(AIHOST_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const RopeFreqs freqs = make_freqs(1.0f, desc->head_dim);
  cudaError_t e = timed_launch(ctx, AIHOST_KERNEL_APPEND, st, [&] {
    return launch_kv_append(k_new, v_new, desc->q_dtype, k_cache, v_cache, kv, seq_len, batch, n_new,
                            desc->n_kv_heads, desc->head_dim, AIHOST_ROPE_NONE, freqs, ctx->d_status, st);
  });
  if (e != cudaSuccess) return cuda_fail(e, "kv append launch");
  return AIHOST_OK;
}

aihost_status aihost_attn_profiler_enable(aihost_attn_ctx* ctx, int32_t enable) {
  aihost_status s = check_ctx(ctx);
  if (s != AIHOST_OK) return s;
  std::lock_guard<std::mutex> lk(ctx->prof_mu);
  ctx->profiling = enable != 0;
  return AIHOST_OK;
}

aihost_status aihost_attn_profiler_read(aihost_attn_ctx* ctx, int32_t kernel, int64_t* launches, double* total_ms) {
  aihost_status s = check_ctx(ctx);
  if (s != AIHOST_OK) return s;
  if (kernel < 0 || kernel >= AIHOST_KERNEL_COUNT) return fail(AIHOST_EINVAL, "kernel id %d out of range", kernel);
  DeviceGuard g(ctx->device);
  std::lock_guard<std::mutex> lk(ctx->prof_mu);
  ProfSlot& slot = ctx->prof[kernel];
  for (auto& pr : slot.pending) {
    cudaError_t e = cudaEventSynchronize(pr.second);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventSynchronize(profiler)");
    float ms = 0.0f;
    e = cudaEventElapsedTime(&ms, pr.first, pr.second);
    if (e != cudaSuccess) return cuda_fail(e, "cudaEventElapsedTime(profiler)");
    slot.total_ms += ms;
    slot.launches += 1;
    ctx->event_pool.push_back(pr.first);
    ctx->event_pool.push_back(pr.second);
  }
  slot.pending.clear();
  if (launches) *launches = slot.launches;
  if (total_ms) *total_ms = slot.total_ms;
  return AIHOST_OK;
}

aihost_status aihost_attn_profiler_reset(aihost_attn_ctx* ctx) {
  aihost_status s = check_ctx(ctx);
  if (s != AIHOST_OK) return s;
  for (int k = 0; k < AIHOST_KERNEL_COUNT; ++k) {
    s = aihost_attn_profiler_read(ctx, k, nullptr, nullptr);
    if (s != AIHOST_OK) return s;
    std::lock_guard<std::mutex> lk(ctx->prof_mu);
    ctx->prof[k].launches = 0;
    ctx->prof[k].total_ms = 0.0;
  }
  return AIHOST_OK;
}

// ------------------------------------------------------------------ weight products
}  // extern "C"

namespace {

bool is_kquant(int32_t t) { return t >= AIHOST_Q2_K && t <= AIHOST_Q6_K; }

aihost_status check_matmul(const aihost_matmul_desc* d) {
  if (!d) return fail(AIHOST_EINVAL, "desc is NULL");
  if (d->rows < 1 || d->k < 1 || d->n_out < 1 || d->n_parts < 1)
    return fail(AIHOST_EINVAL, "rows (%d), k (%d), n_out (%d) and n_parts (%d) must be >= 1", d->rows, d->k,
                d->n_out, d->n_parts);
  if (d->k % 64 || d->k % d->n_parts || (d->k / d->n_parts) % 64)
    return fail(AIHOST_EINVAL, "k (%d) and k / n_parts must be multiples of 64", d->k);
  if (d->n_out % 8) return fail(AIHOST_EINVAL, "n_out (%d) must be a multiple of 8", d->n_out);
  if (d->a_dtype != AIHOST_F16 && d->a_dtype != AIHOST_F32) return fail(AIHOST_EINVAL, "a_dtype must be F16 or F32");
  if (d->out_dtype != AIHOST_F16 && d->out_dtype != AIHOST_F32)
    return fail(AIHOST_EINVAL, "out_dtype must be F16 or F32");
  if (d->w_dtype != AIHOST_F16 && d->w_dtype != AIHOST_F32 && !is_kquant(d->w_dtype))
    return fail(AIHOST_EINVAL, "w_dtype %d must be F16, F32 or a K-quant (Q2_K..Q6_K)", d->w_dtype);
  if (is_kquant(d->w_dtype) && d->k % 256)
    return fail(AIHOST_EINVAL, "k (%d) must be a multiple of 256 for K-quant weights", d->k);
  return AIHOST_OK;
}

struct GemmPlan {
  int32_t block_n, k_splits;
  bool fused;               // K-quant weight dequantised inside the GEMM (no fp16 copy)
  size_t a_stage, w_stage;  // scratch bytes (each rounded to 256)
};

// Output tiles that leave at least half of the CTA slots empty split their K range over a
// cluster of 2, 4 or 8 CTAs (the largest power of two that fits in one wave of slots; with the
// weight dequantised in the GEMM, one that also splits the 256-value super-blocks evenly).
GemmPlan plan_gemm(const aihost_matmul_desc* d, int32_t num_sms) {
  GemmPlan p;
  p.block_n = gemm_block_n(d->rows, d->n_out, num_sms);
  const int64_t tiles = gemm_tiles(d->rows, d->n_out, p.block_n);
  const int64_t kt_total = d->k / 64;
  const int64_t slots = (p.block_n == 64 || p.block_n == -64 ? 2LL : 1LL) * num_sms;
  p.fused = gemm_fuses_dequant(d->w_dtype, p.block_n);
  int32_t splits = 1;
  if (p.block_n != 256)
    while (splits < 8 && 2 * splits <= kt_total && 2 * splits * tiles <= slots &&
           (!p.fused || (d->k / 256) % (2 * splits) == 0))
      splits *= 2;
  p.k_splits = splits;
  p.a_stage = d->a_dtype == AIHOST_F16 ? 0 : round256(static_cast<size_t>(d->rows) * d->k * 2);
  p.w_stage = d->w_dtype == AIHOST_F16 || p.fused ? 0 : round256(static_cast<size_t>(d->n_out) * d->k * 2);
  return p;
}

int32_t current_sms() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms > 0 ? sms : 148;
}

aihost_status encode_2d_f16(CUtensorMap* map, const void* base, uint64_t inner, uint64_t outer, uint64_t stride_bytes,
                            uint32_t box_inner, uint32_t box_outer, const char* what) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(AIHOST_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (!aligned(base, 16) || stride_bytes % 16) return fail(AIHOST_EINVAL, "%s must be 16-byte aligned", what);
  cuuint64_t dims[2] = {inner, outer};
  cuuint64_t strides[1] = {stride_bytes};
  cuuint32_t box[2] = {box_inner, box_outer};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AIHOST_ECUDA, "cuTensorMapEncodeTiled(%s) failed with %d", what, static_cast<int>(r));
  return AIHOST_OK;
}

// The raw GGUF rows of a K-quant weight as bytes: dims {row bytes, rows}, box {one 256-value
// block, 128 rows}, no swizzle (the block sizes used, 144 and 176, are multiples of 16).
aihost_status encode_raw_rows(CUtensorMap* map, const void* base, uint64_t row_bytes, uint64_t rows,
                              uint32_t block_bytes) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(AIHOST_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (!aligned(base, 16) || row_bytes % 16 || block_bytes % 16) return fail(AIHOST_EINVAL, "w must be 16-byte aligned");
  cuuint64_t dims[2] = {row_bytes, rows};
  cuuint64_t strides[1] = {row_bytes};
  cuuint32_t box[2] = {block_bytes, 128};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AIHOST_ECUDA, "cuTensorMapEncodeTiled(w raw) failed with %d", static_cast<int>(r));
  return AIHOST_OK;
}

aihost_status encode_3d_f16(CUtensorMap* map, const void* base, uint64_t d0, uint64_t d1, uint64_t d2, uint64_t s1,
                            uint64_t s2, uint32_t b0, uint32_t b1, const char* what) {
  EncodeTiledFn enc = get_encode_fn();
  if (!enc) return fail(AIHOST_ECUDA, "cuTensorMapEncodeTiled is not available from the driver");
  if (!aligned(base, 16) || s1 % 16 || s2 % 16) return fail(AIHOST_EINVAL, "%s must be 16-byte aligned", what);
  cuuint64_t dims[3] = {d0, d1, d2};
  cuuint64_t strides[2] = {s1, s2};
  cuuint32_t box[3] = {b0, b1, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                   CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(AIHOST_ECUDA, "cuTensorMapEncodeTiled(%s) failed with %d", what, static_cast<int>(r));
  return AIHOST_OK;
}

}  // namespace

extern "C" {

aihost_status aihost_matmul_workspace_size(const aihost_matmul_desc* desc, size_t* out_bytes) {
  if (!out_bytes) return fail(AIHOST_EINVAL, "out_bytes is NULL");
  aihost_status s = check_matmul(desc);
  if (s != AIHOST_OK) return s;
  const GemmPlan p = plan_gemm(desc, current_sms());
  *out_bytes = p.a_stage + p.w_stage;
  return AIHOST_OK;
}

aihost_status aihost_matmul_weights(aihost_attn_ctx* ctx, const aihost_matmul_desc* desc, const void* a,
                                    const void* w, void* out, void* stream) {
  aihost_status s = check_ctx(ctx);
  if (s != AIHOST_OK) return s;
  s = check_matmul(desc);
  if (s != AIHOST_OK) return s;
  if (!a || !w || !out) return fail(AIHOST_EINVAL, "a, w and out must be non-NULL");
  if (!aligned(a, 16) || !aligned(w, 16) || !aligned(out, 16))
    return fail(AIHOST_EINVAL, "a, w and out must be 16-byte aligned");
  DeviceGuard g(ctx->device);
  if (!g.ok()) return fail(AIHOST_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
  const GemmPlan p = plan_gemm(desc, ctx->num_sms);
  const size_t need = p.a_stage + p.w_stage;
  if (need > ctx->scratch_bytes)
    return fail(AIHOST_ENOMEM, "this product needs %zu bytes of scratch, context has %zu (aihost_matmul_workspace_size)",
                need, ctx->scratch_bytes);
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  uint8_t* sp = static_cast<uint8_t*>(ctx->scratch);
  const int64_t M = desc->rows, K = desc->k, N = desc->n_out, parts = desc->n_parts;
  const void* a16 = a;
  const void* w16 = w;
  if (desc->a_dtype == AIHOST_F32) {
    __half* dst = reinterpret_cast<__half*>(sp);
    sp += p.a_stage;
    cudaError_t e = timed_launch(ctx, AIHOST_KERNEL_CONVERT, st, [&] {
      return launch_f32_to_f16(static_cast<const float*>(a), dst, M * K, ctx->num_sms, st);
    });
    if (e != cudaSuccess) return cuda_fail(e, "A conversion launch");
    a16 = dst;
  }
  if (desc->w_dtype != AIHOST_F16 && !p.fused) {
    __half* dst = reinterpret_cast<__half*>(sp);
    sp += p.w_stage;
    cudaError_t e = timed_launch(ctx, AIHOST_KERNEL_CONVERT, st, [&] {
      return desc->w_dtype == AIHOST_F32 ? launch_f32_to_f16(static_cast<const float*>(w), dst, N * K, ctx->num_sms, st)
                                         : launch_dequant(w, desc->w_dtype, N * K, dst, AIHOST_F16, st);
    });
    if (e != cudaSuccess) return cuda_fail(e, "weight dequantisation launch");
    w16 = dst;
  }
  GemmArgs ga;
  memset(&ga, 0, sizeof(ga));
  const int64_t part_cols = K / parts;
  const bool swap = p.block_n < 0;
  const uint32_t a_rows = swap ? static_cast<uint32_t>(-p.block_n) : 128u, w_rows = swap ? 128u : p.block_n;
  s = encode_3d_f16(&ga.a_map, a16, part_cols, M, parts, part_cols * 2, M * part_cols * 2, 64, a_rows, "a");
  if (s != AIHOST_OK) return s;
  ga.w_type = p.fused ? desc->w_dtype : AIHOST_F16;
  if (p.fused) {
    const uint32_t bb = static_cast<uint32_t>(weight_block_bytes(desc->w_dtype));
    s = encode_raw_rows(&ga.w_raw_map, w, K / 256 * bb, N, bb);
  } else {
    s = encode_2d_f16(&ga.b_map, w16, K, N, K * 2, 64, w_rows, "w");
  }
  if (s != AIHOST_OK) return s;
  ga.M = desc->rows;
  ga.N = desc->n_out;
  ga.K = desc->k;
  ga.part_cols = static_cast<int32_t>(part_cols);
  ga.k_splits = p.k_splits;
  ga.out = out;
  ga.out_dtype = desc->out_dtype;
  ga.ldc = N;
  ga.status = ctx->d_status;
  cudaError_t e = timed_launch(ctx, AIHOST_KERNEL_MATMUL, st, [&] { return launch_gemm(ga, p.block_n, ctx->num_sms, st); });
  if (e != cudaSuccess) return cuda_fail(e, "matmul launch");
  return AIHOST_OK;
}

aihost_status aihost_dequantize(const void* w, int32_t w_dtype, int64_t n_elems, void* out, int32_t out_dtype,
                                void* stream) {
  if (!w || !out) return fail(AIHOST_EINVAL, "w and out must be non-NULL");
  if (!is_kquant(w_dtype)) return fail(AIHOST_EINVAL, "w_dtype %d is not a K-quant type (Q2_K..Q6_K)", w_dtype);
  if (out_dtype != AIHOST_F16 && out_dtype != AIHOST_F32) return fail(AIHOST_EINVAL, "out_dtype must be F16 or F32");
  if (n_elems < 0 || n_elems % 256) return fail(AIHOST_EINVAL, "n_elems (%lld) must be a multiple of 256",
                                                static_cast<long long>(n_elems));
  if (!aligned(out, 16)) return fail(AIHOST_EINVAL, "out must be 16-byte aligned");
  cudaError_t e = launch_dequant(w, w_dtype, n_elems, out, out_dtype, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return cuda_fail(e, "dequantisation launch");
  return AIHOST_OK;
}

aihost_status aihost_attn_sync_status(aihost_attn_ctx* ctx, int32_t* out_bits) {
  aihost_status s = check_ctx(ctx);
  if (s != AIHOST_OK) return s;
  DeviceGuard g(ctx->device);
  if (!g.ok()) return fail(AIHOST_ECUDA, "cudaSetDevice(%d) failed", ctx->device);
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e, "cudaDeviceSynchronize");
  int32_t bits = 0;
  e = cudaMemcpy(&bits, ctx->d_status, sizeof(bits), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemcpy(status)");
  e = cudaMemset(ctx->d_status, 0, sizeof(int32_t));
  if (e != cudaSuccess) return cuda_fail(e, "cudaMemset(status)");
  if (out_bits) *out_bits = bits;
  if (bits & kStatusWaitTimeout) return fail(AIHOST_ETIMEOUT, "a kernel's bounded wait expired (status 0x%x)", bits);
  if (bits & kStatusBadLength) return fail(AIHOST_EINVAL, "a device-side sequence length exceeded kv_capacity");
  return AIHOST_OK;
}

}  // extern "C"
