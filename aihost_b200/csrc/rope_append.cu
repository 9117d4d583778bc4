// rope_append.cu — RoPE and KV-cache append kernels.
//
// rope_full_kernel   : ComputeOps.ApplyRoPEFull (ComputeOps.cs:959-979, shader
//                      ComputeShaders.cs:517-543), in place, one thread per rotation pair.
// kv_append_kernel   : KVCache.Add (Inference/InferenceEngine.cs:598-622) into a preallocated
//                      cache instead of a Concat copy of the whole cache per token; optionally
//                      rotates K on the way (the ComputeOps.cs:1283 RoPE of the new K), and
//                      converts to the cache dtype (fp32 copy, fp16 round-to-nearest-even, or
//                      GGUF Q8_0 quantisation with ggml's reference rule d = amax/127,
//                      q = roundf(x * (1/d)), d stored as fp16).
// stage_q_kernel / stage_kv_kernel: fp32 Q and fp32 / Q8_0 cache rows converted to fp16 for
//                      the tensor-core prefill (the reference computes those in fp32 shaders).
// Row RoPE and storage conversion live in rows.cuh (shared with the decode kernels).
#include "common.cuh"
#include "kernels.h"
#include "rows.cuh"

namespace aihost {
namespace {

template <typename T>
__global__ void rope_full_kernel(T* __restrict__ x, int32_t seq, int32_t n_heads, int32_t head_dim,
                                 int32_t start_pos, int32_t rope_mode, RopeFreqs freqs) {
  const int32_t half = head_dim / 2;
  const int64_t total = static_cast<int64_t>(seq) * n_heads * half;
  for (int64_t gid = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; gid < total;
       gid += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int32_t pair = static_cast<int32_t>(gid % half);
    const int64_t row = gid / half;  // = s * n_heads + h
    const int32_t s = static_cast<int32_t>(row / n_heads);
    const float angle = __fmul_rn(static_cast<float>(start_pos + s), freqs.f[pair]);
    float sn, cs;
    sincosf(angle, &sn, &cs);
    const int32_t i1 = rope_mode == AIHOST_ROPE_NEOX ? pair : 2 * pair;
    const int32_t i2 = rope_mode == AIHOST_ROPE_NEOX ? pair + half : 2 * pair + 1;
    T* base = x + row * head_dim;
    float x1 = ld_as_float(base + i1), x2 = ld_as_float(base + i2);
    rotate_pair(x1, x2, cs, sn);
    st_from_float(base + i1, x1);
    st_from_float(base + i2, x2);
  }
}

__device__ __forceinline__ float load_in(const float* p) { return *p; }
__device__ __forceinline__ float load_in(const __half* p) { return __half2float(*p); }

// One warp per (batch, token, kv head) row; lane l holds elements [l*E, l*E+E), E = D/32.
// blockIdx.y selects K (0, rotated) or V (1).
template <typename Tin, int D>
__global__ void kv_append_kernel(const Tin* __restrict__ k_new, const Tin* __restrict__ v_new,
                                 uint8_t* __restrict__ k_cache, uint8_t* __restrict__ v_cache, KvLayout kv,
                                 const int32_t* __restrict__ seq_len, int32_t batch, int32_t n_new,
                                 int32_t n_kv_heads, int32_t rope_mode, RopeFreqs freqs, int32_t* status,
                                 const int32_t* __restrict__ rope_pos) {
  constexpr int E = D / 32;
  griddep_launch_dependents();  // the prefill that follows may start its own set-up now
  __shared__ float s_f[D / 2];  // RoPE frequencies, read below by lane-dependent index
  for (int i = threadIdx.x; i < D / 2; i += blockDim.x) s_f[i] = freqs.f[i];
  __syncthreads();
  const int32_t lane = threadIdx.x & 31;
  const int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
  const int64_t rows = static_cast<int64_t>(batch) * n_new * n_kv_heads;
  if (row >= rows) return;
  const bool is_k = blockIdx.y == 0;
  const int32_t h = static_cast<int32_t>(row % n_kv_heads);
  const int32_t s = static_cast<int32_t>((row / n_kv_heads) % n_new);
  const int32_t b = static_cast<int32_t>(row / (static_cast<int64_t>(n_kv_heads) * n_new));
  const int32_t start = seq_len[b];
  const int32_t t = start + s;
  if (start < 0 || t >= kv.capacity || !kv_row_ok(kv, b, t)) {
    if (lane == 0 && is_k && h == 0) atomicOr(status, kStatusBadLength);
    return;
  }
  const Tin* src = (is_k ? k_new : v_new) + row * D + lane * E;
  float x[E];
#pragma unroll
  for (int e = 0; e < E; ++e) x[e] = load_in(src + e);

  if (is_k && rope_mode != AIHOST_ROPE_NONE) {
    const float pos = static_cast<float>(rope_pos ? rope_pos[b] + s : t);
    rope_row_warp<E>(x, lane, pos, rope_mode, static_cast<const float*>(s_f));
  }

  uint8_t* dst = (is_k ? k_cache : v_cache) + kv_row_offset(kv, b, t) + static_cast<int64_t>(h) * kv.head_stride;
  store_row_warp<E>(x, lane, dst, kv.dtype);
}

// fp16 staging for the tensor-core prefill, whose operands are fp16 (fp32 accumulation).
// stage_q_kernel: q [B][S][Hq][D] fp32 -> fp16, rotated at position start_b + s on the way (one
// rounding to fp16, after the fp32 rotation). One warp per head row.
template <int D>
__global__ void stage_q_kernel(const float* __restrict__ q, __half* __restrict__ dst, const int32_t* __restrict__ seq_len,
                               int32_t start_scalar, int32_t batch, int32_t n_q, int32_t n_heads, int32_t rope_mode,
                               RopeFreqs freqs) {
  constexpr int E = D / 32;
  griddep_launch_dependents();  // the prefill that follows may start its own set-up now
  __shared__ float s_f[D / 2];  // RoPE frequencies, read below by lane-dependent index
  for (int i = threadIdx.x; i < D / 2; i += blockDim.x) s_f[i] = freqs.f[i];
  __syncthreads();
  const int32_t lane = threadIdx.x & 31;
  const int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= static_cast<int64_t>(batch) * n_q * n_heads) return;
  const int32_t s = static_cast<int32_t>((row / n_heads) % n_q);
  const int32_t b = static_cast<int32_t>(row / (static_cast<int64_t>(n_heads) * n_q));
  float x[E];
  const float* src = q + row * D + lane * E;
#pragma unroll
  for (int e = 0; e < E; ++e) x[e] = src[e];
  if (rope_mode != AIHOST_ROPE_NONE) {
    const int32_t start = seq_len ? seq_len[b] : start_scalar;
    rope_row_warp<E>(x, lane, static_cast<float>(start + s), rope_mode, static_cast<const float*>(s_f));
  }
  __half2* d2 = reinterpret_cast<__half2*>(dst + row * D + lane * E);
#pragma unroll
  for (int e = 0; e < E; e += 2) d2[e / 2] = __floats2half2_rn(x[e], x[e + 1]);
}

// stage_kv_kernel: cache rows [0, start_b + len_offset) of an fp32 or Q8_0 cache -> a dense fp16
// [B][rows][Hkv][D] copy (rows past a sequence's length are left as they are: the prefill kernel
// masks them). Q8_0 values are d * q in fp32, then rounded once to fp16. blockIdx.y: 0 = K, 1 = V.
template <int D>
__global__ void stage_kv_kernel(const uint8_t* __restrict__ k_cache, const uint8_t* __restrict__ v_cache, KvLayout kv,
                                __half* __restrict__ k_dst, __half* __restrict__ v_dst, int32_t rows,
                                const int32_t* __restrict__ seq_len, int32_t start_scalar, int32_t len_offset,
                                int32_t batch, int32_t n_kv_heads) {
  constexpr int E = D / 32;
  griddep_launch_dependents();  // the prefill that follows may start its own set-up now
  const int32_t lane = threadIdx.x & 31;
  const int64_t row = blockIdx.x * static_cast<int64_t>(blockDim.x >> 5) + (threadIdx.x >> 5);
  if (row >= static_cast<int64_t>(batch) * rows * n_kv_heads) return;
  const int32_t h = static_cast<int32_t>(row % n_kv_heads);
  const int32_t t = static_cast<int32_t>((row / n_kv_heads) % rows);
  const int32_t b = static_cast<int32_t>(row / (static_cast<int64_t>(n_kv_heads) * rows));
  const int32_t len = (seq_len ? seq_len[b] : start_scalar) + len_offset;
  if (t >= len || t >= kv.capacity) return;
  const bool is_k = blockIdx.y == 0;
  const uint8_t* src = (is_k ? k_cache : v_cache) + kv_row_offset(kv, b, t) + static_cast<int64_t>(h) * kv.head_stride;
  float x[E];
  if (kv.dtype == AIHOST_F32) {
    const float* f = reinterpret_cast<const float*>(src) + lane * E;
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = f[e];
  } else {  // Q8_0: element i is in block i / 32 (34 bytes: fp16 d, then 32 int8)
    const int i0 = lane * E;
    const uint8_t* blk = src + (i0 / 32) * 34;
    const float dsc = __half2float(__ushort_as_half(*reinterpret_cast<const uint16_t*>(blk)));
    const uint16_t* qs = reinterpret_cast<const uint16_t*>(blk + 2 + (i0 % 32));  // even offset: 2-byte loads
#pragma unroll
    for (int e = 0; e < E; e += 2) {
      const uint16_t w = qs[e / 2];
      x[e] = __fmul_rn(dsc, static_cast<float>(static_cast<int8_t>(w & 0xff)));
      x[e + 1] = __fmul_rn(dsc, static_cast<float>(static_cast<int8_t>(w >> 8)));
    }
  }
  __half2* d2 = reinterpret_cast<__half2*>((is_k ? k_dst : v_dst) + row * D + lane * E);
#pragma unroll
  for (int e = 0; e < E; e += 2) d2[e / 2] = __floats2half2_rn(x[e], x[e + 1]);
}

}  // namespace

// Qwen TypeB Q/K prologue (Compute/Formats/QwenHybridFormat.cs:141-142): one CTA per token row
// of x [seq, n_heads * head_dim]. The reference's LayerNorm (ComputeShaders.cs:249-277) takes the
// RMS over the whole row, all heads together, and multiplies by a head_dim weight tiled over the
// heads (TransformerBase.cs:301-319); ApplyRoPEFull then rotates each head. Here both happen in
// one pass over the row: sum of squares (block reduction), then per rotation pair
// x / rms * w and the rotation, stored in place with one rounding.
template <typename T>
__global__ void __launch_bounds__(256) qk_norm_rope_kernel(T* __restrict__ x, int32_t n_heads, int32_t head_dim,
                                                           const float* __restrict__ w, float eps, int32_t start_pos,
                                                           int32_t rope_mode, RopeFreqs freqs) {
  __shared__ float part[8];
  const int32_t cols = n_heads * head_dim;
  T* row = x + static_cast<int64_t>(blockIdx.x) * cols;
  float acc = 0.0f;
  for (int32_t i = threadIdx.x; i < cols; i += blockDim.x) {
    const float v = ld_as_float(row + i);
    acc = fmaf(v, v, acc);
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  float total = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) total += part[i];
  const float rms = sqrtf(total / static_cast<float>(cols) + eps);
  const int32_t half = head_dim / 2;
  const float pos = static_cast<float>(start_pos + static_cast<int32_t>(blockIdx.x));
  for (int32_t p = threadIdx.x; p < n_heads * half; p += blockDim.x) {
    const int32_t h = p / half, i = p % half;
    const int32_t i1 = rope_mode == AIHOST_ROPE_NEOX ? i : 2 * i;
    const int32_t i2 = rope_mode == AIHOST_ROPE_NEOX ? i + half : 2 * i + 1;
    T* base = row + static_cast<int64_t>(h) * head_dim;
    float x1 = ld_as_float(base + i1) / rms * w[i1];
    float x2 = ld_as_float(base + i2) / rms * w[i2];
    if (rope_mode != AIHOST_ROPE_NONE) {
      float sn, cs;
      sincosf(__fmul_rn(pos, freqs.f[i]), &sn, &cs);
      rotate_pair(x1, x2, cs, sn);
    }
    st_from_float(base + i1, x1);
    st_from_float(base + i2, x2);
  }
}

__device__ __forceinline__ void load8(const float* p, float* v) {
  const float4 a = *reinterpret_cast<const float4*>(p), b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x; v[1] = a.y; v[2] = a.z; v[3] = a.w; v[4] = b.x; v[5] = b.y; v[6] = b.z; v[7] = b.w;
}
__device__ __forceinline__ void load8(const __half* p, float* v) {
  const uint4 u = *reinterpret_cast<const uint4*>(p);
  const __half2* h = reinterpret_cast<const __half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float2 f = __half22float2(h[i]);
    v[2 * i] = f.x;
    v[2 * i + 1] = f.y;
  }
}
__device__ __forceinline__ void store8(float* p, const float* v) {
  *reinterpret_cast<float4*>(p) = make_float4(v[0], v[1], v[2], v[3]);
  *reinterpret_cast<float4*>(p + 4) = make_float4(v[4], v[5], v[6], v[7]);
}
__device__ __forceinline__ void store8(__half* p, const float* v) {
  uint4 u;
  __half2* h = reinterpret_cast<__half2*>(&u);
#pragma unroll
  for (int i = 0; i < 4; ++i) h[i] = __floats2half2_rn(v[2 * i], v[2 * i + 1]);
  *reinterpret_cast<uint4*>(p) = u;
}

// The same prologue with the row held in registers: a unit is the two 8-element chunks at
// within-head offsets o and o + head_dim/2 (o < head_dim/2), so a NeoX pair never leaves its
// thread; every thread loads its units with 16- or 32-byte loads before the reduction, then
// normalises, rotates and stores them. Needs head_dim % 16 == 0 and at most 256*K units per row.
// The angles go through the reduced-range sincos (absolute error ~5e-7, positions up to ~4e5).
template <typename T, int K>
__global__ void __launch_bounds__(256, K == 1 ? 6 : 3) qk_norm_rope_vec_kernel(T* __restrict__ x, int32_t n_heads, int32_t head_dim,
                                                               const float* __restrict__ w, float eps,
                                                               int32_t start_pos, int32_t rope_mode, RopeFreqs freqs) {
  __shared__ float part[8];
  // the weight and the RoPE frequencies, read by lane-dependent index below: from shared memory
  // rather than from the kernel parameters (divergent constant reads serialise per address)
  __shared__ __align__(16) float s_w[kMaxHeadDim];
  __shared__ float s_f[kMaxHeadDim / 2];
  const int32_t cols = n_heads * head_dim, half = head_dim / 2, per_head = head_dim / 16;
  const int32_t units = n_heads * per_head;
  if (threadIdx.x < head_dim) s_w[threadIdx.x] = w[threadIdx.x];
  if (threadIdx.x < half) s_f[threadIdx.x] = freqs.f[threadIdx.x];
  T* row = x + static_cast<int64_t>(blockIdx.x) * cols;
  float v[K][16];
  float acc = 0.0f;
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int32_t u = threadIdx.x + 256 * k;
    if (u < units) {
      const int32_t a = (u / per_head) * head_dim + (u % per_head) * 8;
      load8(row + a, v[k]);
      load8(row + a + half, v[k] + 8);
#pragma unroll
      for (int e = 0; e < 16; ++e) acc = fmaf(v[k][e], v[k][e], acc);
    }
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) part[threadIdx.x >> 5] = acc;
  __syncthreads();
  float total = 0.0f;
#pragma unroll
  for (int i = 0; i < 8; ++i) total += part[i];
  // x * (1 / rms) instead of the reference's x / rms: at most one ulp apart, and the division
  // dominated this kernel's instruction count
  const float inv_rms = __frcp_rn(sqrtf(total / static_cast<float>(cols) + eps));
  const float pos = static_cast<float>(start_pos + static_cast<int32_t>(blockIdx.x));
#pragma unroll
  for (int k = 0; k < K; ++k) {
    const int32_t u = threadIdx.x + 256 * k;
    if (u >= units) continue;
    const int32_t o = (u % per_head) * 8;
    const int32_t a = (u / per_head) * head_dim + o;
    float wa[8], wb[8];
    load8(s_w + o, wa);
    load8(s_w + half + o, wb);
#pragma unroll
    for (int e = 0; e < 8; ++e) {
      v[k][e] = v[k][e] * inv_rms * wa[e];
      v[k][8 + e] = v[k][8 + e] * inv_rms * wb[e];
    }
    if (rope_mode == AIHOST_ROPE_INTERLEAVED) {
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float sn, cs;
        sincos_reduced(__fmul_rn(pos, s_f[o / 2 + q]), &sn, &cs);
        rotate_pair(v[k][2 * q], v[k][2 * q + 1], cs, sn);
        sincos_reduced(__fmul_rn(pos, s_f[half / 2 + o / 2 + q]), &sn, &cs);
        rotate_pair(v[k][8 + 2 * q], v[k][8 + 2 * q + 1], cs, sn);
      }
    } else if (rope_mode == AIHOST_ROPE_NEOX) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        float sn, cs;
        sincos_reduced(__fmul_rn(pos, s_f[o + e]), &sn, &cs);
        rotate_pair(v[k][e], v[k][8 + e], cs, sn);
      }
    }
    store8(row + a, v[k]);
    store8(row + a + half, v[k] + 8);
  }
}

cudaError_t launch_qk_norm_rope(void* x, int32_t dtype, int32_t seq, int32_t n_heads, int32_t head_dim,
                                const float* w, float eps, int32_t start_pos, int32_t rope_mode, const RopeFreqs& freqs,
                                cudaStream_t st) {
  if (seq == 0) return cudaSuccess;
  const int64_t units = static_cast<int64_t>(n_heads) * (head_dim / 16);
  if (head_dim % 16 == 0 && reinterpret_cast<uintptr_t>(x) % 16 == 0 && units <= 1024) {
#define AIHOST_QKN(T, K)                                                                                           \
  qk_norm_rope_vec_kernel<T, K><<<seq, 256, 0, st>>>(static_cast<T*>(x), n_heads, head_dim, w, eps, start_pos, \
                                                    rope_mode, freqs)
    if (dtype == AIHOST_F32) {
      if (units <= 256) AIHOST_QKN(float, 1);
      else if (units <= 512) AIHOST_QKN(float, 2);
      else AIHOST_QKN(float, 4);
    } else {
      if (units <= 256) AIHOST_QKN(__half, 1);
      else if (units <= 512) AIHOST_QKN(__half, 2);
      else AIHOST_QKN(__half, 4);
    }
#undef AIHOST_QKN
    return cudaGetLastError();
  }
  if (dtype == AIHOST_F32)
    qk_norm_rope_kernel<float><<<seq, 256, 0, st>>>(static_cast<float*>(x), n_heads, head_dim, w, eps, start_pos,
                                                     rope_mode, freqs);
  else
    qk_norm_rope_kernel<__half><<<seq, 256, 0, st>>>(static_cast<__half*>(x), n_heads, head_dim, w, eps, start_pos,
                                                      rope_mode, freqs);
  return cudaGetLastError();
}

cudaError_t launch_rope_full(void* x, int32_t dtype, int32_t seq, int32_t n_heads, int32_t head_dim,
                             int32_t start_pos, int32_t rope_mode, const RopeFreqs& freqs, cudaStream_t st) {
  const int64_t total = static_cast<int64_t>(seq) * n_heads * (head_dim / 2);
  if (total == 0) return cudaSuccess;
  const int threads = 256;
  const int64_t want = (total + threads - 1) / threads;
  const int blocks = static_cast<int>(want < 148 * 64 ? want : 148 * 64);
  if (dtype == AIHOST_F32)
    rope_full_kernel<float><<<blocks, threads, 0, st>>>(static_cast<float*>(x), seq, n_heads, head_dim, start_pos,
                                                        rope_mode, freqs);
  else
    rope_full_kernel<__half><<<blocks, threads, 0, st>>>(static_cast<__half*>(x), seq, n_heads, head_dim, start_pos,
                                                         rope_mode, freqs);
  return cudaGetLastError();
}

cudaError_t launch_kv_append(const void* k_new, const void* v_new, int32_t in_dtype, void* k_cache,
                             void* v_cache, const KvLayout& kv, const int32_t* seq_len, int32_t batch,
                             int32_t n_new, int32_t n_kv_heads, int32_t head_dim, int32_t rope_mode,
                             const RopeFreqs& freqs, int32_t* status, cudaStream_t st, const int32_t* rope_pos) {
  const int64_t rows = static_cast<int64_t>(batch) * n_new * n_kv_heads;
  if (rows == 0) return cudaSuccess;
  const int warps = 8;
  dim3 grid(static_cast<unsigned>((rows + warps - 1) / warps), 2);
  auto* kc = static_cast<uint8_t*>(k_cache);
  auto* vc = static_cast<uint8_t*>(v_cache);
#define AIHOST_APPEND(TIN, DD)                                                                                   \
  kv_append_kernel<TIN, DD><<<grid, warps * 32, 0, st>>>(static_cast<const TIN*>(k_new),                         \
                                                         static_cast<const TIN*>(v_new), kc, vc, kv, seq_len, \
                                                         batch, n_new, n_kv_heads, rope_mode, freqs, status, rope_pos)
  if (in_dtype == AIHOST_F32) {
    if (head_dim == 64) AIHOST_APPEND(float, 64);
    else AIHOST_APPEND(float, 128);
  } else {
    if (head_dim == 64) AIHOST_APPEND(__half, 64);
    else AIHOST_APPEND(__half, 128);
  }
#undef AIHOST_APPEND
  return cudaGetLastError();
}


cudaError_t launch_stage_q(const float* q, __half* dst, const int32_t* seq_len, int32_t start_scalar, int32_t batch,
                           int32_t n_q, int32_t n_heads, int32_t head_dim, int32_t rope_mode, const RopeFreqs& freqs,
                           cudaStream_t st) {
  const int64_t rows = static_cast<int64_t>(batch) * n_q * n_heads;
  if (rows == 0) return cudaSuccess;
  const int warps = 8;
  const unsigned grid = static_cast<unsigned>((rows + warps - 1) / warps);
  if (head_dim == 64)
    stage_q_kernel<64><<<grid, warps * 32, 0, st>>>(q, dst, seq_len, start_scalar, batch, n_q, n_heads, rope_mode,
                                                    freqs);
  else
    stage_q_kernel<128><<<grid, warps * 32, 0, st>>>(q, dst, seq_len, start_scalar, batch, n_q, n_heads, rope_mode,
                                                     freqs);
  return cudaGetLastError();
}

cudaError_t launch_stage_kv(const void* k_cache, const void* v_cache, const KvLayout& kv, __half* k_dst,
                            __half* v_dst, int32_t rows, const int32_t* seq_len, int32_t start_scalar,
                            int32_t len_offset, int32_t batch, int32_t n_kv_heads, int32_t head_dim, cudaStream_t st) {
  const int64_t n = static_cast<int64_t>(batch) * rows * n_kv_heads;
  if (n == 0) return cudaSuccess;
  const int warps = 8;
  dim3 grid(static_cast<unsigned>((n + warps - 1) / warps), 2);
  auto* kc = static_cast<const uint8_t*>(k_cache);
  auto* vc = static_cast<const uint8_t*>(v_cache);
  if (head_dim == 64)
    stage_kv_kernel<64><<<grid, warps * 32, 0, st>>>(kc, vc, kv, k_dst, v_dst, rows, seq_len, start_scalar,
                                                     len_offset, batch, n_kv_heads);
  else
    stage_kv_kernel<128><<<grid, warps * 32, 0, st>>>(kc, vc, kv, k_dst, v_dst, rows, seq_len, start_scalar,
                                                      len_offset, batch, n_kv_heads);
  return cudaGetLastError();
}

}  // namespace aihost
