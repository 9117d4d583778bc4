// decode.cu — split-K flash-decoding for one new token per sequence.
//
// Replaces FusedMHAGenerate (ComputeShaders.cs:656-733, dispatched by ComputeOps.cs:1015-1043).
// The reference runs one workgroup per Q head, re-reads the K/V rows of its KV head once per Q
// head, keeps every score in a 4096-entry shared array (kvSeqLen <= 4096) and sums P.V with
// one thread per output dimension serially over all rows. Here:
//   - one CTA per (sequence, KV head, group of up to 8 Q heads, split of `chunk` rows): every
//     KV byte is read once for the whole GQA group, and rows are spread over the whole GPU;
//   - lanes own head_dim slices, so each K/V row is one coalesced warp-wide load;
//   - the G dot products of a row are reduced with a multi-value butterfly (G/2 + ... + 1
//     shuffles per row instead of 5*G);
//   - partial (max, sum, unnormalised P.V) per split are merged (the exp-rescaled sum of the
//     standard split softmax), so any length fits: by the split of a (sequence, head group)
//     that arrives last (epoch-tagged counter, no CTA waits on another), or, without counters,
//     by decode_combine_kernel;
//   - with fuse_append (fp32 caches), the CTAs of a sequence's last split rotate the new token's
//     K and load its V themselves; the head group's first CTA also stores both rows into the
//     cache (the append kernel's code, identical bytes), and the new row's scores and P.V use
//     the shared-memory copy, so the whole decode step is one launch.
// Q is rotated inside the kernel (RoPE at the sequence's position). Softmax runs in the
// exp2 domain: s2 = (q.k) * scale * log2(e).
#include "common.cuh"
#include "kernels.h"
#include "rows.cuh"

namespace aihost {
namespace {

constexpr int kDecodeThreads = 256;
constexpr int kDecodeWarps = kDecodeThreads / 32;
constexpr float kLog2e = 1.4426950408889634f;

struct Q8Tag {};

// Load the E consecutive head-row elements starting at `e0` of a row as floats.
template <typename KV, int E>
struct RowLoader;

template <int E>
struct RowLoader<float, E> {
  static __device__ __forceinline__ void load(const uint8_t* row, int e0, float (&x)[E]) {
    const float* p = reinterpret_cast<const float*>(row) + e0;
    if constexpr (E == 4) {
      const float4 v = __ldg(reinterpret_cast<const float4*>(p));
      x[0] = v.x; x[1] = v.y; x[2] = v.z; x[3] = v.w;
    } else {
      const float2 v = __ldg(reinterpret_cast<const float2*>(p));
      x[0] = v.x; x[1] = v.y;
    }
  }
};

template <int E>
struct RowLoader<__half, E> {
  static __device__ __forceinline__ void load(const uint8_t* row, int e0, float (&x)[E]) {
    const __half* p = reinterpret_cast<const __half*>(row) + e0;
    if constexpr (E == 4) {
      const uint2 v = __ldg(reinterpret_cast<const uint2*>(p));
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v.x));
      const float2 b = __half22float2(*reinterpret_cast<const __half2*>(&v.y));
      x[0] = a.x; x[1] = a.y; x[2] = b.x; x[3] = b.y;
    } else {
      const uint32_t v = __ldg(reinterpret_cast<const unsigned int*>(p));
      const float2 a = __half22float2(*reinterpret_cast<const __half2*>(&v));
      x[0] = a.x; x[1] = a.y;
    }
  }
};

// GGUF Q8_0: element i of a head row lives in block i/32 at byte 2 + i%32; the block's fp16
// scale is at byte 0. E consecutive elements never straddle a block (E divides 32).
template <int E>
struct RowLoader<Q8Tag, E> {
  static __device__ __forceinline__ void load(const uint8_t* row, int e0, float (&x)[E]) {
    const uint8_t* blk = row + (e0 >> 5) * 34;
    const uint16_t dbits = static_cast<uint16_t>(__ldg(blk)) | (static_cast<uint16_t>(__ldg(blk + 1)) << 8);
    const float d = __half2float(__ushort_as_half(dbits));
    const uint8_t* qs = blk + 2 + (e0 & 31);
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = d * static_cast<float>(static_cast<int8_t>(__ldg(qs + e)));
  }
};

// Multi-value butterfly: each lane holds v[0..GT) partial sums; afterwards lane l holds the
// full warp sum of v[g] for g = (l >> (5 - log2 GT)) ... returned as the single value for the
// index `my_g` the lane ends up owning.
template <int GT>
__device__ __forceinline__ float butterfly_reduce(float (&v)[GT], int lane, int& my_g) {
  // Stage k halves the number of live values: lanes with bit (4-k) set keep the upper half.
  int base = 0;
#pragma unroll
  for (int width = GT, bit = 16; width > 1; width >>= 1, bit >>= 1) {
    const bool upper = (lane & bit) != 0;
    const int half = width >> 1;
#pragma unroll
    for (int i = 0; i < half; ++i) {
      const float send = upper ? v[i] : v[i + half];
      const float keep = upper ? v[i + half] : v[i];
      v[i] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
    }
    if (upper) base += half;
  }
  // Remaining lanes sharing `base` reduce the single value over the low lane bits.
  float r = v[0];
  int lowbits = 32;
#pragma unroll
  for (int width = GT; width > 1; width >>= 1) lowbits >>= 1;
#pragma unroll
  for (int off = lowbits >> 1; off > 0; off >>= 1) r += __shfl_xor_sync(0xffffffffu, r, off);
  my_g = base;
  return r;
}

// SMALL (splits of at most 64 rows, D = 64): each warp's eight K and eight V rows are loaded at
// kernel entry, before the Q rotation and the append, so a short decode pays one round trip to
// memory for its rows instead of one per loop pass.
template <typename KV, int D, int GT, bool SMALL>
__global__ void __launch_bounds__(kDecodeThreads) decode_splitk_kernel(DecodeArgs a) {
  constexpr int E = D / 32;
  extern __shared__ float4 smem_raw[];
  float* q_s = reinterpret_cast<float*>(smem_raw);      // [GT][D]
  float* sc_s = q_s + GT * D;                            // [GT][chunk]
  float* red_s = sc_s + GT * a.chunk;                    // [warps][GT][D]
  __shared__ float m_s[GT], l_s[GT];

  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int split = blockIdx.x;
  const int G = a.n_q_heads / a.n_kv_heads;
  const int n_sub = (G + GT - 1) / GT;
  const int kvh = blockIdx.y / n_sub, sub = blockIdx.y % n_sub;
  const int b = blockIdx.z;
  const int g_count = min(GT, G - sub * GT);
  const int h0 = kvh * G + sub * GT;

  const int32_t start = a.seq_len ? a.seq_len[b] : a.start_scalar;
  const int32_t Lk = start + a.len_offset;
  if (Lk > a.kv.capacity || Lk < 1) {
    if (threadIdx.x == 0 && split == 0 && blockIdx.y == 0) atomicOr(a.status, kStatusBadLength);
    return;
  }
  const int32_t t0 = split * a.chunk;
  if (t0 >= Lk) return;
  const int32_t n = min(a.chunk, Lk - t0);
  const int n_splits = (Lk + a.chunk - 1) / a.chunk;

  const bool has_new = a.fuse_append && t0 + a.chunk >= Lk;
  const uint8_t* kbase = static_cast<const uint8_t*>(a.k_cache) + kvh * a.kv.head_stride;
  const uint8_t* vbase = static_cast<const uint8_t*>(a.v_cache) + kvh * a.kv.head_stride;
  constexpr int PR = SMALL ? 64 / kDecodeWarps : 1;  // rows per warp preloaded
  float kpre[PR][E], vpre[PR][E];
  if constexpr (SMALL) {
#pragma unroll
    for (int u = 0; u < PR; ++u) {
      const int j = warp + u * kDecodeWarps;
      const bool load = j < n && !(has_new && j == n - 1);  // the new row comes from shared memory
      if (load) {
        RowLoader<KV, E>::load(kbase + kv_row_offset(a.kv, b, t0 + j), lane * E, kpre[u]);
        RowLoader<KV, E>::load(vbase + kv_row_offset(a.kv, b, t0 + j), lane * E, vpre[u]);
      } else {
#pragma unroll
        for (int e = 0; e < E; ++e) kpre[u][e] = vpre[u][e] = 0.0f;
      }
    }
  }

  // ---- the new token's rows (fused append, fp32 caches): rotated K / V of this KV head in
  // shared memory for this split's last row; the group's first CTA also writes them to the cache
  __shared__ __align__(16) float new_s[2][D];
  if (has_new && warp < 2) {
    const bool is_k = warp == 0;
    const int64_t row = static_cast<int64_t>(b) * a.n_kv_heads + kvh;
    const int esz = a.new_dtype == AIHOST_F32 ? 4 : 2;
    const uint8_t* src = static_cast<const uint8_t*>(is_k ? a.k_new : a.v_new) + row * D * esz;
    float x[E];
    load_row_warp<E>(src, a.new_dtype, lane, x);
    const int32_t t = Lk - 1;
    if (is_k && a.rope_mode != AIHOST_ROPE_NONE)
      rope_row_warp<E>(x, lane, static_cast<float>(a.q_pos ? a.q_pos[b] : t), a.rope_mode, a.freqs);
#pragma unroll
    for (int e = 0; e < E; ++e) new_s[warp][lane * E + e] = x[e];
    if (sub == 0) {
      if (!kv_row_ok(a.kv, b, t)) {
        if (lane == 0) atomicOr(a.status, kStatusBadLength);
      } else {
        uint8_t* dst = static_cast<uint8_t*>(const_cast<void*>(is_k ? a.k_cache : a.v_cache)) + kv_row_offset(a.kv, b, t) +
                       static_cast<int64_t>(kvh) * a.kv.head_stride;
        store_row_warp<E>(x, lane, dst, a.kv.dtype);
      }
    }
  }

  // ---- q rows of this group, rotated at the new token's position, kept as floats
  const float pos = static_cast<float>(a.q_pos ? a.q_pos[b] : start + a.rope_pos_offset);
  for (int idx = threadIdx.x; idx < GT * (D / 2); idx += kDecodeThreads) {
    const int g = idx / (D / 2), pair = idx % (D / 2);
    const int i1 = a.rope_mode == AIHOST_ROPE_NEOX ? pair : 2 * pair;
    const int i2 = a.rope_mode == AIHOST_ROPE_NEOX ? pair + D / 2 : 2 * pair + 1;
    float x1 = 0.0f, x2 = 0.0f;
    if (g < g_count) {
      const int64_t qoff = (static_cast<int64_t>(b) * a.n_q_heads + h0 + g) * D;
      if (a.q_dtype == AIHOST_F32) {
        const float* qp = static_cast<const float*>(a.q) + qoff;
        x1 = qp[i1]; x2 = qp[i2];
      } else {
        const __half* qp = static_cast<const __half*>(a.q) + qoff;
        x1 = __half2float(qp[i1]); x2 = __half2float(qp[i2]);
      }
      if (a.rope_mode != AIHOST_ROPE_NONE) {
        float sn, cs;
        sincosf(__fmul_rn(pos, a.freqs.f[pair]), &sn, &cs);
        const float r1 = __fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn));
        const float r2 = __fadd_rn(__fmul_rn(x1, sn), __fmul_rn(x2, cs));
        x1 = r1; x2 = r2;
      }
    }
    q_s[g * D + i1] = x1;
    q_s[g * D + i2] = x2;
  }
  __syncthreads();
  float qr[GT][E];
#pragma unroll
  for (int g = 0; g < GT; ++g)
#pragma unroll
    for (int e = 0; e < E; ++e) qr[g][e] = q_s[g * D + lane * E + e];

  // row t of this sequence: base + kv_row_offset(kv, b, t) (through the block table for a paged cache)
  const float sl2 = a.scale * kLog2e;

  // ---- scores: warp w takes rows t0 + w, t0 + w + 8, ...
  constexpr int U = 4;
  // passes of U rows per warp; with SMALL at most two, unrolled, so the preload slot
  // it * U + u is a compile-time index
  constexpr int kPasses = SMALL ? 2 : (1 << 30);
#pragma unroll
  for (int it = 0; it < kPasses; ++it) {
    const int j0 = warp + it * kDecodeWarps * U;
    if (j0 >= n) break;
    float kx[U][E];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = j0 + u * kDecodeWarps;
      if (has_new && j == n - 1) {
#pragma unroll
        for (int e = 0; e < E; ++e) kx[u][e] = new_s[0][lane * E + e];
      } else if constexpr (SMALL) {
        const int pu = (it * U + u) % PR;  // this row's preload slot (it * U + u < PR for every row read)
#pragma unroll
        for (int e = 0; e < E; ++e) kx[u][e] = kpre[pu][e];
      } else if (j < n) RowLoader<KV, E>::load(kbase + kv_row_offset(a.kv, b, t0 + j), lane * E, kx[u]);
      else {
#pragma unroll
        for (int e = 0; e < E; ++e) kx[u][e] = 0.0f;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = j0 + u * kDecodeWarps;
      float dot[GT];
#pragma unroll
      for (int g = 0; g < GT; ++g) {
        float s = 0.0f;
#pragma unroll
        for (int e = 0; e < E; ++e) s = fmaf(qr[g][e], kx[u][e], s);
        dot[g] = s;
      }
      int my_g;
      const float r = butterfly_reduce<GT>(dot, lane, my_g);
      // every lane now holds the full sum for group member my_g; one lane per g writes
      if (j < n && (lane & ((32 / GT) - 1)) == 0) sc_s[my_g * a.chunk + j] = r * sl2;
    }
  }
  __syncthreads();

  // ---- softmax statistics per group member (warp g owns member g)
  if (warp < GT) {
    float mx = -INFINITY;
    for (int j = lane; j < n; j += 32) mx = fmaxf(mx, sc_s[warp * a.chunk + j]);
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
    float sum = 0.0f;
    for (int j = lane; j < n; j += 32) {
      const float p = exp2f(sc_s[warp * a.chunk + j] - mx);
      sc_s[warp * a.chunk + j] = p;
      sum += p;
    }
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) sum += __shfl_xor_sync(0xffffffffu, sum, off);
    if (lane == 0) { m_s[warp] = mx; l_s[warp] = sum; }
  }
  __syncthreads();

  // ---- P.V: warp w accumulates rows w, w+8, ...; lanes own head_dim slices
  float acc[GT][E];
#pragma unroll
  for (int g = 0; g < GT; ++g)
#pragma unroll
    for (int e = 0; e < E; ++e) acc[g][e] = 0.0f;
#pragma unroll
  for (int it = 0; it < kPasses; ++it) {
    const int j0 = warp + it * kDecodeWarps * U;
    if (j0 >= n) break;
    float vx[U][E];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = j0 + u * kDecodeWarps;
      if (has_new && j == n - 1) {
#pragma unroll
        for (int e = 0; e < E; ++e) vx[u][e] = new_s[1][lane * E + e];
      } else if constexpr (SMALL) {
        const int pu = (it * U + u) % PR;
#pragma unroll
        for (int e = 0; e < E; ++e) vx[u][e] = vpre[pu][e];
      } else if (j < n) RowLoader<KV, E>::load(vbase + kv_row_offset(a.kv, b, t0 + j), lane * E, vx[u]);
      else {
#pragma unroll
        for (int e = 0; e < E; ++e) vx[u][e] = 0.0f;
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int j = j0 + u * kDecodeWarps;
      if (j < n) {
#pragma unroll
        for (int g = 0; g < GT; ++g) {
          const float p = sc_s[g * a.chunk + j];
#pragma unroll
          for (int e = 0; e < E; ++e) acc[g][e] = fmaf(p, vx[u][e], acc[g][e]);
        }
      }
    }
  }
#pragma unroll
  for (int g = 0; g < GT; ++g)
#pragma unroll
    for (int e = 0; e < E; ++e) red_s[(warp * GT + g) * D + lane * E + e] = acc[g][e];
  __syncthreads();

  for (int idx = threadIdx.x; idx < g_count * D; idx += kDecodeThreads) {
    const int g = idx / D, d = idx % D;
    float o = 0.0f;
#pragma unroll
    for (int w = 0; w < kDecodeWarps; ++w) o += red_s[(w * GT + g) * D + d];
    const int h = h0 + g;
    if (n_splits == 1) {
      const float v = o / l_s[g];
      const int64_t oidx = (static_cast<int64_t>(b) * a.n_q_heads + h) * D + d;
      if (a.out_dtype == AIHOST_F32) static_cast<float*>(a.out)[oidx] = v;
      else static_cast<__half*>(a.out)[oidx] = __float2half_rn(v);
      if (a.lse && d == 0) a.lse[static_cast<int64_t>(b) * a.n_q_heads + h] = (m_s[g] + log2f(l_s[g])) * kLn2;
    } else {
      const int64_t pidx = (static_cast<int64_t>(b) * a.n_q_heads + h) * a.max_splits + split;
      a.part_o[pidx * D + d] = o;
      if (d == 0) {
        a.part_ml[pidx * 2] = m_s[g];
        a.part_ml[pidx * 2 + 1] = l_s[g];
      }
    }
  }
  if (n_splits == 1 || !a.counters) return;
  // ---- fused merge: the last split of this (sequence, head group) to arrive combines them all
  __shared__ uint32_t s_last;
  __threadfence();
  __syncthreads();
  unsigned long long* counter = &a.counters[static_cast<int64_t>(b) * gridDim.y + blockIdx.y];
  if (threadIdx.x == 0) {
    const bool last = split_arrive(counter, a.epoch, n_splits, a.status);
    if (last) atomicExch(counter, 0ull);  // a replay of the same launch starts from zero
    s_last = last ? 1u : 0u;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  for (int idx = threadIdx.x; idx < g_count * D; idx += kDecodeThreads) {
    const int g = idx / D, d = idx % D;
    const int h = h0 + g;
    const int64_t base = (static_cast<int64_t>(b) * a.n_q_heads + h) * a.max_splits;
    float m = -INFINITY;
    for (int sp = 0; sp < n_splits; ++sp) m = fmaxf(m, __ldcg(&a.part_ml[(base + sp) * 2]));
    float l = 0.0f, o = 0.0f;
    for (int sp = 0; sp < n_splits; ++sp) {
      const float w = exp2f(__ldcg(&a.part_ml[(base + sp) * 2]) - m);
      l = fmaf(__ldcg(&a.part_ml[(base + sp) * 2 + 1]), w, l);
      o = fmaf(__ldcg(&a.part_o[(base + sp) * D + d]), w, o);
    }
    const float v = o / l;
    const int64_t oidx = (static_cast<int64_t>(b) * a.n_q_heads + h) * D + d;
    if (a.out_dtype == AIHOST_F32) static_cast<float*>(a.out)[oidx] = v;
    else static_cast<__half*>(a.out)[oidx] = __float2half_rn(v);
    if (a.lse && d == 0) a.lse[static_cast<int64_t>(b) * a.n_q_heads + h] = (m + log2f(l)) * kLn2;
  }
}

// Merge the per-split (max, sum, unnormalised output) triples of one (sequence, Q head).
template <int D>
__global__ void __launch_bounds__(D) decode_combine_kernel(DecodeArgs a) {
  const int h = blockIdx.x, b = blockIdx.y, d = threadIdx.x;
  const int32_t start = a.seq_len ? a.seq_len[b] : a.start_scalar;
  const int32_t Lk = start + a.len_offset;
  if (Lk > a.kv.capacity || Lk < 1) return;
  const int n_splits = (Lk + a.chunk - 1) / a.chunk;
  if (n_splits <= 1) return;  // written directly by the split kernel
  const int64_t base = (static_cast<int64_t>(b) * a.n_q_heads + h) * a.max_splits;
  float m = -INFINITY;
  for (int s = 0; s < n_splits; ++s) m = fmaxf(m, a.part_ml[(base + s) * 2]);
  float l = 0.0f, o = 0.0f;
  for (int s = 0; s < n_splits; ++s) {
    const float w = exp2f(a.part_ml[(base + s) * 2] - m);
    l = fmaf(a.part_ml[(base + s) * 2 + 1], w, l);
    o = fmaf(a.part_o[(base + s) * D + d], w, o);
  }
  const float v = o / l;
  const int64_t oidx = (static_cast<int64_t>(b) * a.n_q_heads + h) * D + d;
  if (a.out_dtype == AIHOST_F32) static_cast<float*>(a.out)[oidx] = v;
  else static_cast<__half*>(a.out)[oidx] = __float2half_rn(v);
  if (a.lse && d == 0) a.lse[static_cast<int64_t>(b) * a.n_q_heads + h] = (m + log2f(l)) * kLn2;
}

// One CTA per query row (sequence x head), one thread per output element: the softmax-weighted
// sum of the parts' normalised outputs. Parts with lse = -inf (no rows) get weight 0.
template <typename T>
__global__ void merge_partials_kernel(int32_t n_parts, int64_t rows, int32_t head_dim, const T* __restrict__ o_parts,
                                      const float* __restrict__ lse_parts, T* __restrict__ out, float* lse_out) {
  const int64_t r = blockIdx.x;
  const int d = threadIdx.x;
  float m = -INFINITY;
  for (int p = 0; p < n_parts; ++p) m = fmaxf(m, lse_parts[p * rows + r]);
  float s = 0.0f, acc = 0.0f;
  if (m > -INFINITY) {
    for (int p = 0; p < n_parts; ++p) {
      const float w = expf(lse_parts[p * rows + r] - m);
      s += w;
      if (d < head_dim) acc = fmaf(w, ld_as_float(o_parts + (p * rows + r) * head_dim + d), acc);
    }
  }
  if (d < head_dim) st_from_float(out + r * head_dim + d, s > 0.0f ? acc / s : 0.0f);
  if (lse_out && d == 0) lse_out[r] = s > 0.0f ? m + logf(s) : -INFINITY;
}

template <typename KV, int D, int GT>
cudaError_t launch_split(const DecodeArgs& a, cudaStream_t st) {
  const int G = a.n_q_heads / a.n_kv_heads;
  const int n_sub = (G + GT - 1) / GT;
  const size_t smem = sizeof(float) * (GT * D + GT * a.chunk + kDecodeWarps * GT * D);
  auto kern = D == 64 && a.chunk <= 64 ? decode_splitk_kernel<KV, D, GT, D == 64> : decode_splitk_kernel<KV, D, GT, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
  if (e != cudaSuccess) return e;
  dim3 grid(a.max_splits, a.n_kv_heads * n_sub, a.batch);
  kern<<<grid, kDecodeThreads, smem, st>>>(a);
  return cudaGetLastError();
}

template <typename KV, int D>
cudaError_t launch_g(const DecodeArgs& a, cudaStream_t st) {
  const int G = a.n_q_heads / a.n_kv_heads;
  if (G >= 8) return launch_split<KV, D, 8>(a, st);
  if (G >= 4) return launch_split<KV, D, 4>(a, st);
  if (G >= 2) return launch_split<KV, D, 2>(a, st);
  return launch_split<KV, D, 1>(a, st);
}

template <typename KV>
cudaError_t launch_d(const DecodeArgs& a, cudaStream_t st) {
  return a.head_dim == 64 ? launch_g<KV, 64>(a, st) : launch_g<KV, 128>(a, st);
}

}  // namespace

size_t decode_scratch_bytes(int32_t batch, int32_t n_q_heads, int32_t head_dim, int32_t max_splits) {
  if (max_splits <= 1) return 0;
  return sizeof(float) * static_cast<size_t>(batch) * n_q_heads * max_splits * (head_dim + 2);
}

cudaError_t launch_decode(const DecodeArgs& a, cudaStream_t st) {
  if (a.kv.dtype == AIHOST_F32) return launch_d<float>(a, st);
  if (a.kv.dtype == AIHOST_F16) return launch_d<__half>(a, st);
  return launch_d<Q8Tag>(a, st);
}

cudaError_t launch_decode_combine(const DecodeArgs& a, cudaStream_t st) {
  if (a.max_splits <= 1) return cudaSuccess;
  if (a.head_dim == 64) decode_combine_kernel<64><<<dim3(a.n_q_heads, a.batch), 64, 0, st>>>(a);
  else decode_combine_kernel<128><<<dim3(a.n_q_heads, a.batch), 128, 0, st>>>(a);
  return cudaGetLastError();
}

cudaError_t launch_merge_partials(int32_t n_parts, int64_t rows, int32_t head_dim, int32_t dtype,
                                  const void* o_parts, const float* lse_parts, void* out, float* lse_out,
                                  cudaStream_t st) {
  const int threads = (head_dim + 31) / 32 * 32;
  if (dtype == AIHOST_F32)
    merge_partials_kernel<float><<<static_cast<unsigned>(rows), threads, 0, st>>>(
        n_parts, rows, head_dim, static_cast<const float*>(o_parts), lse_parts, static_cast<float*>(out), lse_out);
  else
    merge_partials_kernel<__half><<<static_cast<unsigned>(rows), threads, 0, st>>>(
        n_parts, rows, head_dim, static_cast<const __half*>(o_parts), lse_parts, static_cast<__half*>(out), lse_out);
  return cudaGetLastError();
}

}  // namespace aihost
