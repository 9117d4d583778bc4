// decode_mma.cu — split-K flash decoding for fp16 and GGUF Q8_0 caches on the tensor cores.
//
// Replaces FusedMHAGenerate (ComputeShaders.cs:656-733) for fp16 / Q8_0 KV caches. One CTA handles
// one (sequence, KV head, group of up to 16 Q heads, split of `chunk` cache rows):
//   producer    TMA: K and V tiles of 64 rows into a multi-stage shared-memory ring (no
//               multicast), completion on mbarriers. fp16 caches land as 128-byte swizzled fp16
//               tiles; Q8_0 caches land as raw 34-byte blocks, which four converter warps turn
//               into the same swizzled fp16 tiles (one cache row per thread);
//   warps 0-3   each takes 16 rows of every fp16 tile: S = Q K^T with m16n8k16 MMAs (the group's Q
//               heads are the 16 MMA rows, rotated by RoPE once per CTA and kept as A fragments
//               in registers), online softmax in the exp2 domain with quad-shuffle row
//               reductions, O += P V with P re-used from the S accumulators as A fragments;
//               the four warps' (max, sum, O) are merged through shared memory at the end.
// The per-split (max, sum, unnormalised O) go to the same scratch / combine kernel as the fp32
// path, or straight to the output when a sequence fits in one split.
// Decode moves ~2 bytes of cache per multiply-add pair and has only G <= 16 query rows per KV
// head, so it is bound by HBM bandwidth: the design goal is many bytes in flight per SM
// (ring depth x 2 x 64 x head_dim x 2 bytes) and few instructions per byte.
#include "common.cuh"
#include "kernels.h"
#include "rows.cuh"

namespace aihost {
namespace {

constexpr int kTileRows = 64;     // cache rows per pipeline stage
constexpr int kComputeWarps = 4;  // 16 rows of each tile per warp
constexpr int kThreads = (kComputeWarps + 1) * 32;
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct DecodeCfg {
  static constexpr int KB = D / 64;                         // 128-byte column blocks
  static constexpr int TILE_BYTES = KB * kTileRows * 128;   // one K or V tile
  static constexpr int NS = D == 64 ? 6 : 3;                // ring depth
  static constexpr int QROW = D + 8;                        // padded Q row (fp16 elements)
  static constexpr int K_OFF = 0;
  static constexpr int V_OFF = NS * TILE_BYTES;
  static constexpr int Q_OFF = 2 * NS * TILE_BYTES;
  static constexpr int Q_BYTES = 16 * QROW * 2;
  static constexpr int BAR_OFF = Q_OFF + Q_BYTES;
  static constexpr int SMEM = BAR_OFF + 128 + 1024;
  static_assert(NS * TILE_BYTES >= kComputeWarps * 16 * (D + 8 + 2) * 4, "merge buffer reuses the K ring");
};

__device__ __forceinline__ void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.x4.m8n8.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.x4.trans.m8n8.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}
__device__ __forceinline__ void mma16816(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ uint32_t pack_h2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}
// Transpose of an 8x8 matrix of 16-bit elements held one 32-bit pair per lane in the mma
// fragment layout (lane 4r + c holds row r, columns 2c and 2c + 1).
__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

// Shared-memory byte address of fp16 element (row, col) of a 64-row tile written by TMA with
// 128-byte swizzle (16-byte chunk index XOR row % 8; 64-column blocks of 64 * 128 bytes).
__device__ __forceinline__ uint32_t sw_addr(uint32_t tile, int row, int col) {
  return tile + (col >> 6) * (kTileRows * 128) + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4);
}

struct DecBars {
  uint64_t full[6], empty[6];
};
static_assert(sizeof(DecBars) <= 128, "decode_mma_kernel reserves 128 bytes for its barriers");

// The new token's K (warp 0, rotated) or V (warp 1) row of KV head kvh, written into cache row
// t the way the append kernel writes it, then made visible to this CTA's later TMA reads.
template <int D>
__device__ __forceinline__ void append_new_row(const DecodeArgs& p, int b, int kvh, int32_t t, int warp, int lane) {
  constexpr int E = D / 32;
  const bool is_k = warp == 0;
  const int64_t row = static_cast<int64_t>(b) * p.n_kv_heads + kvh;
  const int esz = p.new_dtype == AIHOST_F32 ? 4 : 2;
  const uint8_t* src = static_cast<const uint8_t*>(is_k ? p.k_new : p.v_new) + row * D * esz;
  float x[E];
  load_row_warp<E>(src, p.new_dtype, lane, x);
  if (is_k && p.rope_mode != AIHOST_ROPE_NONE)
    rope_row_warp<E>(x, lane, static_cast<float>(p.q_pos ? p.q_pos[b] : t), p.rope_mode, p.freqs);
  if (!kv_row_ok(p.kv, b, t)) {  // a paged cache's block table points outside the pool
    if (lane == 0) atomicOr(p.status, kStatusBadLength);
  } else {
    uint8_t* dst = static_cast<uint8_t*>(const_cast<void*>(is_k ? p.k_cache : p.v_cache)) + kv_row_offset(p.kv, b, t) +
                   static_cast<int64_t>(kvh) * p.kv.head_stride;
    store_row_warp<E>(x, lane, dst, p.kv.dtype);
  }
  asm volatile("fence.proxy.async.global;" ::: "memory");
}


// Output of one split (compute warps, after each warp has put its per-head (max, sum) at
// merge[(warp * 16 + head) * 2] and its unnormalised O row at o_s[(warp * 16 + head) * (D + 8)]):
// the four warps merged per head, then either the output (one split), or the split's partial
// and, when this split is the last of its (sequence, head group) to finish, the merged output.
template <int D>
__device__ __forceinline__ void decode_emit(const DecodeArgs& p, float* merge, int h0, int g_count, int b, int split,
                                            int n_splits) {
  constexpr int OP = D + 8;
  float* ml_s = merge;
  float* o_s = ml_s + kComputeWarps * 16 * 2;
  asm volatile("bar.sync 1, 128;" ::: "memory");
  for (int idx = threadIdx.x; idx < g_count * D; idx += kComputeWarps * 32) {
    const int g = idx / D, d = idx % D;
    float m = -INFINITY;
#pragma unroll
    for (int w = 0; w < kComputeWarps; ++w) m = fmaxf(m, ml_s[(w * 16 + g) * 2]);
    float l = 0.0f, acc = 0.0f;
#pragma unroll
    for (int w = 0; w < kComputeWarps; ++w) {
      const float wt = ex2_approx(ml_s[(w * 16 + g) * 2] - m);
      l = fmaf(ml_s[(w * 16 + g) * 2 + 1], wt, l);
      acc = fmaf(o_s[(w * 16 + g) * OP + d], wt, acc);
    }
    const int h = h0 + g;
    if (n_splits == 1) {
      const float v = acc / l;
      const int64_t oidx = (static_cast<int64_t>(b) * p.n_q_heads + h) * D + d;
      if (p.out_dtype == AIHOST_F32) static_cast<float*>(p.out)[oidx] = v;
      else static_cast<__half*>(p.out)[oidx] = __float2half_rn(v);
      if (p.lse && d == 0) p.lse[static_cast<int64_t>(b) * p.n_q_heads + h] = (m + log2f(l)) * kLn2;
    } else {
      const int64_t pidx = (static_cast<int64_t>(b) * p.n_q_heads + h) * p.max_splits + split;
      p.part_o[pidx * D + d] = acc;
      if (d == 0) {
        p.part_ml[pidx * 2] = m;
        p.part_ml[pidx * 2 + 1] = l;
      }
    }
  }
  if (n_splits == 1 || !p.counters) return;
  // ---- fused combine: the last split of this (sequence, head group) to finish merges them all
  __shared__ int s_last;
  __threadfence();
  asm volatile("bar.sync 1, 128;" ::: "memory");
  unsigned long long* counter = &p.counters[static_cast<int64_t>(b) * gridDim.y + blockIdx.y];
  if (threadIdx.x == 0) s_last = split_arrive(counter, p.epoch, n_splits, p.status);
  asm volatile("bar.sync 1, 128;" ::: "memory");
  if (!s_last) return;
  // every split of this call has arrived: reset the counter, so that a replay of the same launch
  // (a CUDA graph keeps its epoch argument) starts from zero again
  if (threadIdx.x == 0) atomicExch(counter, 0ull);
  __threadfence();
  // per-(head, split) weights 2^(m_s - m) / l first (one thread per head), then every output
  // element as a weighted sum of the splits' partial O, four columns per thread
  float* wts = ml_s;  // [16 heads][max_splits <= kMergeSplits], reusing the merge buffer
  constexpr int kMergeSplits = 64;
  const bool fits = p.max_splits <= kMergeSplits;
  if (fits && threadIdx.x < g_count) {
    const int64_t base = (static_cast<int64_t>(b) * p.n_q_heads + h0 + threadIdx.x) * p.max_splits;
    float m = -INFINITY;
    for (int sp = 0; sp < n_splits; ++sp) m = fmaxf(m, __ldcg(&p.part_ml[(base + sp) * 2]));
    float l = 0.0f;
    for (int sp = 0; sp < n_splits; ++sp) {
      const float w = exp2f(__ldcg(&p.part_ml[(base + sp) * 2]) - m);
      wts[threadIdx.x * kMergeSplits + sp] = w;
      l = fmaf(__ldcg(&p.part_ml[(base + sp) * 2 + 1]), w, l);
    }
    const float inv = 1.0f / l;
    for (int sp = 0; sp < n_splits; ++sp) wts[threadIdx.x * kMergeSplits + sp] *= inv;
    if (p.lse) p.lse[static_cast<int64_t>(b) * p.n_q_heads + h0 + threadIdx.x] = (m + log2f(l)) * kLn2;
  }
  asm volatile("bar.sync 1, 128;" ::: "memory");
  for (int idx = threadIdx.x; idx < g_count * (D / 4); idx += kComputeWarps * 32) {
    const int g = idx / (D / 4), d = (idx % (D / 4)) * 4;
    const int64_t base = (static_cast<int64_t>(b) * p.n_q_heads + h0 + g) * p.max_splits;
    float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
    if (fits) {
      for (int sp = 0; sp < n_splits; ++sp) {
        const float w = wts[g * kMergeSplits + sp];
        const float4 o4 = __ldcg(reinterpret_cast<const float4*>(&p.part_o[(base + sp) * D + d]));
        acc.x = fmaf(o4.x, w, acc.x);
        acc.y = fmaf(o4.y, w, acc.y);
        acc.z = fmaf(o4.z, w, acc.z);
        acc.w = fmaf(o4.w, w, acc.w);
      }
    } else {  // more splits than the weight table holds: weights recomputed per element
      float m = -INFINITY;
      for (int sp = 0; sp < n_splits; ++sp) m = fmaxf(m, __ldcg(&p.part_ml[(base + sp) * 2]));
      float l = 0.0f;
      for (int sp = 0; sp < n_splits; ++sp) {
        const float w = exp2f(__ldcg(&p.part_ml[(base + sp) * 2]) - m);
        l = fmaf(__ldcg(&p.part_ml[(base + sp) * 2 + 1]), w, l);
        const float4 o4 = __ldcg(reinterpret_cast<const float4*>(&p.part_o[(base + sp) * D + d]));
        acc.x = fmaf(o4.x, w, acc.x);
        acc.y = fmaf(o4.y, w, acc.y);
        acc.z = fmaf(o4.z, w, acc.z);
        acc.w = fmaf(o4.w, w, acc.w);
      }
      const float inv = 1.0f / l;
      acc.x *= inv;
      acc.y *= inv;
      acc.z *= inv;
      acc.w *= inv;
      if (p.lse && d == 0) p.lse[static_cast<int64_t>(b) * p.n_q_heads + h0 + g] = (m + log2f(l)) * kLn2;
    }
    const int64_t oidx = (static_cast<int64_t>(b) * p.n_q_heads + h0 + g) * D + d;
    if (p.out_dtype == AIHOST_F32) {
      *reinterpret_cast<float4*>(static_cast<float*>(p.out) + oidx) = acc;
    } else {
      const __half2 lo = __floats2half2_rn(acc.x, acc.y), hi = __floats2half2_rn(acc.z, acc.w);
      uint2 u;
      u.x = *reinterpret_cast<const uint32_t*>(&lo);
      u.y = *reinterpret_cast<const uint32_t*>(&hi);
      *reinterpret_cast<uint2*>(static_cast<__half*>(p.out) + oidx) = u;
    }
  }
}


// Compute-warp half of both kernels (warps 0-3): streams the fp16 K/V tiles of ring `full` /
// `empty` (NS stages of TILE_BYTES each at k_off / v_off), keeps (max, sum, O) per query row in
// registers, then merges the four warps through `merge` and writes the output or the split's
// partials. ZERO_V: rows past the split's end arrive as stale cache bytes and are zeroed here.
template <int D, int NS, bool ZERO_V>
__device__ __forceinline__ void decode_compute(const DecodeArgs& p, uint8_t* smem, int k_off, int v_off,
                                               uint64_t* full, uint64_t* empty, const __half* q_s, float* merge,
                                               int n, int n_tiles, int h0, int g_count, int b, int split,
                                               int n_splits) {
  constexpr int KB = D / 64;
  constexpr int TILE_BYTES = KB * kTileRows * 128;
  constexpr int QROW = D + 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t k_base = smem_u32(smem + k_off), v_base = smem_u32(smem + v_off);
  const int grp = lane >> 2, tig = lane & 3;
  // Q as A fragments: k-step kk covers dims [16kk, 16kk + 16)
  uint32_t qa[D / 16][4];
  {
    const uint32_t qb = smem_u32(q_s);
    const int mi = lane >> 3, r = lane & 7;
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk)
      ldsm_x4(qb + ((r + 8 * (mi & 1)) * QROW + kk * 16 + 8 * (mi >> 1)) * 2, qa[kk][0], qa[kk][1], qa[kk][2],
              qa[kk][3]);
  }
  const float sl2 = p.scale * kLog2e;
  float m_run[2] = {-1e30f, -1e30f}, l_run[2] = {0.0f, 0.0f};
  float o[D / 8][4];
#pragma unroll
  for (int nb = 0; nb < D / 8; ++nb) o[nb][0] = o[nb][1] = o[nb][2] = o[nb][3] = 0.0f;

  bool ok = true;
  for (int i = 0; i < n_tiles && ok; ++i) {
    const int s = i % NS;
    if (!mbar_wait(&full[s], (i / NS) & 1, p.status)) { ok = false; break; }
    const uint32_t kt = k_base + s * TILE_BYTES, vt = v_base + s * TILE_BYTES;
    const int r0 = warp * 16;  // this warp's 16 rows of the tile
    // ---- S = Q K^T for the warp's rows: two n8 blocks
    float sacc[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
    {
      const int mi = lane >> 3, r = lane & 7;
#pragma unroll
      for (int nb = 0; nb < 2; ++nb)
#pragma unroll
        for (int kk = 0; kk < D / 16; kk += 2) {
          uint32_t b0, b1, b2, b3;
          ldsm_x4(sw_addr(kt, r0 + nb * 8 + r, kk * 16 + 8 * mi), b0, b1, b2, b3);
          mma16816(sacc[nb], qa[kk][0], qa[kk][1], qa[kk][2], qa[kk][3], b0, b1);
          mma16816(sacc[nb], qa[kk + 1][0], qa[kk + 1][1], qa[kk + 1][2], qa[kk + 1][3], b2, b3);
        }
    }
    // ---- mask rows past the split's end, then the online softmax (rows grp and grp + 8)
    const int base_row = i * kTileRows + r0;
    float mt[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int nb = 0; nb < 2; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int row = base_row + nb * 8 + 2 * tig + (e & 1);
        float v = sacc[nb][e] * sl2;
        v = row < n ? v : -INFINITY;
        sacc[nb][e] = v;
        mt[e >> 1] = fmaxf(mt[e >> 1], v);
      }
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mt[h] = fmaxf(mt[h], __shfl_xor_sync(0xffffffffu, mt[h], 1));
      mt[h] = fmaxf(mt[h], __shfl_xor_sync(0xffffffffu, mt[h], 2));
    }
    float f[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float m_new = fmaxf(m_run[h], mt[h]);
      f[h] = ex2_approx(m_run[h] - m_new);
      m_run[h] = m_new;
      l_run[h] *= f[h];
    }
#pragma unroll
    for (int nb = 0; nb < D / 8; ++nb) {
      o[nb][0] *= f[0];
      o[nb][1] *= f[0];
      o[nb][2] *= f[1];
      o[nb][3] *= f[1];
    }
    float pv[2][4];
#pragma unroll
    for (int nb = 0; nb < 2; ++nb)
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        pv[nb][e] = ex2_approx(sacc[nb][e] - m_run[e >> 1]);
        l_run[e >> 1] += pv[nb][e];
      }
    const uint32_t pa0 = pack_h2(pv[0][0], pv[0][1]), pa1 = pack_h2(pv[0][2], pv[0][3]);
    const uint32_t pa2 = pack_h2(pv[1][0], pv[1][1]), pa3 = pack_h2(pv[1][2], pv[1][3]);
    // ---- rows past the split's end may hold stale bits (NaN patterns included); P is 0 there,
    // but 0 * NaN is NaN, so the warp zeroes its own V rows beyond n before reading them
    if (ZERO_V && base_row + 16 > n) {
      uint8_t* vrow0 = smem + v_off + s * TILE_BYTES;
      for (int c = lane; c < 16 * KB * 8; c += 32) {
        const int rr = c / (KB * 8), ch = c % (KB * 8);
        if (base_row + rr >= n)
          *reinterpret_cast<uint4*>(vrow0 + (ch >> 3) * (kTileRows * 128) + (r0 + rr) * 128 + (ch & 7) * 16) =
              make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
    }
    // ---- O += P V: V rows r0..r0+15 of the tile, all D columns (ldmatrix.trans gives B frags)
    {
      const int mi = lane >> 3, r = lane & 7;
#pragma unroll
      for (int nb = 0; nb < D / 8; nb += 2) {
        uint32_t b0, b1, b2, b3;
        ldsm_x4_t(sw_addr(vt, r0 + r + 8 * (mi & 1), nb * 8 + 8 * (mi >> 1)), b0, b1, b2, b3);
        mma16816(o[nb], pa0, pa1, pa2, pa3, b0, b1);
        mma16816(o[nb + 1], pa0, pa1, pa2, pa3, b2, b3);
      }
    }
    __syncwarp();
    if (ZERO_V && base_row + 16 > n) fence_proxy_async_smem();  // zeroed rows are rewritten by TMA later
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // ---- merge the four warps: row sums over the quad, then through shared memory
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 1);
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 2);
  }
  // all tiles consumed: `merge` reuses ring memory no producer can target any more
  asm volatile("bar.sync 1, 128;" ::: "memory");
  // O rows padded to D + 8 floats: a quad's float2 stores then cover all 32 banks per half-warp
  constexpr int OP = D + 8;
  float* ml_s = merge;                           // [4 warps][16 rows][2]
  float* o_s = ml_s + kComputeWarps * 16 * 2;    // [4 warps][16 rows][OP]
  if (tig == 0) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      ml_s[(warp * 16 + grp + 8 * h) * 2] = m_run[h];
      ml_s[(warp * 16 + grp + 8 * h) * 2 + 1] = l_run[h];
    }
  }
#pragma unroll
  for (int nb = 0; nb < D / 8; ++nb)
#pragma unroll
    for (int h = 0; h < 2; ++h)
      *reinterpret_cast<float2*>(&o_s[(warp * 16 + grp + 8 * h) * OP + nb * 8 + 2 * tig]) =
          make_float2(o[nb][2 * h], o[nb][2 * h + 1]);
  decode_emit<D>(p, merge, h0, g_count, b, split, n_splits);
}

// Transposed compute for a head group of at most 8 query heads (warps 0-3). The heads are the
// N = 8 columns of every m16n8k16 MMA instead of padded M = 16 rows: S^T = K Q^T (M = the warp's
// 16 cache rows) and O^T = V^T P^T (M = 16 head dimensions), which halves the MMAs and the O
// registers. P^T reaches the B-fragment layout of the P.V product through two movmatrix
// transposes of the S^T accumulators.
template <int D, int NS, bool ZERO_V>
__device__ __forceinline__ void decode_compute_t(const DecodeArgs& p, uint8_t* smem, int k_off, int v_off,
                                                 uint64_t* full, uint64_t* empty, const __half* q_s, float* merge,
                                                 int n, int n_tiles, int h0, int g_count, int b, int split,
                                                 int n_splits) {
  constexpr int KB = D / 64;
  constexpr int TILE_BYTES = KB * kTileRows * 128;
  constexpr int QROW = D + 8;
  constexpr int OP = D + 8;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t k_base = smem_u32(smem + k_off), v_base = smem_u32(smem + v_off);
  const int grp = lane >> 2, tig = lane & 3;
  const int mi = lane >> 3, r8 = lane & 7;
  // Q^T as B fragments (k = head dims, n = heads 0-7): qb[kk] covers dims [16kk, 16kk + 16)
  uint32_t qb[D / 16][2];
  {
    const uint32_t qbase = smem_u32(q_s);
#pragma unroll
    for (int kk = 0; kk < D / 16; kk += 2)
      ldsm_x4(qbase + (r8 * QROW + kk * 16 + 8 * mi) * 2, qb[kk][0], qb[kk][1], qb[kk + 1][0], qb[kk + 1][1]);
  }
  const float sl2 = p.scale * kLog2e;
  // per thread: heads 2tig and 2tig + 1
  float m_run[2] = {-1e30f, -1e30f}, l_run[2] = {0.0f, 0.0f};
  float o[D / 16][4];  // O^T: dims 16mt + grp (+8), heads 2tig (+1)
#pragma unroll
  for (int mt = 0; mt < D / 16; ++mt) o[mt][0] = o[mt][1] = o[mt][2] = o[mt][3] = 0.0f;

  bool ok = true;
  for (int i = 0; i < n_tiles && ok; ++i) {
    const int s = i % NS;
    if (!mbar_wait(&full[s], (i / NS) & 1, p.status)) { ok = false; break; }
    const uint32_t kt = k_base + s * TILE_BYTES, vt = v_base + s * TILE_BYTES;
    const int r0 = warp * 16;  // this warp's 16 rows of the tile
    // ---- S^T = K Q^T: rows r0..r0+15 of the tile (keys) x 8 heads
    float sacc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int kk = 0; kk < D / 16; ++kk) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4(sw_addr(kt, r0 + r8 + 8 * (mi & 1), kk * 16 + 8 * (mi >> 1)), a0, a1, a2, a3);
      mma16816(sacc, a0, a1, a2, a3, qb[kk][0], qb[kk][1]);
    }
    // ---- mask rows past the split's end; online softmax per head (column) over the warp's rows
    const int base_row = i * kTileRows + r0;
    const bool lo_ok = base_row + grp < n, hi_ok = base_row + grp + 8 < n;
    const float s0 = lo_ok ? sacc[0] * sl2 : -INFINITY, s1 = lo_ok ? sacc[1] * sl2 : -INFINITY;
    const float s2 = hi_ok ? sacc[2] * sl2 : -INFINITY, s3 = hi_ok ? sacc[3] * sl2 : -INFINITY;
    float mt[2] = {fmaxf(s0, s2), fmaxf(s1, s3)};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mt[h] = fmaxf(mt[h], __shfl_xor_sync(0xffffffffu, mt[h], 4));
      mt[h] = fmaxf(mt[h], __shfl_xor_sync(0xffffffffu, mt[h], 8));
      mt[h] = fmaxf(mt[h], __shfl_xor_sync(0xffffffffu, mt[h], 16));
    }
    float f[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float m_new = fmaxf(m_run[h], mt[h]);
      f[h] = ex2_approx(m_run[h] - m_new);
      m_run[h] = m_new;
      l_run[h] *= f[h];
    }
#pragma unroll
    for (int m2 = 0; m2 < D / 16; ++m2) {
      o[m2][0] *= f[0];
      o[m2][1] *= f[1];
      o[m2][2] *= f[0];
      o[m2][3] *= f[1];
    }
    const float p0 = ex2_approx(s0 - m_run[0]), p1 = ex2_approx(s1 - m_run[1]);
    const float p2 = ex2_approx(s2 - m_run[0]), p3 = ex2_approx(s3 - m_run[1]);
    l_run[0] += p0 + p2;
    l_run[1] += p1 + p3;
    // P^T as B fragments: transpose the (rows x heads) 8x8 blocks into (heads x rows) order
    const uint32_t pb0 = movmatrix_trans(pack_h2(p0, p1)), pb1 = movmatrix_trans(pack_h2(p2, p3));
    // ---- rows past the split's end may hold stale bits (NaN patterns included); P is 0 there,
    // but 0 * NaN is NaN, so the warp zeroes its own V rows beyond n before reading them
    if (ZERO_V && base_row + 16 > n) {
      uint8_t* vrow0 = smem + v_off + s * TILE_BYTES;
      for (int c = lane; c < 16 * KB * 8; c += 32) {
        const int rr = c / (KB * 8), ch = c % (KB * 8);
        if (base_row + rr >= n)
          *reinterpret_cast<uint4*>(vrow0 + (ch >> 3) * (kTileRows * 128) + (r0 + rr) * 128 + (ch & 7) * 16) =
              make_uint4(0, 0, 0, 0);
      }
      __syncwarp();
    }
    // ---- O^T += V^T P^T: dims in 16-row blocks (ldmatrix.trans of V gives the A fragments)
#pragma unroll
    for (int m2 = 0; m2 < D / 16; ++m2) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4_t(sw_addr(vt, r0 + r8 + 8 * (mi >> 1), m2 * 16 + 8 * (mi & 1)), a0, a1, a2, a3);
      mma16816(o[m2], a0, a1, a2, a3, pb0, pb1);
    }
    __syncwarp();
    if (ZERO_V && base_row + 16 > n) fence_proxy_async_smem();  // zeroed rows are rewritten by TMA later
    if (lane == 0) mbar_arrive(&empty[s]);
  }

  // ---- per-head sums over the warp's rows (lanes sharing tig), then through shared memory
#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 4);
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 8);
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 16);
  }
  // all tiles consumed: `merge` reuses ring memory no producer can target any more
  asm volatile("bar.sync 1, 128;" ::: "memory");
  float* ml_s = merge;
  float* o_s = ml_s + kComputeWarps * 16 * 2;
  if (grp == 0) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      ml_s[(warp * 16 + 2 * tig + h) * 2] = m_run[h];
      ml_s[(warp * 16 + 2 * tig + h) * 2 + 1] = l_run[h];
    }
  }
#pragma unroll
  for (int m2 = 0; m2 < D / 16; ++m2)
#pragma unroll
    for (int e = 0; e < 4; ++e)
      o_s[(warp * 16 + 2 * tig + (e & 1)) * OP + m2 * 16 + grp + 8 * (e >> 1)] = o[m2][e];
  decode_emit<D>(p, merge, h0, g_count, b, split, n_splits);
}

// Q rows of the group, rotated at the new token's position, as fp16 rows of QROW elements
// (rows >= g_count zero). All `nthreads` threads of the CTA take part.
template <int D, int ROWS = 16>
__device__ __forceinline__ void load_q_rows(const DecodeArgs& p, __half* q_s, int b, int h0, int g_count,
                                            int32_t start, int nthreads) {
  constexpr int QROW = D + 8;
  const float pos = static_cast<float>(p.q_pos ? p.q_pos[b] : start + p.rope_pos_offset);
  for (int idx = threadIdx.x; idx < ROWS * (D / 2); idx += nthreads) {
    const int g = idx / (D / 2), pair = idx % (D / 2);
    const int i1 = p.rope_mode == AIHOST_ROPE_NEOX ? pair : 2 * pair;
    const int i2 = p.rope_mode == AIHOST_ROPE_NEOX ? pair + D / 2 : 2 * pair + 1;
    float x1 = 0.0f, x2 = 0.0f;
    if (g < g_count) {
      const int64_t qoff = (static_cast<int64_t>(b) * p.n_q_heads + h0 + g) * D;
      if (p.q_dtype == AIHOST_F32) {
        x1 = static_cast<const float*>(p.q)[qoff + i1];
        x2 = static_cast<const float*>(p.q)[qoff + i2];
      } else {
        x1 = __half2float(static_cast<const __half*>(p.q)[qoff + i1]);
        x2 = __half2float(static_cast<const __half*>(p.q)[qoff + i2]);
      }
      if (p.rope_mode != AIHOST_ROPE_NONE) {
        float sn, cs;
        sincosf(__fmul_rn(pos, p.freqs.f[pair]), &sn, &cs);
        const float r1 = __fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn));
        const float r2 = __fadd_rn(__fmul_rn(x1, sn), __fmul_rn(x2, cs));
        x1 = r1;
        x2 = r2;
      }
    }
    q_s[g * QROW + i1] = __float2half_rn(x1);
    q_s[g * QROW + i2] = __float2half_rn(x2);
  }
}

// TR: the transposed compute for head groups of at most 8 query heads.
template <int D, bool TR>
__global__ void __launch_bounds__(kThreads) decode_mma_kernel(const __grid_constant__ DecodeMmaArgs a) {
  using C = DecodeCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  DecBars& bar = *reinterpret_cast<DecBars*>(smem + C::BAR_OFF);
  __half* q_s = reinterpret_cast<__half*>(smem + C::Q_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const DecodeArgs& p = a.base;
  const int split = blockIdx.x;
  const int G = p.n_q_heads / p.n_kv_heads;
  const int n_sub = (G + 15) / 16;
  const int kvh = blockIdx.y / n_sub, sub = blockIdx.y % n_sub;
  const int b = blockIdx.z;
  const int g_count = min(16, G - sub * 16);
  const int h0 = kvh * G + sub * 16;
  const int32_t start = p.seq_len ? p.seq_len[b] : p.start_scalar;
  const int32_t Lk = start + p.len_offset;
  if (Lk > p.kv.capacity || Lk < 1) {
    if (threadIdx.x == 0 && split == 0 && blockIdx.y == 0) atomicOr(p.status, kStatusBadLength);
    return;
  }
  const int32_t t0 = split * p.chunk;
  if (t0 >= Lk) return;
  const int32_t n = min(p.chunk, Lk - t0);
  const int n_tiles = (n + kTileRows - 1) / kTileRows;
  const int n_splits = (Lk + p.chunk - 1) / p.chunk;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NS; ++i) {
      mbar_init(&bar.full[i], 1);
      mbar_init(&bar.empty[i], kComputeWarps);
    }
    fence_mbar_init();
  }
  // the last split's CTA writes the new token's rows before any TMA reads them
  if (p.fuse_append && sub == 0 && t0 + p.chunk >= Lk && warp < 2) append_new_row<D>(p, b, kvh, Lk - 1, warp, lane);
  load_q_rows<D>(p, q_s, b, h0, g_count, start, kThreads);
  __syncthreads();

  if (warp == kComputeWarps) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&a.k_map);
      tma_prefetch_desc(&a.v_map);
      for (int i = 0; i < n_tiles; ++i) {
        const int s = i % C::NS;
        if (!mbar_wait(&bar.empty[s], ((i / C::NS) & 1) ^ 1, p.status)) break;
        mbar_arrive_expect_tx(&bar.full[s], 2 * C::TILE_BYTES);
        // a paged cache keeps 64-row tiles inside a page: pool row and sequence coordinate 0
        const int row = kv_phys_row(p.kv, b, t0 + i * kTileRows), bc = p.kv.block_table ? 0 : b;
        for (int kb = 0; kb < C::KB; ++kb) {
          tma_load_4d(smem + C::K_OFF + s * C::TILE_BYTES + kb * kTileRows * 128, &a.k_map, &bar.full[s], kb * 64,
                      kvh, row, bc);
          tma_load_4d(smem + C::V_OFF + s * C::TILE_BYTES + kb * kTileRows * 128, &a.v_map, &bar.full[s], kb * 64,
                      kvh, row, bc);
        }
      }
    }
    return;
  }
  if constexpr (TR)
    decode_compute_t<D, C::NS, true>(p, smem, C::K_OFF, C::V_OFF, bar.full, bar.empty, q_s,
                                     reinterpret_cast<float*>(smem + C::K_OFF), n, n_tiles, h0, g_count, b, split,
                                     n_splits);
  else
    decode_compute<D, C::NS, true>(p, smem, C::K_OFF, C::V_OFF, bar.full, bar.empty, q_s,
                                   reinterpret_cast<float*>(smem + C::K_OFF), n, n_tiles, h0, g_count, b, split,
                                   n_splits);
}

// ------------------------------------------------------------------ GGUF Q8_0 caches
// Warps 0-3 compute (as above), warps 4-7 convert; the first converter thread also issues the
// TMA loads (256 threads, so two CTAs per SM keep 128 registers per thread).
// TMA reads each cache row's head slice as a box of 32-bit words that starts at the 16-byte
// boundary at or below the slice (GGUF blocks are only 2-byte aligned); the slice then begins
// `off` bytes into every raw tile row. The box is as narrow as the head offsets allow: with the
// default 136-byte heads (d = 128) it is 144 bytes (68-byte heads, d = 64: 80 bytes), an odd
// number of 16-byte units, so a quarter-warp reading 16 bytes from each of 8 consecutive rows
// touches 8 distinct bank groups.
// A converter thread owns one row of the K or V tile: it reads the raw row with 16-byte loads,
// realigns the 2-byte-aligned blocks with byte permutes, turns each int8 exactly into fp16
// (exponent 0x64 over q + 128, minus 1152), multiplies by the block's fp16 scale (one rounding:
// fp16(d * q), the value an fp32 dequantise-then-round gives) and stores the row swizzled, so
// the compute warps read the same fp16 tiles as for an fp16 cache. Rows past the split's end are
// written as zeros.
constexpr int kQ8ConvWarps = 4;
constexpr int kQ8Threads = (kComputeWarps + kQ8ConvWarps) * 32;

template <int D>
struct Q8Cfg {
  static constexpr int NB = D / 32;                   // blocks per head row
  static constexpr int HEAD_WORDS = NB * 34 / 4;      // 17 (D=64) or 34 (D=128) words
  // box: the head slice plus up to 2 (d = 128) or 3 (d = 64) words of start offset, which
  // covers every head of the default GGUF layout (136- / 68-byte heads).
  static constexpr int BOX_WORDS = (HEAD_WORDS + 2 + 3) / 4 * 4;
  static constexpr int ROW_BYTES = BOX_WORDS * 4;
  static constexpr int RAW_TILE = kTileRows * ROW_BYTES;   // one raw K or V tile
  static constexpr int F_TILE = (D / 64) * kTileRows * 128;  // one fp16 K or V tile
  static constexpr int NSR = D == 64 ? 4 : 2;              // raw ring depth
  static constexpr int NSF = D == 64 ? 4 : 2;              // fp16 ring depth
  static constexpr int QROW = D + 8;
  static constexpr int RAW_OFF = 0;                        // K raw [NSR], then V raw [NSR]
  static constexpr int F_OFF = (2 * NSR * RAW_TILE + 1023) / 1024 * 1024;  // K fp16 [NSF], V fp16
  static constexpr int Q_OFF = F_OFF + 2 * NSF * F_TILE;
  static constexpr int Q_BYTES = 16 * QROW * 2;
  static constexpr int BAR_OFF = Q_OFF + Q_BYTES;
  static constexpr int SMEM = BAR_OFF + 256 + 1024;  // barriers, then alignment slack
  static constexpr int MERGE_BYTES = kComputeWarps * 16 * (D + 8 + 2) * 4;
  static_assert(2 * NSF * F_TILE >= MERGE_BYTES, "merge buffer reuses the fp16 rings");
  static_assert(NSR <= 4 && NSF <= 4, "barrier arrays hold four stages");
};

struct Q8Bars {
  uint64_t raw_full[4], raw_empty[4], f_full[4], f_empty[4];
  uint64_t appended;  // decode_q8k_kernel: the new token's rows are in the cache
};
static_assert(sizeof(Q8Bars) <= 256, "Q8_0 kernels reserve 256 bytes for their barriers");

// Converts one raw row (words w, head slice starting OFFW words in) into 16-byte fp16 chunks
// of the swizzled tile row `row` at `tile`.
template <int D, int OFFW>
__device__ __forceinline__ void q8_row_to_f16(const uint32_t (&w)[Q8Cfg<D>::BOX_WORDS], uint8_t* tile, int row) {
  const __half2 k1152 = __floats2half2_rn(1152.0f, 1152.0f);
#pragma unroll
  for (int blk = 0; blk < D / 32; ++blk) {
    constexpr int kOff = 4 * OFFW;
    const int b0 = kOff + 34 * blk;  // byte offset of the block's scale (even)
    const uint32_t sw = w[b0 >> 2] >> ((b0 & 3) * 8);
    const __half2 d2 = __half2half2(__ushort_as_half(static_cast<unsigned short>(sw & 0xffffu)));
    uint32_t hv[16];
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const int qb = b0 + 2 + 4 * j;  // bytes of dims 4j..4j+3 of the block
      // (the clamp only keeps the index of the unused operand inside the array)
      const int hi = (qb >> 2) + 1 < Q8Cfg<D>::BOX_WORDS ? (qb >> 2) + 1 : (qb >> 2);
      const uint32_t q = (qb & 3) == 0 ? w[qb >> 2] : __byte_perm(w[qb >> 2], w[hi], 0x5432);
      const uint32_t x = q ^ 0x80808080u;
      const uint32_t e01 = __byte_perm(x, 0x64646464u, 0x4140);
      const uint32_t e23 = __byte_perm(x, 0x64646464u, 0x4342);
      const __half2 h01 = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&e01), k1152), d2);
      const __half2 h23 = __hmul2(__hsub2(*reinterpret_cast<const __half2*>(&e23), k1152), d2);
      hv[2 * j] = *reinterpret_cast<const uint32_t*>(&h01);
      hv[2 * j + 1] = *reinterpret_cast<const uint32_t*>(&h23);
    }
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const int col = blk * 32 + 8 * c;
      uint8_t* dst = tile + (col >> 6) * (kTileRows * 128) + row * 128 + ((((col & 63) >> 3) ^ (row & 7)) << 4);
      *reinterpret_cast<uint4*>(dst) = make_uint4(hv[4 * c], hv[4 * c + 1], hv[4 * c + 2], hv[4 * c + 3]);
    }
  }
}

template <int D, bool TR>
__global__ void __launch_bounds__(kQ8Threads, 2) decode_q8_kernel(const __grid_constant__ DecodeMmaArgs a) {
  using C = Q8Cfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Q8Bars& bar = *reinterpret_cast<Q8Bars*>(smem + C::BAR_OFF);
  __half* q_s = reinterpret_cast<__half*>(smem + C::Q_OFF);

  const int warp = threadIdx.x >> 5;
  const DecodeArgs& p = a.base;
  const int split = blockIdx.x;
  const int G = p.n_q_heads / p.n_kv_heads;
  const int n_sub = (G + 15) / 16;
  const int kvh = blockIdx.y / n_sub, sub = blockIdx.y % n_sub;
  const int b = blockIdx.z;
  const int g_count = min(16, G - sub * 16);
  const int h0 = kvh * G + sub * 16;
  const int32_t start = p.seq_len ? p.seq_len[b] : p.start_scalar;
  const int32_t Lk = start + p.len_offset;
  if (Lk > p.kv.capacity || Lk < 1) {
    if (threadIdx.x == 0 && split == 0 && blockIdx.y == 0) atomicOr(p.status, kStatusBadLength);
    return;
  }
  const int32_t t0 = split * p.chunk;
  if (t0 >= Lk) return;
  const int32_t n = min(p.chunk, Lk - t0);
  const int n_tiles = (n + kTileRows - 1) / kTileRows;
  const int n_splits = (Lk + p.chunk - 1) / p.chunk;
  const int head_word = static_cast<int>(kvh * (p.kv.head_stride / 4));
  const int box_x = head_word & ~3;
  const int off_words = head_word - box_x;  // the head slice starts this many words into a row

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NSR; ++i) {
      mbar_init(&bar.raw_full[i], 1);
      mbar_init(&bar.raw_empty[i], kQ8ConvWarps * 32);
    }
    for (int i = 0; i < C::NSF; ++i) {
      mbar_init(&bar.f_full[i], kQ8ConvWarps * 32);
      mbar_init(&bar.f_empty[i], kComputeWarps);
    }
    fence_mbar_init();
  }
  // the last split's CTA writes the new token's rows before any TMA reads them
  if (p.fuse_append && sub == 0 && t0 + p.chunk >= Lk && warp < 2)
    append_new_row<D>(p, b, kvh, Lk - 1, warp, threadIdx.x & 31);
  load_q_rows<D>(p, q_s, b, h0, g_count, start, kQ8Threads);
  __syncthreads();

  if (warp >= kComputeWarps) {
    // ------------------------------------------------------------------ converters
    const int ct = threadIdx.x - kComputeWarps * 32;  // 0..127: K rows 0-63, V rows 0-63
    const int is_v = ct >> 6, row = ct & 63;
    const bool issuer = ct == 0;
    // TMA of tile i into raw slot i % NSR, once every converter has read the slot's last tile
    auto issue = [&](int i) -> bool {
      const int s = i % C::NSR;
      if (!mbar_wait(&bar.raw_empty[s], ((i / C::NSR) & 1) ^ 1, p.status)) return false;
      mbar_arrive_expect_tx(&bar.raw_full[s], 2 * C::RAW_TILE);  // bytes the two boxes deliver
      const int r = kv_phys_row(p.kv, b, t0 + i * kTileRows), bc = p.kv.block_table ? 0 : b;  // paged: pool row
      tma_load_4d(smem + C::RAW_OFF + s * C::RAW_TILE, &a.k_map, &bar.raw_full[s], box_x, r, bc, 0);
      tma_load_4d(smem + C::RAW_OFF + (C::NSR + s) * C::RAW_TILE, &a.v_map, &bar.raw_full[s], box_x, r, bc, 0);
      return true;
    };
    bool feed = issuer;
    if (issuer) {
      tma_prefetch_desc(&a.k_map);
      tma_prefetch_desc(&a.v_map);
      for (int i = 0; feed && i < C::NSR && i < n_tiles; ++i) feed = issue(i);
    }
    for (int i = 0; i < n_tiles; ++i) {
      const int sr = i % C::NSR, sf = i % C::NSF;
      if (!mbar_wait(&bar.raw_full[sr], (i / C::NSR) & 1, p.status)) break;
      uint32_t w[C::BOX_WORDS];
      const uint4* src =
          reinterpret_cast<const uint4*>(smem + C::RAW_OFF + (is_v * C::NSR + sr) * C::RAW_TILE + row * C::ROW_BYTES);
#pragma unroll
      for (int c = 0; c < C::BOX_WORDS / 4; ++c) {
        const uint4 v = src[c];
        w[4 * c] = v.x;
        w[4 * c + 1] = v.y;
        w[4 * c + 2] = v.z;
        w[4 * c + 3] = v.w;
      }
      mbar_arrive(&bar.raw_empty[sr]);
      if (feed && i + C::NSR < n_tiles) feed = issue(i + C::NSR);
      if (!mbar_wait(&bar.f_empty[sf], ((i / C::NSF) & 1) ^ 1, p.status)) break;
      uint8_t* tile = smem + C::F_OFF + (is_v * C::NSF + sf) * C::F_TILE;
      if (i * kTileRows + row < n) {
        if constexpr (D == 128) {
          if (off_words == 0) q8_row_to_f16<D, 0>(w, tile, row);
          else q8_row_to_f16<D, 2>(w, tile, row);
        } else {
          switch (off_words) {
            case 0: q8_row_to_f16<D, 0>(w, tile, row); break;
            case 1: q8_row_to_f16<D, 1>(w, tile, row); break;
            case 2: q8_row_to_f16<D, 2>(w, tile, row); break;
            default: q8_row_to_f16<D, 3>(w, tile, row); break;
          }
        }
      } else {
#pragma unroll
        for (int c = 0; c < D / 8; ++c)
          *reinterpret_cast<uint4*>(tile + (c >> 3) * (kTileRows * 128) + row * 128 + (((c & 7) ^ (row & 7)) << 4)) =
              make_uint4(0, 0, 0, 0);
      }
      mbar_arrive(&bar.f_full[sf]);
    }
    return;
  }
  if constexpr (TR)
    decode_compute_t<D, C::NSF, false>(p, smem, C::F_OFF, C::F_OFF + C::NSF * C::F_TILE, bar.f_full, bar.f_empty,
                                       q_s, reinterpret_cast<float*>(smem + C::F_OFF), n, n_tiles, h0, g_count, b,
                                       split, n_splits);
  else
    decode_compute<D, C::NSF, false>(p, smem, C::F_OFF, C::F_OFF + C::NSF * C::F_TILE, bar.f_full, bar.f_empty,
                                     q_s, reinterpret_cast<float*>(smem + C::F_OFF), n, n_tiles, h0, g_count, b,
                                     split, n_splits);
}

// ------------------------------------------------------------------ Q8_0, head groups of <= 8
// K straight from the raw tiles: the compute warps turn each 2-byte pair of int8 into an exact
// fp16 pair in registers (the A fragments of S^T = K Q^T), keep one fp32 accumulator per
// 32-element block and apply each row's fp16 block scale in fp32 (exactly the dequantise-then-
// dot sum, up to fp32 rounding). Only V, whose A fragments need a transpose, goes through the
// fp16 tiles, written by two converter warps (one V row per thread). A producer warp issues
// the TMA loads (a raw slot is free once the compute warps have read its K and the converters
// its V). The freed shared memory holds a 4-deep raw ring.
constexpr int kQ8kConvWarps = 2;
constexpr int kQ8kThreads = (kComputeWarps + kQ8kConvWarps + 1) * 32;

template <int D>
struct Q8kCfg {
  using B = Q8Cfg<D>;
  static constexpr int NSR = 4;                               // raw K+V ring depth
  static constexpr int NSF = 2;                               // fp16 V ring depth
  static constexpr int RAW_OFF = 0;                           // K raw [NSR], then V raw [NSR]
  static constexpr int F_OFF = (2 * NSR * B::RAW_TILE + 1023) / 1024 * 1024;  // V fp16 [NSF]
  static constexpr int Q_OFF = F_OFF + NSF * B::F_TILE;
  static constexpr int BAR_OFF = Q_OFF + B::Q_BYTES;
  static constexpr int SMEM = BAR_OFF + 256 + 1024;  // barriers, then alignment slack
  static_assert(2 * NSR * B::RAW_TILE >= B::MERGE_BYTES, "merge buffer reuses the raw ring");
};

template <int D>
__global__ void __launch_bounds__(kQ8kThreads, 2) decode_q8k_kernel(const __grid_constant__ DecodeMmaArgs a) {
  using C = Q8kCfg<D>;
  using B = Q8Cfg<D>;
  constexpr int ROW = B::ROW_BYTES;
  constexpr int OP = D + 8;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Q8Bars& bar = *reinterpret_cast<Q8Bars*>(smem + C::BAR_OFF);
  __half* q_s = reinterpret_cast<__half*>(smem + C::Q_OFF);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const DecodeArgs& p = a.base;
  const int split = blockIdx.x;
  const int G = p.n_q_heads / p.n_kv_heads;
  const int kvh = blockIdx.y;  // one head group per KV head (G <= 8)
  const int b = blockIdx.z;
  const int g_count = G;
  const int h0 = kvh * G;
  const int32_t start = p.seq_len ? p.seq_len[b] : p.start_scalar;
  const int32_t Lk = start + p.len_offset;
  if (Lk > p.kv.capacity || Lk < 1) {
    if (threadIdx.x == 0 && split == 0 && blockIdx.y == 0) atomicOr(p.status, kStatusBadLength);
    return;
  }
  const int32_t t0 = split * p.chunk;
  if (t0 >= Lk) return;
  const int32_t n = min(p.chunk, Lk - t0);
  const int n_tiles = (n + kTileRows - 1) / kTileRows;
  const int n_splits = (Lk + p.chunk - 1) / p.chunk;
  const int head_word = static_cast<int>(kvh * (p.kv.head_stride / 4));
  const int box_x = head_word & ~3;
  const int off = (head_word - box_x) * 4;  // byte offset of the head slice in a raw row

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NSR; ++i) {
      mbar_init(&bar.raw_full[i], 1);
      mbar_init(&bar.raw_empty[i], kQ8kConvWarps * 32 + kComputeWarps);  // V rows read + K reads done
    }
    for (int i = 0; i < C::NSF; ++i) {
      mbar_init(&bar.f_full[i], kQ8kConvWarps * 32);
      mbar_init(&bar.f_empty[i], kComputeWarps);
    }
    mbar_init(&bar.appended, 64);
    fence_mbar_init();
  }
  __syncthreads();
  // The producer starts streaming at once; the compute warps rotate Q meanwhile. The last
  // split's CTA writes the new token's rows first (warps 0 and 1); the producer waits for them
  // only before the one tile that holds that row.
  const bool appends = p.fuse_append && t0 + p.chunk >= Lk;
  if (appends && warp < 2) {
    append_new_row<D>(p, b, kvh, Lk - 1, warp, lane);
    mbar_arrive(&bar.appended);
  }

  if (warp == kComputeWarps + kQ8kConvWarps) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&a.k_map);
      tma_prefetch_desc(&a.v_map);
      for (int i = 0; i < n_tiles; ++i) {
        const int s = i % C::NSR;
        if (appends && i == (Lk - 1 - t0) / kTileRows && !mbar_wait(&bar.appended, 0, p.status)) break;
        if (!mbar_wait(&bar.raw_empty[s], ((i / C::NSR) & 1) ^ 1, p.status)) break;
        mbar_arrive_expect_tx(&bar.raw_full[s], 2 * B::RAW_TILE);  // bytes the two boxes deliver
        const int r = kv_phys_row(p.kv, b, t0 + i * kTileRows), bc = p.kv.block_table ? 0 : b;  // paged: pool row
        tma_load_4d(smem + C::RAW_OFF + s * B::RAW_TILE, &a.k_map, &bar.raw_full[s], box_x, r, bc, 0);
        tma_load_4d(smem + C::RAW_OFF + (C::NSR + s) * B::RAW_TILE, &a.v_map, &bar.raw_full[s], box_x, r, bc, 0);
      }
    }
    return;
  }
  if (warp >= kComputeWarps) {
    // ------------------------------------------------------------------ V converters
    const int row = threadIdx.x - kComputeWarps * 32;  // 0..63
    const int off_words = off / 4;
    for (int i = 0; i < n_tiles; ++i) {
      const int sr = i % C::NSR, sf = i % C::NSF;
      if (!mbar_wait(&bar.raw_full[sr], (i / C::NSR) & 1, p.status)) break;
      uint32_t w[B::BOX_WORDS];
      const uint4* src = reinterpret_cast<const uint4*>(smem + C::RAW_OFF + (C::NSR + sr) * B::RAW_TILE + row * ROW);
#pragma unroll
      for (int c = 0; c < B::BOX_WORDS / 4; ++c) {
        const uint4 v = src[c];
        w[4 * c] = v.x;
        w[4 * c + 1] = v.y;
        w[4 * c + 2] = v.z;
        w[4 * c + 3] = v.w;
      }
      mbar_arrive(&bar.raw_empty[sr]);
      if (!mbar_wait(&bar.f_empty[sf], ((i / C::NSF) & 1) ^ 1, p.status)) break;
      uint8_t* tile = smem + C::F_OFF + sf * B::F_TILE;
      if (i * kTileRows + row < n) {
        if constexpr (D == 128) {
          if (off_words == 0) q8_row_to_f16<D, 0>(w, tile, row);
          else q8_row_to_f16<D, 2>(w, tile, row);
        } else {
          switch (off_words) {
            case 0: q8_row_to_f16<D, 0>(w, tile, row); break;
            case 1: q8_row_to_f16<D, 1>(w, tile, row); break;
            case 2: q8_row_to_f16<D, 2>(w, tile, row); break;
            default: q8_row_to_f16<D, 3>(w, tile, row); break;
          }
        }
      } else {  // rows past the split's end: zeros (their stale bytes could decode to NaN)
#pragma unroll
        for (int c = 0; c < D / 8; ++c)
          *reinterpret_cast<uint4*>(tile + (c >> 3) * (kTileRows * 128) + row * 128 + (((c & 7) ^ (row & 7)) << 4)) =
              make_uint4(0, 0, 0, 0);
      }
      mbar_arrive(&bar.f_full[sf]);
    }
    return;
  }

  // ------------------------------------------------------------------ compute warps
  load_q_rows<D>(p, q_s, b, h0, g_count, start, kComputeWarps * 32);
  asm volatile("bar.sync 1, 128;" ::: "memory");
  constexpr int QROW = D + 8;
  const int grp = lane >> 2, tig = lane & 3;
  const int mi = lane >> 3, r8 = lane & 7;
  uint32_t qb[D / 16][2];  // Q^T as B fragments, as in decode_compute_t
  {
    const uint32_t qbase = smem_u32(q_s);
#pragma unroll
    for (int kk = 0; kk < D / 16; kk += 2)
      ldsm_x4(qbase + (r8 * QROW + kk * 16 + 8 * mi) * 2, qb[kk][0], qb[kk][1], qb[kk + 1][0], qb[kk + 1][1]);
  }
  const __half2 k1152 = __floats2half2_rn(1152.0f, 1152.0f);
  auto i8pair = [&](const uint8_t* p2) -> uint32_t {  // two int8 (2-byte aligned) -> exact fp16 pair
    const uint32_t x = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(p2)) ^ 0x8080u;
    const uint32_t e = __byte_perm(x, 0x64646464u, 0x4140);
    const __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&e), k1152);
    return *reinterpret_cast<const uint32_t*>(&h);
  };
  const float sl2 = p.scale * kLog2e;
  float m_run[2] = {-1e30f, -1e30f}, l_run[2] = {0.0f, 0.0f};
  float o[D / 16][4];
#pragma unroll
  for (int m2 = 0; m2 < D / 16; ++m2) o[m2][0] = o[m2][1] = o[m2][2] = o[m2][3] = 0.0f;
  const uint32_t v_base = smem_u32(smem + C::F_OFF);

  bool ok = true;
  for (int i = 0; i < n_tiles && ok; ++i) {
    const int sr = i % C::NSR, sf = i % C::NSF;
    if (!mbar_wait(&bar.raw_full[sr], (i / C::NSR) & 1, p.status)) { ok = false; break; }
    const int r0 = warp * 16;  // this warp's 16 rows of the tile
    const uint8_t* k_lo = smem + C::RAW_OFF + sr * B::RAW_TILE + (r0 + grp) * ROW + off;  // row r0 + grp
    const uint8_t* k_hi = k_lo + 8 * ROW;                                                   // row r0 + grp + 8
    // ---- S^T = K Q^T, one accumulator per 32-element block, then the rows' block scales
    float sacc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
    for (int blk = 0; blk < D / 32; ++blk) {
      float sb[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const int cb = blk * 34 + 2 + h * 16 + 2 * tig;  // byte of dims (16h + 2tig, +1) of the block
        mma16816(sb, i8pair(k_lo + cb), i8pair(k_hi + cb), i8pair(k_lo + cb + 8), i8pair(k_hi + cb + 8),
                 qb[2 * blk + h][0], qb[2 * blk + h][1]);
      }
      const float d_lo = __half2float(*reinterpret_cast<const __half*>(k_lo + blk * 34));
      const float d_hi = __half2float(*reinterpret_cast<const __half*>(k_hi + blk * 34));
      sacc[0] = fmaf(d_lo, sb[0], sacc[0]);
      sacc[1] = fmaf(d_lo, sb[1], sacc[1]);
      sacc[2] = fmaf(d_hi, sb[2], sacc[2]);
      sacc[3] = fmaf(d_hi, sb[3], sacc[3]);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&bar.raw_empty[sr]);  // this warp's K reads are done
    // ---- mask rows past the split's end (their raw bytes may be anything); online softmax
    const int base_row = i * kTileRows + r0;
    const bool lo_ok = base_row + grp < n, hi_ok = base_row + grp + 8 < n;
    const float s0 = lo_ok ? sacc[0] * sl2 : -INFINITY, s1 = lo_ok ? sacc[1] * sl2 : -INFINITY;
    const float s2 = hi_ok ? sacc[2] * sl2 : -INFINITY, s3 = hi_ok ? sacc[3] * sl2 : -INFINITY;
    float mt[2] = {fmaxf(s0, s2), fmaxf(s1, s3)};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      mt[h] = fmaxf(mt[h], __shfl_xor_sync(0xffffffffu, mt[h], 4));
      mt[h] = fmaxf(mt[h], __shfl_xor_sync(0xffffffffu, mt[h], 8));
      mt[h] = fmaxf(mt[h], __shfl_xor_sync(0xffffffffu, mt[h], 16));
    }
    float f[2];
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const float m_new = fmaxf(m_run[h], mt[h]);
      f[h] = ex2_approx(m_run[h] - m_new);
      m_run[h] = m_new;
      l_run[h] *= f[h];
    }
#pragma unroll
    for (int m2 = 0; m2 < D / 16; ++m2) {
      o[m2][0] *= f[0];
      o[m2][1] *= f[1];
      o[m2][2] *= f[0];
      o[m2][3] *= f[1];
    }
    const float p0 = ex2_approx(s0 - m_run[0]), p1 = ex2_approx(s1 - m_run[1]);
    const float p2 = ex2_approx(s2 - m_run[0]), p3 = ex2_approx(s3 - m_run[1]);
    l_run[0] += p0 + p2;
    l_run[1] += p1 + p3;
    const uint32_t pb0 = movmatrix_trans(pack_h2(p0, p1)), pb1 = movmatrix_trans(pack_h2(p2, p3));
    // ---- O^T += V^T P^T from the converted fp16 V tile
    if (!mbar_wait(&bar.f_full[sf], (i / C::NSF) & 1, p.status)) { ok = false; break; }
    const uint32_t vt = v_base + sf * B::F_TILE;
#pragma unroll
    for (int m2 = 0; m2 < D / 16; ++m2) {
      uint32_t a0, a1, a2, a3;
      ldsm_x4_t(sw_addr(vt, r0 + r8 + 8 * (mi >> 1), m2 * 16 + 8 * (mi & 1)), a0, a1, a2, a3);
      mma16816(o[m2], a0, a1, a2, a3, pb0, pb1);
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(&bar.f_empty[sf]);
  }

#pragma unroll
  for (int h = 0; h < 2; ++h) {
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 4);
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 8);
    l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 16);
  }
  // all tiles consumed (every raw slot's K and V were read): the raw ring holds the merge
  asm volatile("bar.sync 1, 128;" ::: "memory");
  float* merge = reinterpret_cast<float*>(smem + C::RAW_OFF);
  float* ml_s = merge;
  float* o_s = ml_s + kComputeWarps * 16 * 2;
  if (grp == 0) {
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      ml_s[(warp * 16 + 2 * tig + h) * 2] = m_run[h];
      ml_s[(warp * 16 + 2 * tig + h) * 2 + 1] = l_run[h];
    }
  }
#pragma unroll
  for (int m2 = 0; m2 < D / 16; ++m2)
#pragma unroll
    for (int e = 0; e < 4; ++e)
      o_s[(warp * 16 + 2 * tig + (e & 1)) * OP + m2 * 16 + grp + 8 * (e >> 1)] = o[m2][e];
  decode_emit<D>(p, merge, h0, g_count, b, split, n_splits);
}

// ------------------------------------------------------------------ Q8_0 decode, stream-K schedule
// The same per-tile work as decode_q8k_kernel (K straight from the raw tiles, V through two
// converter warps), scheduled as one wave: the sequences' 64-row cache tiles are laid end to end,
// and for every KV head the k-th of C CTAs takes tiles [k*T/C, (k+1)*T/C) of the T in total
// (CTA k * Hkv + kvh: the heads of a token block are streamed together). A (sequence, KV head)
// unit is a sequence's tiles for one head. A CTA's range
// covers one or more units, whole or in part; the producer streams straight across unit
// boundaries (the ring never drains between units), the compute warps restart their softmax
// state at each unit. A unit that lies inside one range is written directly; a unit split
// between CTAs leaves one partial (max, sum, unnormalised O) per part in its CTA's slot (first
// or last segment of the range: two slots per CTA) and the part that arrives last merges them
// (epoch-tagged counter per unit, nobody waits). Every CTA streams about the same number of
// tiles, so there is no partial last wave and each CTA pays its fixed costs once. The four
// compute warps' partials go to per-CTA slots in scratch (read back from L2), which keeps the
// shared memory for a 4-deep raw ring at two CTAs per SM.
constexpr int kSkMaxUnits = kQ8StreamKMaxUnits;  // sequences this schedule handles
constexpr int kSkMinTiles = 8;     // fewest tiles a range gets (small problems use fewer CTAs)

template <int D>
struct Q8sCfg {
  using B = Q8Cfg<D>;
  static constexpr int NSR = 4;                                 // raw K+V ring depth
  static constexpr int NSF = 2;                                 // fp16 V ring depth
  static constexpr int RAW_OFF = 0;
  static constexpr int F_OFF = (2 * NSR * B::RAW_TILE + 1023) / 1024 * 1024;
  static constexpr int Q_OFF = F_OFF + NSF * B::F_TILE;
  static constexpr int Q_BYTES = 8 * (D + 8) * 2;               // the head group's 8 rows of Q
  static constexpr int TS_OFF = Q_OFF + Q_BYTES;                // tile prefix sums [units + 1]
  static constexpr int BAR_OFF = TS_OFF + ((kSkMaxUnits + 1) * 4 + 15) / 16 * 16;
  static constexpr int SMEM = BAR_OFF + 256 + 1024;
  static_assert(SMEM <= 115712, "two stream-K Q8_0 CTAs must fit one SM");
};
// Per-warp partial slots of a CTA in scratch: [3 slots][4 warps][8 heads] x (D + 2) floats; slot
// 0 = the range's first segment, 1 = its last, 2 = a unit that lies wholly inside the range.
constexpr int kSkSlots = 3;

// Owner CTA of flattened tile t when CTA c covers [c*T/C, (c+1)*T/C).
__device__ __forceinline__ int sk_owner(int64_t t, int64_t T, int64_t C) {
  return static_cast<int>(((t + 1) * C - 1) / T);
}

template <int D>
__global__ void __launch_bounds__(kQ8kThreads, 2) decode_q8s_kernel(const __grid_constant__ DecodeMmaArgs a) {
  using C = Q8sCfg<D>;
  using B = Q8Cfg<D>;
  constexpr int ROW = B::ROW_BYTES;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Q8Bars& bar = *reinterpret_cast<Q8Bars*>(smem + C::BAR_OFF);
  __half* q_s = reinterpret_cast<__half*>(smem + C::Q_OFF);
  int32_t* ts = reinterpret_cast<int32_t*>(smem + C::TS_OFF);
  __shared__ int s_last;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const DecodeArgs& p = a.base;
  const int G = p.n_q_heads / p.n_kv_heads;  // <= 8: one head group per KV head
  const int NB = p.batch;
  // CTA c = k * Hkv + kvh: every KV head has the same ranges, taken by adjacent CTAs, so the
  // heads of a token block are streamed side by side (one DRAM page serves all of a row's heads)
  const int kvh = static_cast<int>(blockIdx.x) % p.n_kv_heads;
  const int k_cta = static_cast<int>(blockIdx.x) / p.n_kv_heads;
  const int64_t Ch = gridDim.x / p.n_kv_heads;

  // ---- tiles per sequence and their prefix sums over the batch, by warp 0
  if (warp == 0) {
    const int per = (NB + 31) / 32;
    const int b0 = lane * per, b1 = min(NB, b0 + per);
    auto tiles_of = [&](int b) -> int {
      const int32_t Lk = (p.seq_len ? p.seq_len[b] : p.start_scalar) + p.len_offset;
      if (Lk > p.kv.capacity || Lk < 1) {
        if (blockIdx.x == 0) atomicOr(p.status, kStatusBadLength);
        return 0;
      }
      return (Lk + kTileRows - 1) / kTileRows;
    };
    int sum = 0;
    for (int b = b0; b < b1; ++b) sum += tiles_of(b);
    int incl = sum;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
      const int v = __shfl_up_sync(0xffffffffu, incl, off);
      if (lane >= off) incl += v;
    }
    int run = incl - sum;
    for (int b = b0; b < b1; ++b) {
      ts[b] = run;
      run += tiles_of(b);
    }
    if (lane == 31) ts[NB] = incl;
  }
  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NSR; ++i) {
      mbar_init(&bar.raw_full[i], 1);
      mbar_init(&bar.raw_empty[i], kQ8kConvWarps * 32 + kComputeWarps);
    }
    for (int i = 0; i < C::NSF; ++i) {
      mbar_init(&bar.f_full[i], kQ8kConvWarps * 32);
      mbar_init(&bar.f_empty[i], kComputeWarps);
    }
    mbar_init(&bar.appended, 64);
    fence_mbar_init();
  }
  __syncthreads();
  const int64_t T = ts[NB];  // tiles of one KV head over the whole batch
  const int64_t min_ctas = (T + kSkMinTiles - 1) / kSkMinTiles;
  const int64_t Cn = Ch < min_ctas ? Ch : (min_ctas > 0 ? min_ctas : 1);
  const int c = blockIdx.x;
  if (T == 0 || k_cta >= Cn) return;
  const int64_t lo = k_cta * T / Cn, hi = (k_cta + 1) * T / Cn;
  if (lo >= hi) return;
  // first sequence of the range: the last b with ts[b] <= lo (empty sequences have ts[b] == ts[b + 1])
  int b_first = 0;
  {
    int l = 0, r = NB - 1;
    while (l < r) {
      const int m = (l + r + 1) >> 1;
      if (ts[m] <= lo) l = m; else r = m - 1;
    }
    b_first = l;
    while (b_first < NB - 1 && ts[b_first + 1] <= lo) ++b_first;
  }
  // Walks this range's segments: f(u, b, kvh, seg_lo, seg_hi, Lk) with tile indices local to the
  // sequence; u = b * Hkv + kvh is the (sequence, KV head) unit.
  auto for_segments = [&](auto&& f) {
    int64_t t = lo;
    for (int b = b_first; b < NB && t < hi; ++b) {
      if (ts[b + 1] <= t) continue;
      const int32_t Lk = (p.seq_len ? p.seq_len[b] : p.start_scalar) + p.len_offset;
      const int s_lo = static_cast<int>(t - ts[b]);
      const int64_t seg_end = hi < ts[b + 1] ? hi : static_cast<int64_t>(ts[b + 1]);
      const int s_hi = static_cast<int>(seg_end - ts[b]);
      if (!f(b * p.n_kv_heads + kvh, b, kvh, s_lo, s_hi, Lk)) return;
      t = ts[b] + s_hi;
    }
  };
  const int head_off_words = static_cast<int>(p.kv.head_stride / 4);

  // ---- the new token's rows of every unit whose last tile is in this range (warps 0 and 1),
  // before the producer loads those tiles
  const bool appends = p.fuse_append != 0;
  if (appends && warp < 2) {
    for_segments([&](int u, int b, int kvh, int s_lo, int s_hi, int32_t Lk) {
      if (ts[b] + s_hi == ts[b + 1]) append_new_row<D>(p, b, kvh, Lk - 1, warp, lane);
      return true;
    });
    mbar_arrive(&bar.appended);
  }

  if (warp == kComputeWarps + kQ8kConvWarps) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&a.k_map);
      tma_prefetch_desc(&a.v_map);
      int g = 0;
      bool ok = true;
      for_segments([&](int u, int b, int kvh, int s_lo, int s_hi, int32_t Lk) {
        const int head_word = kvh * head_off_words, box_x = head_word & ~3;
        for (int i = s_lo; i < s_hi; ++i, ++g) {
          const int s = g % C::NSR;
          if (appends && i == (Lk - 1) / kTileRows && !mbar_wait(&bar.appended, 0, p.status)) { ok = false; break; }
          if (!mbar_wait(&bar.raw_empty[s], ((g / C::NSR) & 1) ^ 1, p.status)) { ok = false; break; }
          mbar_arrive_expect_tx(&bar.raw_full[s], 2 * B::RAW_TILE);
          const int r = kv_phys_row(p.kv, b, i * kTileRows), bc = p.kv.block_table ? 0 : b;
          tma_load_4d(smem + C::RAW_OFF + s * B::RAW_TILE, &a.k_map, &bar.raw_full[s], box_x, r, bc, 0);
          tma_load_4d(smem + C::RAW_OFF + (C::NSR + s) * B::RAW_TILE, &a.v_map, &bar.raw_full[s], box_x, r, bc, 0);
        }
        return ok;
      });
    }
    return;
  }
  if (warp >= kComputeWarps) {
    // ------------------------------------------------------------------ V converters
    const int row = threadIdx.x - kComputeWarps * 32;  // 0..63
    int g = 0;
    bool ok = true;
    for_segments([&](int u, int b, int kvh, int s_lo, int s_hi, int32_t Lk) {
      const int off_words = (kvh * head_off_words) & 3;
      for (int i = s_lo; i < s_hi; ++i, ++g) {
        const int sr = g % C::NSR, sf = g % C::NSF;
        if (!mbar_wait(&bar.raw_full[sr], (g / C::NSR) & 1, p.status)) { ok = false; break; }
        uint32_t w[B::BOX_WORDS];
        const uint4* src = reinterpret_cast<const uint4*>(smem + C::RAW_OFF + (C::NSR + sr) * B::RAW_TILE + row * ROW);
#pragma unroll
        for (int cc = 0; cc < B::BOX_WORDS / 4; ++cc) {
          const uint4 v = src[cc];
          w[4 * cc] = v.x;
          w[4 * cc + 1] = v.y;
          w[4 * cc + 2] = v.z;
          w[4 * cc + 3] = v.w;
        }
        mbar_arrive(&bar.raw_empty[sr]);
        if (!mbar_wait(&bar.f_empty[sf], ((g / C::NSF) & 1) ^ 1, p.status)) { ok = false; break; }
        uint8_t* tile = smem + C::F_OFF + sf * B::F_TILE;
        if (i * kTileRows + row < Lk) {
          if constexpr (D == 128) {
            if (off_words == 0) q8_row_to_f16<D, 0>(w, tile, row);
            else q8_row_to_f16<D, 2>(w, tile, row);
          } else {
            switch (off_words) {
              case 0: q8_row_to_f16<D, 0>(w, tile, row); break;
              case 1: q8_row_to_f16<D, 1>(w, tile, row); break;
              case 2: q8_row_to_f16<D, 2>(w, tile, row); break;
              default: q8_row_to_f16<D, 3>(w, tile, row); break;
            }
          }
        } else {  // rows past the unit's end: zeros (their stale bytes could decode to NaN)
#pragma unroll
          for (int cc = 0; cc < D / 8; ++cc)
            *reinterpret_cast<uint4*>(tile + (cc >> 3) * (kTileRows * 128) + row * 128 + (((cc & 7) ^ (row & 7)) << 4)) =
                make_uint4(0, 0, 0, 0);
        }
        mbar_arrive(&bar.f_full[sf]);
      }
      return ok;
    });
    return;
  }

  // ------------------------------------------------------------------ compute warps
  const int grp = lane >> 2, tig = lane & 3;
  const int mi = lane >> 3, r8 = lane & 7;
  const __half2 k1152 = __floats2half2_rn(1152.0f, 1152.0f);
  auto i8pair = [&](const uint8_t* p2) -> uint32_t {  // two int8 (2-byte aligned) -> exact fp16 pair
    const uint32_t x = static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(p2)) ^ 0x8080u;
    const uint32_t e = __byte_perm(x, 0x64646464u, 0x4140);
    const __half2 h = __hsub2(*reinterpret_cast<const __half2*>(&e), k1152);
    return *reinterpret_cast<const uint32_t*>(&h);
  };
  const float sl2 = p.scale * kLog2e;
  const uint32_t v_base = smem_u32(smem + C::F_OFF);
  // scratch: part_o [C][slot][warp][8][D], then part_ml [C][slot][warp][8][2]
  float* part_o = p.part_o;
  float* part_ml = p.part_o + static_cast<int64_t>(gridDim.x) * kSkSlots * kComputeWarps * 8 * D;
  int g = 0;
  bool ok = true;
  bool first_seg = true;
  for_segments([&](int u, int b, int kvh, int s_lo, int s_hi, int32_t Lk) {
    const int h0 = kvh * G;
    const int32_t start = Lk - p.len_offset;
    load_q_rows<D, 8>(p, q_s, b, h0, G, start, kComputeWarps * 32);
    asm volatile("bar.sync 1, 128;" ::: "memory");
    uint32_t qb[D / 16][2];
    {
      const uint32_t qbase = smem_u32(q_s);
#pragma unroll
      for (int kk = 0; kk < D / 16; kk += 2)
        ldsm_x4(qbase + (r8 * (D + 8) + kk * 16 + 8 * mi) * 2, qb[kk][0], qb[kk][1], qb[kk + 1][0], qb[kk + 1][1]);
    }
    float m_run[2] = {-1e30f, -1e30f}, l_run[2] = {0.0f, 0.0f};
    float o[D / 16][4];
#pragma unroll
    for (int m2 = 0; m2 < D / 16; ++m2) o[m2][0] = o[m2][1] = o[m2][2] = o[m2][3] = 0.0f;
    const int off = ((kvh * head_off_words) & 3) * 4;
    for (int i = s_lo; i < s_hi && ok; ++i, ++g) {
      const int sr = g % C::NSR, sf = g % C::NSF;
      if (!mbar_wait(&bar.raw_full[sr], (g / C::NSR) & 1, p.status)) { ok = false; break; }
      const int r0 = warp * 16;
      const uint8_t* k_lo = smem + C::RAW_OFF + sr * B::RAW_TILE + (r0 + grp) * ROW + off;
      const uint8_t* k_hi = k_lo + 8 * ROW;
      float sacc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
      for (int blk = 0; blk < D / 32; ++blk) {
        float sb[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          const int cb = blk * 34 + 2 + h * 16 + 2 * tig;
          mma16816(sb, i8pair(k_lo + cb), i8pair(k_hi + cb), i8pair(k_lo + cb + 8), i8pair(k_hi + cb + 8),
                   qb[2 * blk + h][0], qb[2 * blk + h][1]);
        }
        const float d_lo = __half2float(*reinterpret_cast<const __half*>(k_lo + blk * 34));
        const float d_hi = __half2float(*reinterpret_cast<const __half*>(k_hi + blk * 34));
        sacc[0] = fmaf(d_lo, sb[0], sacc[0]);
        sacc[1] = fmaf(d_lo, sb[1], sacc[1]);
        sacc[2] = fmaf(d_hi, sb[2], sacc[2]);
        sacc[3] = fmaf(d_hi, sb[3], sacc[3]);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.raw_empty[sr]);
      const int base_row = i * kTileRows + r0;
      const bool lo_ok = base_row + grp < Lk, hi_ok = base_row + grp + 8 < Lk;
      const float s0 = lo_ok ? sacc[0] * sl2 : -INFINITY, s1 = lo_ok ? sacc[1] * sl2 : -INFINITY;
      const float s2 = hi_ok ? sacc[2] * sl2 : -INFINITY, s3 = hi_ok ? sacc[3] * sl2 : -INFINITY;
      float mt[2] = {fmaxf(s0, s2), fmaxf(s1, s3)};
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        mt[h] = fmaxf(mt[h], __shfl_xor_sync(0xffffffffu, mt[h], 4));
        mt[h] = fmaxf(mt[h], __shfl_xor_sync(0xffffffffu, mt[h], 8));
        mt[h] = fmaxf(mt[h], __shfl_xor_sync(0xffffffffu, mt[h], 16));
      }
      float f[2];
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        const float m_new = fmaxf(m_run[h], mt[h]);
        f[h] = ex2_approx(m_run[h] - m_new);
        m_run[h] = m_new;
        l_run[h] *= f[h];
      }
#pragma unroll
      for (int m2 = 0; m2 < D / 16; ++m2) {
        o[m2][0] *= f[0];
        o[m2][1] *= f[1];
        o[m2][2] *= f[0];
        o[m2][3] *= f[1];
      }
      const float p0 = ex2_approx(s0 - m_run[0]), p1 = ex2_approx(s1 - m_run[1]);
      const float p2 = ex2_approx(s2 - m_run[0]), p3 = ex2_approx(s3 - m_run[1]);
      l_run[0] += p0 + p2;
      l_run[1] += p1 + p3;
      const uint32_t pb0 = movmatrix_trans(pack_h2(p0, p1)), pb1 = movmatrix_trans(pack_h2(p2, p3));
      if (!mbar_wait(&bar.f_full[sf], (g / C::NSF) & 1, p.status)) { ok = false; break; }
      const uint32_t vt = v_base + sf * B::F_TILE;
#pragma unroll
      for (int m2 = 0; m2 < D / 16; ++m2) {
        uint32_t a0, a1, a2, a3;
        ldsm_x4_t(sw_addr(vt, r0 + r8 + 8 * (mi >> 1), m2 * 16 + 8 * (mi & 1)), a0, a1, a2, a3);
        mma16816(o[m2], a0, a1, a2, a3, pb0, pb1);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.f_empty[sf]);
    }
    // every compute thread takes the same path out, so the named barriers below always meet
    if (!bar1_and_128(ok)) return false;
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 4);
      l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 8);
      l_run[h] += __shfl_xor_sync(0xffffffffu, l_run[h], 16);
    }
    // ---- this warp's (max, sum, unnormalised O) per head into its slot (heads in N: 2 * tig + h)
    const int n_parts = sk_owner(ts[b + 1] - 1, T, Cn) - sk_owner(ts[b], T, Cn) + 1;
    const int slot = n_parts == 1 ? 2 : first_seg ? 0 : 1;
    first_seg = false;
    const int64_t wbase = ((static_cast<int64_t>(c) * kSkSlots + slot) * kComputeWarps + warp) * 8;
    if (grp == 0) {
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        part_ml[(wbase + 2 * tig + h) * 2] = m_run[h];
        part_ml[(wbase + 2 * tig + h) * 2 + 1] = l_run[h];
      }
    }
#pragma unroll
    for (int m2 = 0; m2 < D / 16; ++m2)
#pragma unroll
      for (int e = 0; e < 4; ++e)
        part_o[(wbase + 2 * tig + (e & 1)) * D + m2 * 16 + grp + 8 * (e >> 1)] = o[m2][e];
    __threadfence();
    asm volatile("bar.sync 1, 128;" ::: "memory");
    // the warps' partials to merge: this slot alone (a whole unit), or every part's slot, once the
    // part that arrives last has seen all of them
    int c0 = 0, n_merge = 1;
    bool c0_first = slot == 0;
    bool merge = true;
    if (n_parts > 1) {
      unsigned long long* counter = &p.counters[u];
      if (threadIdx.x == 0) {
        const bool last = split_arrive(counter, p.epoch, n_parts, p.status);
        if (last) atomicExch(counter, 0ull);
        s_last = last ? 1 : 0;
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
      merge = s_last != 0;
      c0 = sk_owner(ts[b], T, Cn);       // this KV head's range index of the unit's first part
      c0_first = c0 * T / Cn >= ts[b];  // the unit is that range's first segment
      n_merge = n_parts;
      if (merge) __threadfence();
    }
    if (merge) {
      for (int idx = threadIdx.x; idx < G * (D / 4); idx += kComputeWarps * 32) {
        const int gg = idx / (D / 4), d = (idx % (D / 4)) * 4;
        auto slot_base = [&](int k, int w) -> int64_t {
          const int sl = n_parts == 1 ? 2 : (k > 0 || c0_first) ? 0 : 1;
          const int64_t cc = n_parts == 1 ? c : static_cast<int64_t>(c0 + k) * p.n_kv_heads + kvh;  // CTA of part k
          return ((cc * kSkSlots + sl) * kComputeWarps + w) * 8 + gg;
        };
        float m = -INFINITY;
        for (int k = 0; k < n_merge; ++k)
#pragma unroll
          for (int w = 0; w < kComputeWarps; ++w) m = fmaxf(m, __ldcg(&part_ml[slot_base(k, w) * 2]));
        float l = 0.0f;
        float4 acc = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
        for (int k = 0; k < n_merge; ++k)
#pragma unroll
          for (int w = 0; w < kComputeWarps; ++w) {
            const int64_t pb = slot_base(k, w);
            const float wt = exp2f(__ldcg(&part_ml[pb * 2]) - m);
            l = fmaf(__ldcg(&part_ml[pb * 2 + 1]), wt, l);
            const float4 o4 = __ldcg(reinterpret_cast<const float4*>(&part_o[pb * D + d]));
            acc.x = fmaf(o4.x, wt, acc.x);
            acc.y = fmaf(o4.y, wt, acc.y);
            acc.z = fmaf(o4.z, wt, acc.z);
            acc.w = fmaf(o4.w, wt, acc.w);
          }
        const float inv = 1.0f / l;
        const int h = h0 + gg;
        const int64_t oidx = (static_cast<int64_t>(b) * p.n_q_heads + h) * D + d;
        if (p.out_dtype == AIHOST_F32) {
          *reinterpret_cast<float4*>(static_cast<float*>(p.out) + oidx) =
              make_float4(acc.x * inv, acc.y * inv, acc.z * inv, acc.w * inv);
        } else {
          *reinterpret_cast<uint2*>(static_cast<__half*>(p.out) + oidx) =
              make_uint2(pack_h2(acc.x * inv, acc.y * inv), pack_h2(acc.z * inv, acc.w * inv));
        }
        if (p.lse && d == 0) p.lse[static_cast<int64_t>(b) * p.n_q_heads + h] = (m + log2f(l)) * kLn2;
      }
    }
    // slot 2 and q_s are reused by the next segment
    asm volatile("bar.sync 1, 128;" ::: "memory");
    return true;
  });
}

template <int D>
cudaError_t launch_q8s(const DecodeMmaArgs& a, int32_t num_sms, cudaStream_t st) {
  using C = Q8sCfg<D>;
  auto kern = decode_q8s_kernel<D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int hkv = a.base.n_kv_heads;
  kern<<<(2 * num_sms) / hkv * hkv, kQ8kThreads, C::SMEM, st>>>(a);
  return cudaGetLastError();
}

template <int D>
cudaError_t launch_q8k(const DecodeMmaArgs& a, cudaStream_t st) {
  using C = Q8kCfg<D>;
  auto kern = decode_q8k_kernel<D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid(a.base.max_splits, a.base.n_kv_heads, a.base.batch);
  kern<<<grid, kQ8kThreads, C::SMEM, st>>>(a);
  return cudaGetLastError();
}

template <int D>
cudaError_t launch_q8(const DecodeMmaArgs& a, cudaStream_t st) {
  using C = Q8Cfg<D>;
  const bool tr = a.base.n_q_heads / a.base.n_kv_heads <= 8;
  if (tr) return launch_q8k<D>(a, st);
  auto kern = tr ? decode_q8_kernel<D, true> : decode_q8_kernel<D, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int G = a.base.n_q_heads / a.base.n_kv_heads;
  dim3 grid(a.base.max_splits, a.base.n_kv_heads * ((G + 15) / 16), a.base.batch);
  kern<<<grid, kQ8Threads, C::SMEM, st>>>(a);
  return cudaGetLastError();
}

template <int D>
cudaError_t launch_d(const DecodeMmaArgs& a, cudaStream_t st) {
  using C = DecodeCfg<D>;
  const bool tr = a.base.n_q_heads / a.base.n_kv_heads <= 8;
  auto kern = tr ? decode_mma_kernel<D, true> : decode_mma_kernel<D, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  const int G = a.base.n_q_heads / a.base.n_kv_heads;
  dim3 grid(a.base.max_splits, a.base.n_kv_heads * ((G + 15) / 16), a.base.batch);
  kern<<<grid, kThreads, C::SMEM, st>>>(a);
  return cudaGetLastError();
}

}  // namespace

size_t q8_stream_k_bytes(int32_t head_dim, int32_t num_sms) {
  return sizeof(float) * static_cast<size_t>(2 * num_sms) * kSkSlots * kComputeWarps * 8 * (head_dim + 2);
}

cudaError_t launch_decode_mma(const DecodeMmaArgs& a, cudaStream_t st) {
  if (a.base.kv.dtype == AIHOST_Q8_0 && a.base.stream_k)
    return a.base.head_dim == 64 ? launch_q8s<64>(a, a.base.num_sms, st) : launch_q8s<128>(a, a.base.num_sms, st);
  if (a.base.kv.dtype == AIHOST_Q8_0) return a.base.head_dim == 64 ? launch_q8<64>(a, st) : launch_q8<128>(a, st);
  return a.base.head_dim == 64 ? launch_d<64>(a, st) : launch_d<128>(a, st);
}

uint32_t q8_box_words(int32_t head_dim, int64_t head_stride) {
  // 0 when some head would start further past its 16-byte boundary than the box allows
  const int64_t hs = head_stride / 4;
  const int max_off = hs % 4 == 0 ? 0 : hs % 2 == 0 ? 2 : 3;
  const int head_words = head_dim / 32 * 34 / 4;
  const int box = head_dim == 64 ? Q8Cfg<64>::BOX_WORDS : Q8Cfg<128>::BOX_WORDS;
  return head_words + max_off <= box ? static_cast<uint32_t>(box) : 0u;
}

}  // namespace aihost
