// prefill_sm100.cu — causal prefill attention on the 5th-generation tensor cores.
//
// Replaces the prefill branch of ComputeOps.MultiHeadAttention (ComputeOps.cs:1076-1101): per
// Q head the reference slices Q/K/V, materialises K^T and the [S, Lk] fp32 score matrix in
// global memory, scales, masks (j > P + i -> -1e38), runs a three-pass row softmax and a
// second fp32 GEMM — about ten dispatches per head, each followed by a fence wait.
//
// Here one CTA owns 128 query rows of one Q head and streams its KV head's cache rows in
// 128-row tiles (flash attention, online softmax), never writing scores to memory:
//   warp 0      TMA producer: Q tile once, then K/V tiles into a 2-3 stage ring (no multicast)
//   warp 1      TMEM owner and MMA issuer: S = Q K^T and O += P V with tcgen05.mma
//               (kind::f16, M=128, fp32 accumulators in TMEM; S double-buffered)
//   warps 2-5   one thread per query row: RoPE of the Q tile in shared memory, then per tile
//               tcgen05.ld of S, causal mask, online softmax in the exp2 domain, P (fp16) into
//               shared memory for the P.V MMA, lazy O rescale (only when the running max grows
//               by more than 2^8), and the final O / l epilogue.
// Tiles entirely above the diagonal are never loaded (causal tile skipping); CTAs take the
// longest query tiles first.
#include "common.cuh"
#include "kernels.h"

namespace aihost {
namespace {

constexpr int kBM = 128;  // query rows per CTA
constexpr int kBN = 128;  // cache rows per tile
constexpr int kThreads = 192;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

template <int D>
struct PrefillCfg {
  static constexpr int KB = D / 64;                 // 64-element (128-byte) column blocks
  static constexpr int TILE_BYTES = KB * kBN * 128;  // one [128 x D] fp16 tile
  static constexpr int NS = D == 64 ? 3 : 2;        // K and V ring depth
  static constexpr int Q_OFF = 0;
  static constexpr int K_OFF = Q_OFF + TILE_BYTES;
  static constexpr int V_OFF = K_OFF + NS * TILE_BYTES;
  static constexpr int P_OFF = V_OFF + NS * TILE_BYTES;
  static constexpr int P_BYTES = 2 * kBM * 128;      // [128 rows x 128 keys] fp16, two 64-key blocks
  static constexpr int BAR_OFF = P_OFF + P_BYTES;
  static constexpr int SMEM = BAR_OFF + 256 + 1024;  // barriers + alignment slack
  static constexpr uint32_t TMEM_COLS = 512;
  static constexpr uint32_t S_COL0 = 0, S_COL1 = 128, O_COL = 256;
};

// Byte offset of fp16 element (row, col) inside a [rows x 64k] block stack written by TMA with
// 128-byte swizzle: 128 bytes per row, 16-byte chunk index XOR (row % 8), 64-column blocks of
// rows*128 bytes each.
__device__ __forceinline__ uint32_t sw128_off(int row, int col, int rows_per_block) {
  const int kb = col >> 6, within = col & 63;
  const int chunk = (within >> 3) ^ (row & 7);
  return static_cast<uint32_t>(kb * rows_per_block * 128 + row * 128 + (chunk << 4) + ((within & 7) << 1));
}

struct Barriers {
  uint64_t q_full, q_ready, p_full, pv_done;
  uint64_t s_full[2];
  uint64_t k_full[3], k_empty[3], v_full[3], v_empty[3];
  uint32_t tmem_base;
};

template <int D>
__global__ void __launch_bounds__(kThreads, 1) prefill_kernel(const __grid_constant__ PrefillArgs a) {
  using C = PrefillCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers& bar = *reinterpret_cast<Barriers*>(smem + C::BAR_OFF);
  uint8_t* q_s = smem + C::Q_OFF;
  uint8_t* k_s = smem + C::K_OFF;
  uint8_t* v_s = smem + C::V_OFF;
  uint8_t* p_s = smem + C::P_OFF;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (a.n_new + kBM - 1) / kBM;
  const int qt = n_qt - 1 - static_cast<int>(blockIdx.x);  // longest tiles first
  const int h = blockIdx.y, b = blockIdx.z;
  const int kvh = h / (a.n_q_heads / a.n_kv_heads);
  const int q0 = qt * kBM;
  const int32_t start = a.seq_len ? a.seq_len[b] : a.start_scalar;
  const int32_t Lk = start + a.len_offset;
  // rows visible to this tile: j <= start + q0 + 127, j < Lk
  const int32_t kv_end = min(Lk, start + q0 + kBM);
  const int n_tiles = kv_end > 0 ? (kv_end + kBN - 1) / kBN : 0;
  const bool bad = Lk < 1 || start < 0;
  int32_t* status = a.status;

  if (threadIdx.x == 0) {
    mbar_init(&bar.q_full, 1);
    mbar_init(&bar.q_ready, 128);
    mbar_init(&bar.p_full, 128);
    mbar_init(&bar.pv_done, 1);
    for (int i = 0; i < 2; ++i) mbar_init(&bar.s_full[i], 1);
    for (int i = 0; i < C::NS; ++i) {
      mbar_init(&bar.k_full[i], 1);
      mbar_init(&bar.k_empty[i], 1);
      mbar_init(&bar.v_full[i], 1);
      mbar_init(&bar.v_empty[i], 1);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&bar.tmem_base, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar.tmem_base;

  if (bad) {
    if (threadIdx.x == 0 && blockIdx.x == 0 && h == 0) atomicOr(status, kStatusBadLength);
  } else if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&a.q_map);
      tma_prefetch_desc(&a.k_map);
      tma_prefetch_desc(&a.v_map);
      mbar_arrive_expect_tx(&bar.q_full, C::TILE_BYTES);
      for (int kb = 0; kb < C::KB; ++kb)
        tma_load_4d(q_s + kb * kBM * 128, &a.q_map, &bar.q_full, kb * 64, h, q0, b);
      for (int j = 0; j < n_tiles; ++j) {
        const int s = j % C::NS;
        const uint32_t par = ((j / C::NS) & 1) ^ 1;
        if (!mbar_wait(&bar.k_empty[s], par, status)) break;
        mbar_arrive_expect_tx(&bar.k_full[s], C::TILE_BYTES);
        for (int kb = 0; kb < C::KB; ++kb)
          tma_load_4d(k_s + s * C::TILE_BYTES + kb * kBN * 128, &a.k_map, &bar.k_full[s], kb * 64, kvh, j * kBN, b);
        if (!mbar_wait(&bar.v_empty[s], par, status)) break;
        mbar_arrive_expect_tx(&bar.v_full[s], C::TILE_BYTES);
        for (int kb = 0; kb < C::KB; ++kb)
          tma_load_4d(v_s + s * C::TILE_BYTES + kb * kBN * 128, &a.v_map, &bar.v_full[s], kb * 64, kvh, j * kBN, b);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc_qk = make_idesc_f16(kBM, kBN, 0, 0);
      constexpr uint32_t idesc_pv = make_idesc_f16(kBM, D, 0, 1);
      const uint32_t q_addr = smem_u32(q_s), k_addr = smem_u32(k_s), v_addr = smem_u32(v_s), p_addr = smem_u32(p_s);
      bool ok = mbar_wait(&bar.q_ready, 0, status);
      tc_fence_after();
      auto issue_qk = [&](int j) -> bool {
        const int s = j % C::NS;
        if (!mbar_wait(&bar.k_full[s], (j / C::NS) & 1, status)) return false;
        tc_fence_after();
        const uint32_t d_tmem = tmem + ((j & 1) ? C::S_COL1 : C::S_COL0);
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (kBN * 128) + (kk & 3) * 32;
          const uint64_t ad = make_sw128_desc(q_addr + off, 16, 1024);
          const uint64_t bd = make_sw128_desc(k_addr + s * C::TILE_BYTES + off, 16, 1024);
          umma_f16_ss(d_tmem, ad, bd, idesc_qk, kk > 0);
        }
        umma_commit(&bar.k_empty[s]);
        umma_commit(&bar.s_full[j & 1]);
        return true;
      };
      if (ok && n_tiles > 0) ok = issue_qk(0);
      if (ok && n_tiles > 1) ok = issue_qk(1);
      for (int j = 0; ok && j < n_tiles; ++j) {
        if (!mbar_wait(&bar.p_full, j & 1, status)) break;
        tc_fence_after();
        const int s = j % C::NS;
        if (!mbar_wait(&bar.v_full[s], (j / C::NS) & 1, status)) break;
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint64_t ad = make_sw128_desc(p_addr + (kk >> 2) * (kBM * 128) + (kk & 3) * 32, 16, 1024);
          const uint64_t bd = make_sw128_desc(v_addr + s * C::TILE_BYTES + kk * 2048, kBN * 128, 1024);
          umma_f16_ss(tmem + C::O_COL, ad, bd, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        }
        umma_commit(&bar.v_empty[s]);
        umma_commit(&bar.pv_done);
        if (j + 2 < n_tiles) ok = issue_qk(j + 2);
      }
    }
  } else {
    // ------------------------------------------------------------------ softmax warps
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;        // query row within the tile == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int32_t qpos = start + q0 + r;     // absolute position of this query row
    const int32_t limit = min(qpos, Lk - 1); // last visible cache row
    bool ok = mbar_wait(&bar.q_full, 0, status);
    if (ok && a.rope_mode != AIHOST_ROPE_NONE) {
      const float pos = static_cast<float>(qpos);
      __half* qh = reinterpret_cast<__half*>(q_s);
      for (int pair = 0; pair < D / 2; ++pair) {
        const int c1 = a.rope_mode == AIHOST_ROPE_NEOX ? pair : 2 * pair;
        const int c2 = a.rope_mode == AIHOST_ROPE_NEOX ? pair + D / 2 : 2 * pair + 1;
        __half* p1 = reinterpret_cast<__half*>(q_s + sw128_off(r, c1, kBM));
        __half* p2 = reinterpret_cast<__half*>(q_s + sw128_off(r, c2, kBM));
        const float x1 = __half2float(*p1), x2 = __half2float(*p2);
        float sn, cs;
        sincosf(__fmul_rn(pos, a.freqs.f[pair]), &sn, &cs);
        *p1 = __float2half_rn(__fsub_rn(__fmul_rn(x1, cs), __fmul_rn(x2, sn)));
        *p2 = __float2half_rn(__fadd_rn(__fmul_rn(x1, sn), __fmul_rn(x2, cs)));
      }
      (void)qh;
    }
    fence_proxy_async_smem();
    mbar_arrive(&bar.q_ready);

    const float sl2 = a.scale * kLog2e;
    float m = -1e30f, l = 0.0f;
    for (int j = 0; ok && j < n_tiles; ++j) {
      if (!mbar_wait(&bar.s_full[j & 1], (j >> 1) & 1, status)) { ok = false; break; }
      tc_fence_after();
      const uint32_t s_tmem = tmem + lane_base + ((j & 1) ? C::S_COL1 : C::S_COL0);
      uint32_t sreg[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(s_tmem + c * 32, sreg[c]);
      tmem_wait_ld();
      const int kv0 = j * kBN;
      float mx = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 32; ++i) {
          const int kv = kv0 + c * 32 + i;
          float v = __uint_as_float(sreg[c][i]) * sl2;
          v = kv <= limit ? v : -INFINITY;
          sreg[c][i] = __float_as_uint(v);
          mx = fmaxf(mx, v);
        }
      const float m_new = fmaxf(m, mx);
      const bool resc = m_new > m + kRescaleThreshold;
      const float factor = resc ? exp2f(m - m_new) : 1.0f;
      if (resc) { m = m_new; l *= factor; }
      float rs = 0.0f;
      // P = exp2(s - m) in fp16, into the K-major swizzled P tile (A operand of P.V)
      // (written only after P.V of the previous tile has finished reading the buffer)
      uint32_t ph[4][16];
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float p0 = exp2f(__uint_as_float(sreg[c][2 * i]) - m);
          const float p1 = exp2f(__uint_as_float(sreg[c][2 * i + 1]) - m);
          rs += p0 + p1;
          const __half2 hp = __floats2half2_rn(p0, p1);
          ph[c][i] = *reinterpret_cast<const uint32_t*>(&hp);
        }
      l += rs;
      if (j > 0 && !mbar_wait(&bar.pv_done, (j - 1) & 1, status)) { ok = false; break; }
      tc_fence_after();
      // last tile: cache rows >= Lk may hold stale bits; make them zero so that 0 * V stays 0
      if (kv0 + kBN > Lk) {
        const int s = j % C::NS;
        if (!mbar_wait(&bar.v_full[s], (j / C::NS) & 1, status)) { ok = false; break; }
        uint8_t* vt = v_s + s * C::TILE_BYTES;
        const int first = max(Lk - kv0, 0);
        for (int row = first + (threadIdx.x - 64) / (C::KB * 8); row < kBN; row += 128 / (C::KB * 8)) {
          const int chunk = (threadIdx.x - 64) % (C::KB * 8);
          *reinterpret_cast<uint4*>(vt + (chunk >> 3) * (kBN * 128) + row * 128 + (chunk & 7) * 16) =
              make_uint4(0, 0, 0, 0);
        }
      }
      // lazy rescale of this row's O accumulator (warp-uniform so tcgen05.ld/st stay convergent)
      if (j > 0 && __any_sync(0xffffffffu, resc)) {
        const uint32_t o_tmem = tmem + lane_base + C::O_COL;
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(o_tmem + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * factor);
          tmem_st32(o_tmem + c * 32, o);
        }
        tmem_wait_st();
      }
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int chunk16 = c * 4 + i;  // 8 keys per 16-byte chunk, 16 chunks per row
          const int kb = chunk16 >> 3, ch = chunk16 & 7;
          uint8_t* dst = p_s + kb * (kBM * 128) + r * 128 + ((ch ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(dst) = make_uint4(ph[c][4 * i], ph[c][4 * i + 1], ph[c][4 * i + 2], ph[c][4 * i + 3]);
        }
      fence_proxy_async_smem();
      tc_fence_before();
      mbar_arrive(&bar.p_full);
    }
    // ---- epilogue: O / l -> out[b][q0 + r][h][:]
    if (ok && n_tiles > 0 && mbar_wait(&bar.pv_done, (n_tiles - 1) & 1, status)) {
      tc_fence_after();
      const uint32_t o_tmem = tmem + lane_base + C::O_COL;
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      const bool valid = q0 + r < a.n_new;
      const int64_t orow = ((static_cast<int64_t>(b) * a.n_new + q0 + r) * a.n_q_heads + h) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t o[32];
        tmem_ld32(o_tmem + c * 32, o);
        tmem_wait_ld();
        if (valid) {
          if (a.out_dtype == AIHOST_F16) {
            uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(a.out) + orow + c * 32);
#pragma unroll
            for (int v = 0; v < 4; ++v) {
              uint32_t w[4];
#pragma unroll
              for (int i = 0; i < 4; ++i) {
                const __half2 hv = __floats2half2_rn(__uint_as_float(o[8 * v + 2 * i]) * inv,
                                                     __uint_as_float(o[8 * v + 2 * i + 1]) * inv);
                w[i] = *reinterpret_cast<const uint32_t*>(&hv);
              }
              dst[v] = make_uint4(w[0], w[1], w[2], w[3]);
            }
          } else {
            float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + orow + c * 32);
#pragma unroll
            for (int v = 0; v < 8; ++v)
              dst[v] = make_float4(__uint_as_float(o[4 * v]) * inv, __uint_as_float(o[4 * v + 1]) * inv,
                                   __uint_as_float(o[4 * v + 2]) * inv, __uint_as_float(o[4 * v + 3]) * inv);
          }
        }
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

template <int D>
cudaError_t launch_d(const PrefillArgs& a, cudaStream_t st) {
  using C = PrefillCfg<D>;
  auto kern = prefill_kernel<D>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  dim3 grid((a.n_new + kBM - 1) / kBM, a.n_q_heads, a.batch);
  kern<<<grid, kThreads, C::SMEM, st>>>(a);
  return cudaGetLastError();
}

}  // namespace

bool prefill_supported(int32_t head_dim) { return head_dim == 64 || head_dim == 128; }

cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t st) {
  return a.head_dim == 64 ? launch_d<64>(a, st) : launch_d<128>(a, st);
}

}  // namespace aihost
