// matmul_sm100.cu — the weight products around the attention op on the 5th-generation tensor
// cores: C[M, N] = A[M, K] · W[N, K]^T, W a GGUF weight (column-major [K x N] in GGUF terms,
// element (k, n) at n * K + k, i.e. one contiguous K-row per output column).
//
// Replaces ComputeOps.MatMulWeights (ComputeOps.cs:275-313, GLSL 16x16 fp32 tiles, k ascending)
// where the reference calls it next to attention: the Q/K/V projections that feed the op
// (ComputeOps.cs:1274-1276) and the output projection right after it (ComputeOps.cs:1317). The
// reference dequantises every K-quant weight to an fp32 scratch tensor first, per token
// (TransformerBase.TempF32 -> ComputeOps.DequantizeInto, ComputeOps.cs:761-861); here the
// weight is dequantised to fp16 (dequant_kernel below, the reference's formulas bit for bit
// before the one fp16 rounding) and multiplied on the tensor cores with fp32 accumulation.
//
// A is read through a 3-D tensor map over [n_parts][rows][K / n_parts]: K tile k comes from
// part k / (K / n_parts). With n_parts = N ranks this is the rank-major buffer the KV-head
// sharded all-gather leaves ([N][B][S][Hq/N][d]), consumed in place, with no permute.
//
// Kernel: one CTA per SM (BN = 256, 128) or two (BN = 64), 256 threads:
//   warp 0      TMA producer: A [128 x 64] and W [BN x 64] tiles into an NS-stage ring
//   warp 1      TMEM owner (2 x BN fp32 columns: two accumulators) and the tcgen05.mma issuer
//               (M = 128, N = BN, K = 16, both operands K-major, 128-byte swizzle)
//   warps 4-7   epilogue: tcgen05.ld of one accumulator (row per thread) while the MMA fills the
//               other, then the output stores.
// Enough tiles to fill the SMs: a persistent grid over the tiles. Too few (small M): the K range
// is split over the CTAs of a thread-block cluster, which sum their fp32 partial tiles through
// distributed shared memory (gemm_kernel's CL form). No TMA multicast anywhere.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace aihost {
namespace {

constexpr int kGemmThreads = 256;
constexpr int kGemmMaxSplits = 8;  // largest portable cluster
constexpr int kGBM = 128;  // rows of A per tile (TMEM lanes)
constexpr int kGBK = 64;   // K per stage: one 128-byte swizzle row of fp16

template <int BN>
struct GemmCfg {
  static constexpr int NS = 4;
  static constexpr int A_BYTES = kGBM * kGBK * 2;
  static constexpr int B_BYTES = BN * kGBK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int BAR_OFF = NS * STAGE;
  static constexpr int SMEM = BAR_OFF + 256 + 1024;
  static constexpr uint32_t TMEM_COLS = 2 * BN;  // 128 or 512: powers of two >= 32
};

struct GemmBars {
  uint64_t full[4], empty[4], acc_full[2], acc_empty[2];
  uint64_t slices_in;  // CL: the peers' slices of this CTA's output rows have landed
  uint32_t tmem_base;
};
static_assert(sizeof(GemmBars) <= 256, "gemm_kernel reserves 256 bytes for its barriers");

__device__ __forceinline__ uint32_t pack2h(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Eight consecutive outputs of one row (n a multiple of 8, n + 8 <= N checked by the caller).
__device__ __forceinline__ void store8(void* out, int32_t out_dtype, int64_t idx, const float* v) {
  if (out_dtype == AIHOST_F16) {
    *reinterpret_cast<uint4*>(static_cast<__half*>(out) + idx) =
        make_uint4(pack2h(v[0], v[1]), pack2h(v[2], v[3]), pack2h(v[4], v[5]), pack2h(v[6], v[7]));
  } else {
    float4* d = reinterpret_cast<float4*>(static_cast<float*>(out) + idx);
    d[0] = make_float4(v[0], v[1], v[2], v[3]);
    d[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

// SWAP (few rows of A, i.e. decode): the MMA's M = 128 rows are weight rows (output columns) and
// its N = BN columns are rows of A, so the weight, not zero padding, fills the 128-row operand;
// the accumulator then holds C^T and the epilogue stores it transposed (one row of C per TMEM
// column: 32 lanes write 32 consecutive outputs).
//
// CL (split K): the grid is the output tiles x k_splits (a power of two, <= 8), one unit per
// CTA, and the k_splits CTAs of a tile form one thread-block cluster, CTA (cluster rank) s taking
// K tiles [s * kt / k_splits, (s + 1) * kt / k_splits). Each CTA writes its fp32 partial tile
// into its drained operand ring as [output row][output column] (rows = TMEM columns when
// swapped, else TMEM lanes with one pad column, so a warp's 32 lanes hit 32 banks either way).
// After a cluster barrier (every peer's ring is drained too), one thread bulk-copies slice q of
// the tile's output rows to cluster rank q, counted on that rank's mbarrier; rank s then sums
// slice s over the k_splits partials in rank order (the same fixed order every call) from its own
// shared memory and stores it. A second cluster barrier keeps every CTA resident until all
// copies out of it have landed. No global scratch, no counters, no CTA spins on another.
template <int BN, bool SWAP, bool CL>
__global__ void __launch_bounds__(kGemmThreads, BN == 64 ? 2 : 1) gemm_kernel(const __grid_constant__ GemmArgs a) {
  using C = GemmCfg<BN>;
  // CL: partial tile [OUT_ROWS][PS] floats at the ring's start, then k_splits receive slots of one
  // slice (OUT_ROWS / k_splits rows) each
  constexpr int OUT_ROWS = SWAP ? BN : kGBM, OUT_COLS = SWAP ? kGBM : BN;
  constexpr int PS = SWAP ? OUT_COLS : OUT_COLS + 1;
  static_assert(!CL || (((OUT_ROWS * PS + 31) & ~31) + OUT_ROWS * PS) * 4 <= C::BAR_OFF,
                "partial tile and slices must fit in the ring");
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  GemmBars& bar = *reinterpret_cast<GemmBars*>(smem + C::BAR_OFF);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // tile rows (TMEM lanes) and tile columns: C's rows and columns, or its columns and rows (SWAP)
  const int R = SWAP ? a.N : a.M, NC = SWAP ? a.M : a.N;
  const int m_tiles = (R + kGBM - 1) / kGBM, n_tiles = (NC + BN - 1) / BN;
  const int kt_total = a.K / kGBK;
  const int splits = CL ? a.k_splits : 1;
  const int units = m_tiles * n_tiles * splits;
  int32_t* status = a.status;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::NS; ++i) {
      mbar_init(&bar.full[i], 1);
      mbar_init(&bar.empty[i], 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bar.acc_full[i], 1);
      mbar_init(&bar.acc_empty[i], 128);
    }
    mbar_init(&bar.slices_in, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&bar.tmem_base, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar.tmem_base;

  // unit u -> (m tile, n tile, K range); a tile's splits are adjacent (one cluster), tiles n-fastest
  auto unit_coords = [&](int u, int& mt, int& nt, int& kt0, int& kt1) {
    const int ks = u % splits, tile = u / splits;
    nt = tile % n_tiles;
    mt = tile / n_tiles;
    kt0 = ks * kt_total / splits;
    kt1 = (ks + 1) * kt_total / splits;
  };

  if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&a.a_map);
      tma_prefetch_desc(&a.b_map);
      int g = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
        int mt, nt, kt0, kt1;
        unit_coords(u, mt, nt, kt0, kt1);
        for (int kt = kt0; kt < kt1; ++kt, ++g) {
          const int s = g % C::NS;
          if (!mbar_wait(&bar.empty[s], ((g / C::NS) & 1) ^ 1, status)) { ok = false; break; }
          uint8_t* st = smem + s * C::STAGE;
          mbar_arrive_expect_tx(&bar.full[s], C::STAGE);
          const int k = kt * kGBK;
          if constexpr (SWAP) {  // A operand: weight rows; B operand: rows of A
            tma_load_2d(st, &a.b_map, &bar.full[s], k, mt * kGBM);
            tma_load_3d(st + C::A_BYTES, &a.a_map, &bar.full[s], k % a.part_cols, nt * BN, k / a.part_cols);
          } else {
            tma_load_3d(st, &a.a_map, &bar.full[s], k % a.part_cols, mt * kGBM, k / a.part_cols);
            tma_load_2d(st + C::A_BYTES, &a.b_map, &bar.full[s], k, nt * BN);
          }
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = make_idesc_f16(kGBM, BN, 0, 0);
      const uint32_t base = smem_u32(smem);
      int g = 0, j = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < units; u += gridDim.x, ++j) {
        int mt, nt, kt0, kt1;
        unit_coords(u, mt, nt, kt0, kt1);
        const int buf = j & 1;
        if (!mbar_wait(&bar.acc_empty[buf], ((j >> 1) & 1) ^ 1, status)) break;
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(buf * BN);
        for (int kt = kt0; kt < kt1; ++kt, ++g) {
          const int s = g % C::NS;
          if (!mbar_wait(&bar.full[s], (g / C::NS) & 1, status)) { ok = false; break; }
          tc_fence_after();
          const uint32_t sa = base + s * C::STAGE, sb = sa + C::A_BYTES;
#pragma unroll
          for (int kk = 0; kk < kGBK / 16; ++kk)
            umma_f16_ss(d, make_sw128_desc(sa + kk * 32, 16, 1024), make_sw128_desc(sb + kk * 32, 16, 1024), idesc,
                        (kt > kt0 || kk > 0) ? 1u : 0u);
          umma_commit(&bar.empty[s]);
        }
        if (ok) umma_commit(&bar.acc_full[buf]);
      }
    }
  } else if (warp >= 4) {
    // ------------------------------------------------------------------ epilogue
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // accumulator row == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    float* const part = reinterpret_cast<float*>(smem);  // CL: this CTA's partial tile
    int j = 0;
    for (int u = blockIdx.x; u < units; u += gridDim.x, ++j) {
      int mt, nt, kt0, kt1;
      unit_coords(u, mt, nt, kt0, kt1);
      const int buf = j & 1;
      // the four epilogue warps leave together (they meet at named barrier 1 inside)
      if (!bar1_and_128(mbar_wait(&bar.acc_full[buf], (j >> 1) & 1, status))) break;
      tc_fence_after();
#pragma unroll 1
      for (int c = 0; c < BN / 32; ++c) {
        uint32_t v[32];
        tmem_ld32(tmem + lane_base + static_cast<uint32_t>(buf * BN + c * 32), v);
        tmem_wait_ld();
        if constexpr (CL) {
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            const int col = c * 32 + jj;  // TMEM column
            part[SWAP ? col * PS + r : r * PS + col] = __uint_as_float(v[jj]);
          }
        } else if constexpr (SWAP) {
          // lane r = output column n, TMEM column = output row m: for each m the warp's 32 lanes
          // write 32 consecutive outputs of row m
          const int n = mt * kGBM + r, m0 = nt * BN + c * 32;
          if (n >= a.N) continue;
#pragma unroll
          for (int jj = 0; jj < 32; ++jj) {
            const int m = m0 + jj;
            if (m >= a.M) break;
            const float f = __uint_as_float(v[jj]);
            if (a.out_dtype == AIHOST_F16) static_cast<__half*>(a.out)[static_cast<int64_t>(m) * a.ldc + n] = __float2half_rn(f);
            else static_cast<float*>(a.out)[static_cast<int64_t>(m) * a.ldc + n] = f;
          }
        } else {
          const int m = mt * kGBM + r, n0 = nt * BN + c * 32;
          if (m >= a.M) continue;
#pragma unroll
          for (int g8 = 0; g8 < 4; ++g8) {
            const int n = n0 + g8 * 8;
            if (n >= a.N) break;
            float f[8];
#pragma unroll
            for (int i = 0; i < 8; ++i) f[i] = __uint_as_float(v[g8 * 8 + i]);
            store8(a.out, a.out_dtype, static_cast<int64_t>(m) * a.ldc + n, f);
          }
        }
      }
      // the accumulator may be overwritten by the unit after next
      tc_fence_before();
      mbar_arrive(&bar.acc_empty[buf]);
    }
  }

  if constexpr (CL) {
    // ---------------------------------------------------------------- split-K sum over the cluster
    const int ks = static_cast<int>(blockIdx.x) % splits;  // == cluster rank (clusters of `splits` CTAs)
    const int slice_rows = OUT_ROWS / splits, slice_floats = slice_rows * PS;
    const uint32_t slice_bytes = static_cast<uint32_t>(slice_floats) * 4u;
    float* const part = reinterpret_cast<float*>(smem);
    float* const slots = part + ((OUT_ROWS * PS + 31) & ~31);  // 128-byte aligned
    if (warp >= 4) fence_proxy_async_smem();  // the partial tile, for the bulk copies
    if (threadIdx.x == 0) mbar_arrive_expect_tx(&bar.slices_in, static_cast<uint32_t>(splits - 1) * slice_bytes);
    __syncwarp();
    cluster_sync_all();  // every CTA's partial tile is written and its operand ring drained
    if (threadIdx.x == 0) {
      for (int q = 1; q < splits; ++q) {
        const int dst = (ks + q) % splits;
        bulk_copy_to_peer(map_to_rank(smem_u32(slots + ks * slice_floats), dst), part + dst * slice_floats,
                          slice_bytes, map_to_rank(smem_u32(&bar.slices_in), dst));
      }
    }
    const bool ok = mbar_wait(&bar.slices_in, 0, status);
    int mt, nt, kt0, kt1;
    unit_coords(blockIdx.x, mt, nt, kt0, kt1);
    const int m_base = SWAP ? nt * BN : mt * kGBM, n_base = SWAP ? mt * kGBM : nt * BN;
    for (int e = threadIdx.x; ok && e < slice_floats; e += kGemmThreads) {
      const int orow = ks * slice_rows + e / PS, ocol = e % PS;
      if (ocol >= OUT_COLS) continue;  // pad column
      float acc = 0.0f;
      for (int p = 0; p < splits; ++p) {
        const float x = p == ks ? part[ks * slice_floats + e] : slots[p * slice_floats + e];
        acc = p == 0 ? x : acc + x;
      }
      const int m = m_base + orow, n = n_base + ocol;
      if (m < a.M && n < a.N) {
        const int64_t o = static_cast<int64_t>(m) * a.ldc + n;
        if (a.out_dtype == AIHOST_F16) static_cast<__half*>(a.out)[o] = __float2half_rn(acc);
        else static_cast<float*>(a.out)[o] = acc;
      }
    }
    __syncwarp();
    cluster_sync_all();  // every copy out of every CTA has landed: none leaves with one in flight
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
    tc_fence_after();
    tmem_dealloc(tmem, C::TMEM_COLS);
  }
}

// ------------------------------------------------------------------------------ dequantisation
// GGUF weight blocks -> fp16 [N][K], one warp per 256-element superblock, 8 elements per lane.
// Each value is the reference shader's fp32 expression evaluated in its order with one rounding
// per operation (no contraction), then rounded once to fp16. Reference formulas:
// QuantizationFormats.cs (DequantizeQ2K_Correct ... DequantizeQ6K_Correct), block layouts in the
// same file's header; f16 scales converted exactly.
__device__ __forceinline__ float h2f(const uint8_t* p) {
  return __half2float(__ushort_as_half(static_cast<unsigned short>(p[0] | (p[1] << 8))));
}

// K_SCALE unpacking of Q4_K / Q5_K (get_scale_min_k4): 6-bit scale and min of sub-block j.
__device__ __forceinline__ void scale_min_k4(int j, const uint8_t* q, float* sc, float* mn) {
  if (j < 4) {
    *sc = static_cast<float>(q[j] & 63);
    *mn = static_cast<float>(q[j + 4] & 63);
  } else {
    *sc = static_cast<float>((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
    *mn = static_cast<float>((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
  }
}

// d * sc * q - dmin * mn with the shader's association: ((d * sc) * q) - (dmin * mn)
__device__ __forceinline__ float affine(float d, float sc, float q, float dmin, float mn) {
  return __fsub_rn(__fmul_rn(__fmul_rn(d, sc), q), __fmul_rn(dmin, mn));
}

__device__ float dequant_one(int32_t wt, const uint8_t* blk, int e) {
  switch (wt) {
    case AIHOST_Q2_K: {  // scales[16] | qs[64] | d | dmin (84 bytes)
      const uint8_t sc = blk[e / 16];
      const int chunk = e / 128, local = e % 128;
      const int qv = (blk[16 + chunk * 32 + local % 32] >> ((local / 32) * 2)) & 3;
      return affine(h2f(blk + 80), static_cast<float>(sc & 0xF), static_cast<float>(qv), h2f(blk + 82),
                    static_cast<float>((sc >> 4) & 0xF));
    }
    case AIHOST_Q3_K: {  // hmask[32] | qs[64] | scales[12] | d (110 bytes)
      const int chunk = e / 128, local = e % 128;
      const int low2 = (blk[32 + chunk * 32 + local % 32] >> ((local / 32) * 2)) & 3;
      const int high1 = (blk[local % 32] >> (chunk * 4 + local / 32)) & 1;
      const int qval = (low2 | (high1 << 2)) - 4;
      const int is = e / 16, k = is % 4, ag = is / 4;
      const uint8_t* sc = blk + 96;
      const int tmp = sc[8 + k];
      int sb;
      if (ag == 0) sb = (sc[k] & 0xF) | (((tmp >> 0) & 3) << 4);
      else if (ag == 1) sb = (sc[k + 4] & 0xF) | (((tmp >> 2) & 3) << 4);
      else if (ag == 2) sb = ((sc[k] >> 4) & 0xF) | (((tmp >> 4) & 3) << 4);
      else sb = ((sc[k + 4] >> 4) & 0xF) | (((tmp >> 6) & 3) << 4);
      const float dl = __fmul_rn(h2f(blk + 108), static_cast<float>(sb - 32));
      return __fmul_rn(dl, static_cast<float>(qval));
    }
    case AIHOST_Q4_K: {  // d | dmin | scales[12] | qs[128] (144 bytes)
      const int group = e / 64, within = e % 64, upper = within >= 32 ? 1 : 0;
      float sc, mn;
      scale_min_k4(group * 2 + upper, blk + 4, &sc, &mn);
      const int q = (blk[16 + group * 32 + within % 32] >> (upper * 4)) & 0xF;
      return affine(h2f(blk), sc, static_cast<float>(q), h2f(blk + 2), mn);
    }
    case AIHOST_Q5_K: {  // d | dmin | scales[12] | qh[32] | qs[128] (176 bytes)
      float sc, mn;
      scale_min_k4(e / 32, blk + 4, &sc, &mn);
      const int j = e / 64, local = e % 64, upper = local >= 32 ? 1 : 0, l = local % 32;
      const int ql = (blk[48 + j * 32 + l] >> (upper * 4)) & 0xF;
      const int qh = (blk[16 + j * 32 + l] >> (j * 2 + upper)) & 1;
      return affine(h2f(blk), sc, static_cast<float>(ql | (qh << 4)), h2f(blk + 2), mn);
    }
    default: {  // AIHOST_Q6_K: ql[128] | qh[64] | scales[16] | d (210 bytes)
      const int half = e / 128, w = e % 128, quarter = w / 32, wq = w % 32;
      const int ql_extra = (quarter == 1 || quarter == 3) ? 32 : 0;
      const int upper = (quarter >= 2) ? 1 : 0;
      const int lower4 = (blk[half * 64 + ql_extra + wq] >> (upper * 4)) & 0xF;
      const int upper2 = (blk[128 + half * 32 + wq] >> (quarter * 2)) & 3;
      const int q = lower4 | (upper2 << 4);
      const float sc = static_cast<float>(static_cast<int8_t>(blk[192 + e / 16]));
      return __fmul_rn(__fmul_rn(h2f(blk + 208), sc), __fsub_rn(static_cast<float>(q), 32.0f));
    }
  }
}

// Lane l's eight values [8l, 8l + 8) of a 256-value block with vector loads: the same fp32
// operations as dequant_one (and the reference shaders), one load per field.
__device__ __forceinline__ void dequant8_q4k(const uint8_t* blk, int l, float (&v)[8]) {
  const uint32_t dw = *reinterpret_cast<const uint32_t*>(blk);  // 144-byte blocks are 16-byte aligned
  const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(dw & 0xffffu)));
  const float dmin = __half2float(__ushort_as_half(static_cast<unsigned short>(dw >> 16)));
  uint8_t sc8[12];
  *reinterpret_cast<uint32_t*>(sc8) = *reinterpret_cast<const uint32_t*>(blk + 4);
  *reinterpret_cast<uint32_t*>(sc8 + 4) = *reinterpret_cast<const uint32_t*>(blk + 8);
  *reinterpret_cast<uint32_t*>(sc8 + 8) = *reinterpret_cast<const uint32_t*>(blk + 12);
  float sc, mn;
  scale_min_k4(l >> 2, sc8, &sc, &mn);  // sub-block (l / 8) * 2 + upper == l / 4
  const uint2 q = *reinterpret_cast<const uint2*>(blk + 16 + (l >> 3) * 32 + (l & 3) * 8);
  const int shift = ((l & 7) >> 2) * 4;
  const float t = __fmul_rn(d, sc), dm = __fmul_rn(dmin, mn);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t byte = ((i < 4 ? q.x : q.y) >> ((i & 3) * 8)) & 0xffu;
    v[i] = __fsub_rn(__fmul_rn(t, static_cast<float>((byte >> shift) & 0xFu)), dm);
  }
}

__device__ __forceinline__ void dequant8_q5k(const uint8_t* blk, int l, float (&v)[8]) {
  const uint32_t dw = *reinterpret_cast<const uint32_t*>(blk);  // 176-byte blocks are 16-byte aligned
  const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(dw & 0xffffu)));
  const float dmin = __half2float(__ushort_as_half(static_cast<unsigned short>(dw >> 16)));
  uint8_t sc8[12];
  *reinterpret_cast<uint32_t*>(sc8) = *reinterpret_cast<const uint32_t*>(blk + 4);
  *reinterpret_cast<uint32_t*>(sc8 + 4) = *reinterpret_cast<const uint32_t*>(blk + 8);
  *reinterpret_cast<uint32_t*>(sc8 + 8) = *reinterpret_cast<const uint32_t*>(blk + 12);
  float sc, mn;
  scale_min_k4(l >> 2, sc8, &sc, &mn);
  const int j = l >> 3, upper = (l & 7) >> 2, off = j * 32 + (l & 3) * 8;
  const uint2 ql = *reinterpret_cast<const uint2*>(blk + 48 + off);
  const uint2 qh = *reinterpret_cast<const uint2*>(blk + 16 + off);  // the reference reads byte 16 + j*32 + l
  const int hb = j * 2 + upper;
  const float t = __fmul_rn(d, sc), dm = __fmul_rn(dmin, mn);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t lo = (((i < 4 ? ql.x : ql.y) >> ((i & 3) * 8)) >> (upper * 4)) & 0xFu;
    const uint32_t hi = (((i < 4 ? qh.x : qh.y) >> ((i & 3) * 8)) >> hb) & 1u;
    v[i] = __fsub_rn(__fmul_rn(t, static_cast<float>(lo | (hi << 4))), dm);
  }
}

__device__ __forceinline__ void dequant8_q6k(const uint8_t* blk, int l, float (&v)[8]) {
  // 210-byte blocks: 2-byte alignment only, so 16-bit loads
  const int half = l >> 4, quarter = (l & 15) >> 2, wq = (l & 3) * 8;
  const uint16_t* ql = reinterpret_cast<const uint16_t*>(blk + half * 64 + ((quarter & 1) ? 32 : 0) + wq);
  const uint16_t* qh = reinterpret_cast<const uint16_t*>(blk + 128 + half * 32 + wq);
  const int upper = quarter >> 1;
  const float t = __fmul_rn(h2f(blk + 208), static_cast<float>(static_cast<int8_t>(blk[192 + (l >> 1)])));
#pragma unroll
  for (int i2 = 0; i2 < 4; ++i2) {
    const uint32_t lw = ql[i2], hw = qh[i2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const uint32_t lo = ((lw >> (k * 8)) >> (upper * 4)) & 0xFu;
      const uint32_t hi = ((hw >> (k * 8)) >> (quarter * 2)) & 3u;
      v[2 * i2 + k] = __fmul_rn(t, __fsub_rn(static_cast<float>(lo | (hi << 4)), 32.0f));
    }
  }
}

template <typename T>
__global__ void __launch_bounds__(256) dequant_kernel(const uint8_t* __restrict__ w, int32_t wt, int64_t n_blocks,
                                                      int32_t block_bytes, T* __restrict__ out) {
  const int64_t blk = static_cast<int64_t>(blockIdx.x) * 8 + (threadIdx.x >> 5);
  if (blk >= n_blocks) return;
  const int lane = threadIdx.x & 31;
  const uint8_t* src = w + blk * block_bytes;
  float v[8];
  if (wt == AIHOST_Q4_K) dequant8_q4k(src, lane, v);
  else if (wt == AIHOST_Q5_K) dequant8_q5k(src, lane, v);
  else if (wt == AIHOST_Q6_K) dequant8_q6k(src, lane, v);
  else {
#pragma unroll
    for (int i = 0; i < 8; ++i) v[i] = dequant_one(wt, src, lane * 8 + i);
  }
  if constexpr (std::is_same<T, __half>::value) {
    *reinterpret_cast<uint4*>(out + blk * 256 + lane * 8) =
        make_uint4(pack2h(v[0], v[1]), pack2h(v[2], v[3]), pack2h(v[4], v[5]), pack2h(v[6], v[7]));
  } else {
    float4* d = reinterpret_cast<float4*>(out + blk * 256 + lane * 8);
    d[0] = make_float4(v[0], v[1], v[2], v[3]);
    d[1] = make_float4(v[4], v[5], v[6], v[7]);
  }
}

__global__ void __launch_bounds__(256) f32_to_f16_kernel(const float* __restrict__ x, __half* __restrict__ y,
                                                         int64_t n8) {
  for (int64_t i = static_cast<int64_t>(blockIdx.x) * 256 + threadIdx.x; i < n8; i += static_cast<int64_t>(gridDim.x) * 256) {
    const float4 a = __ldg(reinterpret_cast<const float4*>(x) + 2 * i);
    const float4 b = __ldg(reinterpret_cast<const float4*>(x) + 2 * i + 1);
    reinterpret_cast<uint4*>(y)[i] = make_uint4(pack2h(a.x, a.y), pack2h(a.z, a.w), pack2h(b.x, b.y), pack2h(b.z, b.w));
  }
}

template <int BN, bool SWAP, bool CL>
cudaError_t launch_gemm_bn(const GemmArgs& a, int grid, cudaStream_t st) {
  using C = GemmCfg<BN>;
  auto kern = gemm_kernel<BN, SWAP, CL>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(kGemmThreads, 1, 1);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  if (CL) {
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(a.k_splits);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
  }
  return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace

int32_t weight_block_bytes(int32_t wt) {
  switch (wt) {
    case AIHOST_Q2_K: return 84;
    case AIHOST_Q3_K: return 110;
    case AIHOST_Q4_K: return 144;
    case AIHOST_Q5_K: return 176;
    case AIHOST_Q6_K: return 210;
    default: return 0;
  }
}

cudaError_t launch_dequant(const void* w, int32_t wt, int64_t n_elems, void* out, int32_t out_dtype, cudaStream_t st) {
  const int64_t n_blocks = n_elems / 256;
  if (n_blocks == 0) return cudaSuccess;
  const unsigned grid = static_cast<unsigned>((n_blocks + 7) / 8);
  const uint8_t* src = static_cast<const uint8_t*>(w);
  if (out_dtype == AIHOST_F16)
    dequant_kernel<__half><<<grid, 256, 0, st>>>(src, wt, n_blocks, weight_block_bytes(wt), static_cast<__half*>(out));
  else
    dequant_kernel<float><<<grid, 256, 0, st>>>(src, wt, n_blocks, weight_block_bytes(wt), static_cast<float*>(out));
  return cudaGetLastError();
}

cudaError_t launch_f32_to_f16(const float* x, __half* y, int64_t n, int32_t num_sms, cudaStream_t st) {
  const int64_t n8 = n / 8;
  if (n8 == 0) return cudaSuccess;
  int64_t grid = (n8 + 255) / 256;
  if (grid > 8LL * num_sms) grid = 8LL * num_sms;
  f32_to_f16_kernel<<<static_cast<unsigned>(grid), 256, 0, st>>>(x, y, n8);
  return cudaGetLastError();
}

int32_t gemm_block_n(int32_t M, int32_t N, int32_t num_sms) {
  if (M <= 128) return M <= 64 ? -64 : -128;  // few rows: swapped operands, BN = rows of A
  const int64_t tiles256 = static_cast<int64_t>((M + kGBM - 1) / kGBM) * ((N + 255) / 256);
  return tiles256 >= num_sms ? 256 : 64;
}

int64_t gemm_tiles(int32_t M, int32_t N, int32_t block_n) {
  const bool swap = block_n < 0;
  const int bn = swap ? -block_n : block_n;
  const int R = swap ? N : M, NC = swap ? M : N;
  return static_cast<int64_t>((R + kGBM - 1) / kGBM) * ((NC + bn - 1) / bn);
}

cudaError_t launch_gemm(const GemmArgs& a, int32_t block_n, int32_t num_sms, cudaStream_t st) {
  if (a.k_splits < 1 || a.k_splits > kGemmMaxSplits || (a.k_splits & (a.k_splits - 1)) || (a.k_splits > 1 && block_n == 256))
    return cudaErrorInvalidValue;
  const int64_t tiles = gemm_tiles(a.M, a.N, block_n);
  if (a.k_splits > 1) {  // one CTA per (tile, split), clusters of k_splits
    const int grid = static_cast<int>(tiles * a.k_splits);
    switch (block_n) {
      case -64: return launch_gemm_bn<64, true, true>(a, grid, st);
      case -128: return launch_gemm_bn<128, true, true>(a, grid, st);
      default: return launch_gemm_bn<64, false, true>(a, grid, st);
    }
  }
  const int64_t per_sm = (block_n == 64 || block_n == -64) ? 2 : 1;
  const int grid = static_cast<int>(tiles < per_sm * num_sms ? tiles : per_sm * num_sms);
  switch (block_n) {
    case 256: return launch_gemm_bn<256, false, false>(a, grid, st);
    case -64: return launch_gemm_bn<64, true, false>(a, grid, st);
    case -128: return launch_gemm_bn<128, true, false>(a, grid, st);
    default: return launch_gemm_bn<64, false, false>(a, grid, st);
  }
}

}  // namespace aihost
