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
// WQ forms: warps 8-11 join warps 4-7 in dequantising (two threads per weight row)
__host__ __device__ constexpr int gemm_threads(int wq) { return wq == 0 ? kGemmThreads : kGemmThreads + 128; }
constexpr int kGemmMaxSplits = 8;  // largest portable cluster
constexpr int kGBM = 128;  // rows of A per tile (TMEM lanes)
constexpr int kGBK = 64;   // K per stage: one 128-byte swizzle row of fp16

// Bytes of one row's 256-value super-block for the weight types dequantised inside the GEMM.
__host__ __device__ constexpr int fused_block_bytes(int wq) {
  return wq == AIHOST_Q4_K ? 144 : wq == AIHOST_Q5_K ? 176 : 0;
}

// WQ = 0: NS stages, each one A tile and one B tile by TMA (STAGE apart, B A_BYTES after A).
// WQ = Q4_K / Q5_K (swapped: the MMA's A operand is the weight): the raw super-blocks of 128
// weight rows by TMA into a two-deep raw ring; the dequantising warps write each fp16 weight tile
// into tensor memory (row r in TMEM lane r, 32 columns per 64-wide K tile, a two-deep ring after
// the accumulators), which the MMA reads as its A operand; the TMA keeps NS activation tiles in
// flight in shared memory (B_STEP apart from offset 0). The ring sizes leave room for the CL
// partial tile.
template <int BN, int WQ = 0>
struct GemmCfg {
  static constexpr int NS = WQ == 0 ? 4 : (BN == 128 ? 6 : 4);  // WQ: activation tiles only
  static constexpr int NSA = 4;  // WQ: weight tiles in tensor memory
  static constexpr int A_BYTES = kGBM * kGBK * 2;
  static constexpr int B_BYTES = BN * kGBK * 2;
  static constexpr int STAGE = A_BYTES + B_BYTES;
  static constexpr int B_OFF = WQ == 0 ? A_BYTES : 0;
  static constexpr int B_STEP = WQ == 0 ? STAGE : B_BYTES;  // between consecutive B tiles
  static constexpr int RAW_ROW = fused_block_bytes(WQ);
  static constexpr int RAW_STAGE = kGBM * RAW_ROW;
  static constexpr int RAW_OFF = WQ == 0 ? NS * STAGE : NS * B_BYTES;
  static constexpr int BAR_OFF = RAW_OFF + 2 * RAW_STAGE;
  static constexpr int SMEM = BAR_OFF + 512 + 1024;
  static constexpr uint32_t A_COL = 2 * BN;  // WQ: first TMEM column of the weight-tile ring
  // powers of two >= 32: two accumulators (+ the WQ weight tiles)
  static constexpr uint32_t TMEM_COLS = WQ == 0 ? 2 * BN : (BN == 64 ? 256 : 512);
  static_assert(WQ == 0 || A_COL + NSA * 32 <= TMEM_COLS, "weight-tile ring exceeds the TMEM allocation");
};

struct GemmBars {
  uint64_t full[8], empty[8], acc_full[2], acc_empty[2];
  uint64_t slices_in;                  // CL: the peers' slices of this CTA's output rows have landed
  uint64_t raw_full[2], raw_empty[2];  // WQ: raw super-block ring
  uint64_t a_full[4], a_empty[4];      // WQ: dequantised weight-tile ring
  uint32_t tmem_base;
};
static_assert(sizeof(GemmBars) <= 512, "gemm_kernel reserves 512 bytes for its barriers");

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

__device__ __forceinline__ float2 fmul2_rn(float2 a, float2 b) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n mul.rn.f32x2 rd, ra, rb;\n"
      " mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
__device__ __forceinline__ float2 fadd2_rn(float2 a, float2 b) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n add.rn.f32x2 rd, ra, rb;\n"
      " mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

// Eight fp16 weights (t * q) - dm from the eight unsigned quants held in the bytes of w0 and w1:
// each byte becomes the float 2^23 + q exactly (byte permute under exponent 0x4B), minus 2^23
// gives q; then the dequantisation shaders' two fp32 roundings, then one rounding to fp16, the
// same values dequant_kernel writes.
__device__ __forceinline__ uint4 dequant_chunk8(uint32_t w0, uint32_t w1, float t, float dm) {
  const float2 shift = make_float2(-8388608.0f, -8388608.0f), tt = make_float2(t, t), ndm = make_float2(-dm, -dm);
  uint32_t h[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const uint32_t w = i < 2 ? w0 : w1, b = (i & 1) * 2;
    const float2 q = fadd2_rn(make_float2(__uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u | b)),
                                          __uint_as_float(__byte_perm(w, 0x4B000000u, 0x7540u | (b + 1)))),
                              shift);
    const float2 v = fadd2_rn(fmul2_rn(tt, q), ndm);
    h[i] = pack2h(v.x, v.y);
  }
  return make_uint4(h[0], h[1], h[2], h[3]);
}

// Byte i (0..11) of the 12 scale bytes held in words y, z, w of a Q4_K / Q5_K block header.
__device__ __forceinline__ uint32_t scale_byte(const uint4& hdr, int i) {
  const uint32_t word = i < 4 ? hdr.y : (i < 8 ? hdr.z : hdr.w);
  return (word >> ((i & 3) * 8)) & 0xffu;
}
// get_scale_min_k4 on the header in registers (the integer steps of scale_min_k4 below).
__device__ __forceinline__ void scale_min_k4_hdr(int j, const uint4& hdr, float* sc, float* mn) {
  if (j < 4) {
    *sc = static_cast<float>(scale_byte(hdr, j) & 63);
    *mn = static_cast<float>(scale_byte(hdr, j + 4) & 63);
  } else {
    *sc = static_cast<float>((scale_byte(hdr, j + 4) & 0xF) | ((scale_byte(hdr, j - 4) >> 6) << 4));
    *mn = static_cast<float>((scale_byte(hdr, j + 4) >> 4) | ((scale_byte(hdr, j) >> 6) << 4));
  }
}

// Half `hf` of one weight row's 64 values of K tile `quarter` (0..3) of a raw Q4_K / Q5_K
// super-block in shared memory (hf 0: tile values 0..31, the low nibbles; hf 1: values 32..63,
// the high ones) as 16 fp16 pairs, value 2i in the low half of out[i]. The fields and formulas are
// dequant8_q4k's / dequant8_q5k's (including the Q5_K high-bit offset the reference shader uses).
template <int WQ>
__device__ __forceinline__ void dequant_row_half(const uint8_t* raw_row, int quarter, int hf, uint32_t (&out)[16]) {
  const uint4 hdr = *reinterpret_cast<const uint4*>(raw_row);
  const float d = __half2float(__ushort_as_half(static_cast<unsigned short>(hdr.x & 0xffffu)));
  const float dmin = __half2float(__ushort_as_half(static_cast<unsigned short>(hdr.x >> 16)));
  float sc, mn;
  scale_min_k4_hdr(2 * quarter + hf, hdr, &sc, &mn);
  const float t = __fmul_rn(d, sc), dm = __fmul_rn(dmin, mn);
  constexpr int QL = WQ == AIHOST_Q4_K ? 16 : 48;  // low-bit quants of K tile 0
  const uint4* ql = reinterpret_cast<const uint4*>(raw_row + QL + 32 * quarter);
  const uint4 qa = ql[0], qb = ql[1];
  const uint32_t w[8] = {qa.x, qa.y, qa.z, qa.w, qb.x, qb.y, qb.z, qb.w};
  uint32_t hb[8];
  if constexpr (WQ == AIHOST_Q5_K) {
    const uint4* qh = reinterpret_cast<const uint4*>(raw_row + 16 + 32 * quarter);
    const uint4 ha = qh[0], hbv = qh[1];
    hb[0] = ha.x; hb[1] = ha.y; hb[2] = ha.z; hb[3] = ha.w;
    hb[4] = hbv.x; hb[5] = hbv.y; hb[6] = hbv.z; hb[7] = hbv.w;
  }
  const int nshift = 4 * hf, hshift = 2 * quarter + hf;
#pragma unroll
  for (int c = 0; c < 4; ++c) {
    uint32_t q0 = (w[2 * c] >> nshift) & 0x0F0F0F0Fu, q1 = (w[2 * c + 1] >> nshift) & 0x0F0F0F0Fu;
    if constexpr (WQ == AIHOST_Q5_K) {
      q0 |= ((hb[2 * c] >> hshift) & 0x01010101u) << 4;
      q1 |= ((hb[2 * c + 1] >> hshift) & 0x01010101u) << 4;
    }
    const uint4 h = dequant_chunk8(q0, q1, t, dm);
    out[4 * c] = h.x;
    out[4 * c + 1] = h.y;
    out[4 * c + 2] = h.z;
    out[4 * c + 3] = h.w;
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
//
// WQ (Q4_K / Q5_K, swapped CL form only): the weight stays in its GGUF blocks in HBM. The producer
// moves the raw super-block of the tile's 128 weight rows (one row per 144 / 176-byte box row)
// into a two-deep raw ring every four K tiles, and each activation tile into the operand ring;
// the four epilogue warps, idle until the accumulator is ready, dequantise one weight row each
// into the operand tile and arrive on its full barrier with the producer.
template <int BN, bool SWAP, bool CL, int WQ>
__global__ void __launch_bounds__(gemm_threads(WQ), BN == 64 ? 2 : 1) gemm_kernel(const __grid_constant__ GemmArgs a) {
  using C = GemmCfg<BN, WQ>;
  static_assert(WQ == 0 || (SWAP && CL), "weights are dequantised in the GEMM only in the swapped split-K form");
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
      mbar_init(&bar.raw_full[i], 1);
      mbar_init(&bar.raw_empty[i], 8);  // the eight dequantising warps
    }
    for (int i = 0; i < C::NSA; ++i) {
      mbar_init(&bar.a_full[i], 8);
      mbar_init(&bar.a_empty[i], 1);
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
      if constexpr (WQ != 0) tma_prefetch_desc(&a.w_raw_map);
      else tma_prefetch_desc(&a.b_map);
      int g = 0;
      bool ok = true;
      for (int u = blockIdx.x; ok && u < units; u += gridDim.x) {
        int mt, nt, kt0, kt1;
        unit_coords(u, mt, nt, kt0, kt1);
        for (int kt = kt0; kt < kt1; ++kt, ++g) {
          if constexpr (WQ != 0) {
            if (((kt - kt0) & 3) == 0) {  // a new super-block (K ranges start on one)
              const int lsb = (kt - kt0) >> 2, rs = lsb & 1;
              if (!mbar_wait(&bar.raw_empty[rs], ((lsb >> 1) & 1) ^ 1, status)) { ok = false; break; }
              mbar_arrive_expect_tx(&bar.raw_full[rs], C::RAW_STAGE);
              tma_load_2d(smem + C::RAW_OFF + rs * C::RAW_STAGE, &a.w_raw_map, &bar.raw_full[rs], (kt >> 2) * C::RAW_ROW,
                          mt * kGBM);
            }
          }
          const int s = g % C::NS;
          if (!mbar_wait(&bar.empty[s], ((g / C::NS) & 1) ^ 1, status)) { ok = false; break; }
          uint8_t* st = smem + s * C::STAGE;
          const int k = kt * kGBK;
          if constexpr (WQ != 0) {  // the activation ring; the weight tiles come from the dequantising warps
            mbar_arrive_expect_tx(&bar.full[s], C::B_BYTES);
            tma_load_3d(smem + C::B_OFF + s * C::B_BYTES, &a.a_map, &bar.full[s], k % a.part_cols, nt * BN,
                        k / a.part_cols);
            continue;
          }
          mbar_arrive_expect_tx(&bar.full[s], C::STAGE);
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
      // descriptors of the ring's first tiles; a tile's K step adds its byte offset / 16 to the
      // 14-bit start-address field (shared addresses stay below 2^18, so it never carries)
      const uint64_t a_desc0 = make_sw128_desc(base, 16, 1024), b_desc0 = make_sw128_desc(base + C::B_OFF, 16, 1024);
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
          const int s = g % C::NS, sw = g % C::NSA;
          if (!mbar_wait(&bar.full[s], (g / C::NS) & 1, status)) { ok = false; break; }
          if (WQ != 0 && !mbar_wait(&bar.a_full[sw], (g / C::NSA) & 1, status)) { ok = false; break; }
          tc_fence_after();
          const uint64_t ad = a_desc0 + static_cast<uint64_t>((s * C::STAGE) >> 4);
          const uint64_t bd = b_desc0 + static_cast<uint64_t>((s * C::B_STEP) >> 4);
#pragma unroll
          for (int kk = 0; kk < kGBK / 16; ++kk) {
            if constexpr (WQ != 0)  // the weight tile from tensor memory: 16 values = 8 columns per K step
              umma_f16_ts(d, tmem + C::A_COL + sw * 32 + kk * 8, bd + 2 * kk, idesc, (kt > kt0 || kk > 0) ? 1u : 0u);
            else
              umma_f16_ss(d, ad + 2 * kk, bd + 2 * kk, idesc, (kt > kt0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&bar.empty[s]);
          if constexpr (WQ != 0) umma_commit(&bar.a_empty[sw]);
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
    const int hf = warp >= 8 ? 1 : 0;                    // WQ: which half of weight row r
    if constexpr (WQ != 0) {
      // ---------------------------------------------------------------- weight dequantisation
      int mt, nt, kt0, kt1;
      unit_coords(blockIdx.x, mt, nt, kt0, kt1);
      bool ok = true;
      for (int kt = kt0, g = 0; ok && kt < kt1; ++kt, ++g) {
        const int lsb = (kt - kt0) >> 2, rs = lsb & 1, sw = g % C::NSA;
        if (((kt - kt0) & 3) == 0) ok = mbar_wait(&bar.raw_full[rs], (lsb >> 1) & 1, status);
        if (ok) ok = mbar_wait(&bar.a_empty[sw], ((g / C::NSA) & 1) ^ 1, status);
        // the vote keeps the tcgen05.st warp-collective (a lane that gave up leaves the warp with it)
        ok = __all_sync(0xffffffffu, ok);
        if (ok) {
          tc_fence_after();  // the MMA that read this slot is complete
          uint32_t h[16];
          dequant_row_half<WQ>(smem + C::RAW_OFF + rs * C::RAW_STAGE + r * C::RAW_ROW, kt & 3, hf, h);
          tmem_st16(tmem + lane_base + C::A_COL + sw * 32 + hf * 16, h);
          tmem_wait_st();
          tc_fence_before();
        }
        __syncwarp();
        if (ok && lane == 0) mbar_arrive(&bar.a_full[sw]);
        if (ok && ((kt & 3) == 3 || kt + 1 == kt1) && lane == 0) mbar_arrive(&bar.raw_empty[rs]);
      }
    }
    int j = 0;
    for (int u = blockIdx.x; hf == 0 && u < units; u += gridDim.x, ++j) {
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
    for (int e = threadIdx.x; ok && e < slice_floats; e += gemm_threads(WQ)) {
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

template <int BN, bool SWAP, bool CL, int WQ = 0>
cudaError_t launch_gemm_bn(const GemmArgs& a, int grid, cudaStream_t st) {
  using C = GemmCfg<BN, WQ>;
  auto kern = gemm_kernel<BN, SWAP, CL, WQ>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::SMEM);
  if (e != cudaSuccess) return e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(gemm_threads(WQ), 1, 1);
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

bool gemm_fuses_dequant(int32_t w_dtype, int32_t block_n) {
  return block_n < 0 && (w_dtype == AIHOST_Q4_K || w_dtype == AIHOST_Q5_K);
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
  if (a.w_type != AIHOST_F16) {  // raw K-quant weight, dequantised in the GEMM (swapped, clusters)
    const int grid = static_cast<int>(tiles * a.k_splits);
    if (block_n == -64 && a.w_type == AIHOST_Q4_K) return launch_gemm_bn<64, true, true, AIHOST_Q4_K>(a, grid, st);
    if (block_n == -64 && a.w_type == AIHOST_Q5_K) return launch_gemm_bn<64, true, true, AIHOST_Q5_K>(a, grid, st);
    if (block_n == -128 && a.w_type == AIHOST_Q4_K) return launch_gemm_bn<128, true, true, AIHOST_Q4_K>(a, grid, st);
    if (block_n == -128 && a.w_type == AIHOST_Q5_K) return launch_gemm_bn<128, true, true, AIHOST_Q5_K>(a, grid, st);
    return cudaErrorInvalidValue;
  }
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
