// prefill_sm100.cu — causal prefill attention on the 5th-generation tensor cores.
//
// Replaces the prefill branch of ComputeOps.MultiHeadAttention (ComputeOps.cs:1076-1101): per
// Q head the reference slices Q/K/V, materialises K^T and the [S, Lk] fp32 score matrix in
// global memory, scales, masks (j > P + i -> -1e38), runs a three-pass row softmax and a
// second fp32 GEMM — about ten dispatches per head, each followed by a fence wait.
//
// Here one CTA owns two 128-row query tiles of one Q head and streams the KV head's cache rows
// in 128-row tiles (flash attention, online softmax); scores never leave the SM:
//   warp 0      TMA producer: both Q tiles once, then K and V tiles into 2-3 stage rings
//               (no multicast anywhere)
//   warps 1, 2  TMEM owner (warp 1) and tcgen05.mma issuers: per cache tile j a group's
//               O += P V_j and S = Q K_{j+1}^T, so one softmax group's exponentials overlap
//               the other group's matrix products (ping-pong). D = 64: one issuing thread per
//               group (warps 1 and 2); D = 128: warp 1 issues for both groups in turn. S and O accumulate in TMEM (fp32); P (fp16) goes back to TMEM and
//               the P.V MMA reads it from there (A operand in TMEM, V from shared memory).
//   warps 4-7   softmax group A (query tile A), warps 8-11 group B: one thread per query row.
//               RoPE of the Q tile in shared memory; per tile tcgen05.ld of S, row max, lazy
//               rescale of O (only when the running max grows by more than 2^8), exp2 on the
//               SFU, fp16 P via tcgen05.st; causal masking only on tiles that cross the
//               diagonal or the end of the sequence; final O / l epilogue.
// Tile pairing: a CTA takes adjacent query tiles 2x and 2x+1, so both softmax groups stay busy
// for the CTA's whole life (the ping-pong needs two live groups); CTAs with the longest causal
// ranges launch first. Cache tiles above a tile's diagonal are never loaded or multiplied.
// For head_dim 64, P has its own TMEM columns, so the next QK^T can overwrite S as soon as the
// softmax has read it, ahead of this tile's P.V; for 128 P is written over S (no spare columns).
// One thread's stream of tcgen05.mma (M = 128, K = 16) advances about one instruction per
// 100-120 cycles whatever N is up to 128, hence one issuing thread per softmax group.
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace aihost {
namespace {

constexpr int kBM = 128;  // query rows per tile
constexpr int kBN = 128;  // cache rows per tile
// Three warpgroups: WG0 = producer warp, MMA issuer warps, spare warps; WG1 / WG2 = softmax
// groups A / B (a full 128-column score row stays in registers).
constexpr int kThreads = 384;
// setmaxnreg split of the 168 x 384 registers the CTA launches with: producer / MMA warpgroup
// 72, each softmax warpgroup 216 (128 * 72 + 2 * 128 * 216 = 168 * 384).
constexpr uint32_t kRegsWG0 = 72;
constexpr uint32_t kRegsSoftmax = 216;
static_assert(128 * kRegsWG0 + 2 * 128 * kRegsSoftmax <= 168 * kThreads, "setmaxnreg split exceeds the launch");
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleThreshold = 8.0f;  // log2 units

template <int D>
struct PrefillCfg {
  static constexpr int KB = D / 64;                  // 64-element (128-byte) column blocks
  static constexpr int TILE_BYTES = KB * kBN * 128;  // one [128 x D] fp16 tile
  static constexpr int NS = D == 64 ? 3 : 2;         // K and V ring depth
  static constexpr int QA_OFF = 0;
  static constexpr int QB_OFF = QA_OFF + TILE_BYTES;
  static constexpr int K_OFF = QB_OFF + TILE_BYTES;
  static constexpr int V_OFF = K_OFF + NS * TILE_BYTES;
  // P in its own TMEM columns (D = 64: S 128 + P 64 + O 64 columns per group), else over S
  static constexpr bool P_SEP = D == 64;
  static constexpr int BAR_OFF = V_OFF + NS * TILE_BYTES;
  static constexpr int SMEM = BAR_OFF + 256 + 1024;  // barriers + alignment slack
  static constexpr uint32_t TMEM_COLS = 512;
  // TMEM columns: S_A, S_B (fp32), then P_A, P_B (fp16 pairs) and O_A, O_B for D = 64; for
  // D = 128, O_A, O_B after S, with P aliased onto the first 64 columns of its S
  static __device__ __forceinline__ uint32_t s_col(int t) { return t ? 128u : 0u; }
  static __device__ __forceinline__ uint32_t p_col(int t) {
    return P_SEP ? 256u + static_cast<uint32_t>(t * 64) : s_col(t);
  }
  static __device__ __forceinline__ uint32_t o_col(int t) {
    return (P_SEP ? 384u : 256u) + static_cast<uint32_t>(t * D);
  }
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
  uint64_t q_full;
  uint64_t q_ready[2], s_full[2], p_full[2], o_full[2];
  uint64_t k_full[3], k_empty[3], v_full[3], v_empty[3];
  uint64_t s_free[2], pv_done[2];  // separate P: S read into registers / P.V complete
  uint64_t v_fix;  // last V tile's rows past the sequence end have been zeroed
  uint32_t tmem_base;
};
static_assert(sizeof(Barriers) <= 256, "prefill_kernel reserves 256 bytes for its barriers");

__device__ __forceinline__ uint32_t pack_half2(float lo, float hi) {
  const __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// Packed fp32 pairs (sm_100): one instruction for two lanes' worth of IEEE fma / add.
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n mov.b64 rc, {%6, %7};\n"
      " fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 fadd2(float2 a, float2 b) {
  float2 d;
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n add.rn.f32x2 rd, ra, rb;\n"
      " mov.b64 {%0, %1}, rd;\n}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}
// max of three (sm_100 three-input form; a NaN operand is ignored like fmaxf)
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

template <int D>
__global__ void __launch_bounds__(kThreads, 1) prefill_kernel(const __grid_constant__ PrefillArgs a) {
  using C = PrefillCfg<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Barriers& bar = *reinterpret_cast<Barriers*>(smem + C::BAR_OFF);
  uint8_t* q_s[2] = {smem + C::QA_OFF, smem + C::QB_OFF};
  uint8_t* k_s = smem + C::K_OFF;
  uint8_t* v_s = smem + C::V_OFF;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n_qt = (a.n_new + kBM - 1) / kBM;
  // grid: (sequence x head, work rank) with the heads fastest, so CTAs dispatch in order of
  // decreasing causal work across all heads and sequences
  const int h = static_cast<int>(blockIdx.x) % a.n_q_heads, b = static_cast<int>(blockIdx.x) / a.n_q_heads;
  const int kvh = h / (a.n_q_heads / a.n_kv_heads);
  // Pair mode: adjacent query tiles 2x and 2x+1 (B absent past the end), both groups read the
  // same K/V tile j. Split mode: both groups take query tile x, group A cache tiles [0, n/2),
  // group B [n/2, n), merged at the end. The longest work launches first in both.
  const bool split = a.split_kv != 0;
  const int x = static_cast<int>(gridDim.y) - 1 - static_cast<int>(blockIdx.y);
  const int qt[2] = {split ? x : 2 * x, split ? x : 2 * x + 1};
  const bool has_b = split || qt[1] < n_qt;
  const int32_t start = a.seq_len ? a.seq_len[b] : a.start_scalar;
  const int32_t Lk = start + a.len_offset;
  const bool bad = Lk < 1 || start < 0;
  int n_kv[2], kv_lo[2] = {0, 0};
#pragma unroll
  for (int t = 0; t < 2; ++t) {
    const int32_t kv_end = min(Lk, start + qt[t] * kBM + kBM);  // rows j <= start + q0 + 127, j < Lk
    n_kv[t] = (t == 1 && !has_b) || kv_end <= 0 ? 0 : (kv_end + kBN - 1) / kBN;
  }
  if (split) {
    const int n = n_kv[0];
    n_kv[0] = n / 2;
    n_kv[1] = n - n / 2;
    kv_lo[1] = n / 2;
  }
  // K/V tiles loaded, in load order: pair mode tile j at step j; split mode A0, B0, A1, B1, ...
  // (B has at most one tile more than A, loaded last).
  const int n_load = split ? n_kv[0] + n_kv[1] : max(n_kv[0], n_kv[1]);
  auto load_index = [&](int t, int j) -> int {
    if (!split) return j;
    return j < n_kv[0] ? 2 * j + t : 2 * n_kv[0] + (j - n_kv[0]);
  };
  int32_t* status = a.status;

  if (threadIdx.x == 0) {
    mbar_init(&bar.q_full, 1);
    for (int t = 0; t < 2; ++t) {
      mbar_init(&bar.q_ready[t], split && t == 0 ? 256 : 128);
      mbar_init(&bar.s_full[t], 1);
      mbar_init(&bar.p_full[t], 128);
      mbar_init(&bar.o_full[t], 1);
      mbar_init(&bar.s_free[t], 128);
      mbar_init(&bar.pv_done[t], 1);
    }
    mbar_init(&bar.v_fix, 1);
    // a ring slot is free once every issuing thread that reads its tile is done with it: both
    // issuers when two threads share the tiles (pair mode, D = 64; group B's one extra last
    // tile is never reloaded), else one commit per slot use
    const int readers = C::P_SEP && !split && has_b ? 2 : 1;
    for (int i = 0; i < C::NS; ++i) {
      mbar_init(&bar.k_full[i], 1);
      mbar_init(&bar.k_empty[i], readers);
      mbar_init(&bar.v_full[i], 1);
      mbar_init(&bar.v_empty[i], readers);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(&bar.tmem_base, C::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = bar.tmem_base;

  if (bad) {
    if (threadIdx.x == 0 && x == 0 && h == 0) atomicOr(status, kStatusBadLength);
  } else if (warp < 4) {
    regs_dealloc<kRegsWG0>();
    if (warp == 0) {
    // ------------------------------------------------------------------ TMA producer
    if (lane == 0) {
      tma_prefetch_desc(&a.q_map);
      tma_prefetch_desc(&a.k_map);
      tma_prefetch_desc(&a.v_map);
      // Q may be read before the preceding kernel finishes when that kernel does not write it;
      // the cache rows (appended or staged by the preceding kernel) only after griddep_wait.
      const int n_q_tiles = has_b && !split ? 2 : 1;
      auto load_q = [&] {
        mbar_arrive_expect_tx(&bar.q_full, n_q_tiles * C::TILE_BYTES);
        for (int t = 0; t < n_q_tiles; ++t)
          for (int kb = 0; kb < C::KB; ++kb)
            tma_load_4d((t ? q_s[1] : q_s[0]) + kb * kBM * 128, &a.q_map, &bar.q_full, kb * 64, h,
                        (t ? qt[1] : qt[0]) * kBM, b);
      };
      if (a.q_early) load_q();
      griddep_wait();
      if (!a.q_early) load_q();
      for (int g = 0; g < n_load; ++g) {
        // cache tile of load g: pair mode g; split mode A's g/2, B's, then B's last
        const int tile = !split ? g : g < 2 * n_kv[0] ? ((g & 1) ? kv_lo[1] : 0) + (g >> 1) : g;
        const int s = g % C::NS;
        const uint32_t par = ((g / C::NS) & 1) ^ 1;
        // paged cache: the 128-row tile lies inside one page of the pool (sequence coordinate 0)
        const int row = a.block_table ? a.block_table[static_cast<int64_t>(b) * a.max_pages + tile * kBN / a.page_rows] *
                                                a.page_rows + (tile * kBN) % a.page_rows
                                      : tile * kBN;
        const int bc = a.block_table ? 0 : b;
        if (!mbar_wait(&bar.k_empty[s], par, status)) break;
        mbar_arrive_expect_tx(&bar.k_full[s], C::TILE_BYTES);
        for (int kb = 0; kb < C::KB; ++kb)
          tma_load_4d(k_s + s * C::TILE_BYTES + kb * kBN * 128, &a.k_map, &bar.k_full[s], kb * 64, kvh, row, bc);
        if (!mbar_wait(&bar.v_empty[s], par, status)) break;
        mbar_arrive_expect_tx(&bar.v_full[s], C::TILE_BYTES);
        for (int kb = 0; kb < C::KB; ++kb)
          tma_load_4d(v_s + s * C::TILE_BYTES + kb * kBN * 128, &a.v_map, &bar.v_full[s], kb * 64, kvh, row, bc);
      }
    }
    // Cache rows >= Lk in the last V tile may hold stale bits (NaN patterns included); P is 0
    // there, but 0 * NaN is NaN, so the whole warp zeroes them before any P.V reads the tile.
    __syncwarp();
    const int jl = n_load - 1;
    if (jl >= 0 && (jl + 1) * kBN > Lk) {
      const int s = jl % C::NS;
      if (mbar_wait(&bar.v_full[s], (jl / C::NS) & 1, status)) {
        uint8_t* vt = v_s + s * C::TILE_BYTES;
        const int first = max(Lk - jl * kBN, 0);
        const int chunks = (kBN - first) * C::KB * 8;  // 16-byte chunks to clear
        for (int i = lane; i < chunks; i += 32) {
          const int row = first + i / (C::KB * 8), ch = i % (C::KB * 8);
          *reinterpret_cast<uint4*>(vt + (ch >> 3) * (kBN * 128) + row * 128 + (ch & 7) * 16) = make_uint4(0, 0, 0, 0);
        }
        fence_proxy_async_smem();
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&bar.v_fix);
    }
    } else if (warp == 1 || warp == 2) {
    // ------------------------------------------------------------------ MMA issuers
    // A thread's tcgen05.mma stream advances by about one M = 128, K = 16 instruction per
    // 100-120 cycles whatever N is, so with P in its own columns (D = 64) each softmax group gets
    // its own issuing thread (warp 1: A, warp 2: B). With P over S (D = 128) a group's next QK^T
    // must follow its P.V anyway; there warp 1 alone issues both groups' products in turn, which
    // keeps the groups half a step apart (one group's exponentials overlap the other's products).
    // Each group's products stay in issue order on one thread.
    constexpr bool kTwo = C::P_SEP;
    if (lane == 0 && (kTwo || warp == 1)) {
      const int t_lo = kTwo ? warp - 1 : 0;
      constexpr uint32_t idesc_qk = make_idesc_f16(kBM, kBN, 0, 0);
      constexpr uint32_t idesc_pv = make_idesc_f16(kBM, D, 0, 1);
      const uint32_t k_addr = smem_u32(k_s), v_addr = smem_u32(v_s);
      const uint32_t q_addr0 = smem_u32(q_s[0]), q_addr1 = smem_u32(q_s[split ? 0 : 1]);
      // per-group values by selection, not by indexing with a run-time t (no local memory on
      // the issuing thread, whose latency paces the tensor pipe)
      auto nkv = [&](int t) { return t ? n_kv[1] : n_kv[0]; };
      // S_t = Q_t K^T with the K tile in ring slot s
      auto issue_qk = [&](int t, int s) {
        const uint32_t qa = t ? q_addr1 : q_addr0;
#pragma unroll
        for (int kk = 0; kk < D / 16; ++kk) {
          const uint32_t off = (kk >> 2) * (kBN * 128) + (kk & 3) * 32;
          umma_f16_ss(tmem + C::s_col(t), make_sw128_desc(qa + off, 16, 1024),
                      make_sw128_desc(k_addr + s * C::TILE_BYTES + off, 16, 1024), idesc_qk, kk > 0);
        }
        umma_commit(&bar.s_full[t]);
      };
      // O_t (+)= P_t V with P in TMEM and the V tile in ring slot s; j = the group's tile count
      auto issue_pv = [&](int t, int j, int s) {
#pragma unroll
        for (int kk = 0; kk < kBN / 16; ++kk) {
          const uint64_t vd = make_sw128_desc(v_addr + s * C::TILE_BYTES + kk * 2048, kBN * 128, 1024);
          umma_f16_ts(tmem + C::o_col(t), tmem + C::p_col(t) + kk * 8, vd, idesc_pv, (j > 0 || kk > 0) ? 1u : 0u);
        }
      };
      // wait for the K tile of group t's step j; its ring slot in s
      auto k_ready = [&](int t, int j, int& s) -> bool {
        const int g = load_index(t, j);
        s = g % C::NS;
        return mbar_wait(&bar.k_full[s], (g / C::NS) & 1, status);
      };
      if constexpr (kTwo) {
        // this thread's group T: P.V of cache tile j and, as soon as the softmax has read S(j)
        // (P has its own columns), the QK^T of tile j + 1 ahead of it
        auto run_group = [&](auto T) {
          constexpr int t = decltype(T)::value;
          const int nk = nkv(t);
          int s0 = 0;
          bool ok = mbar_wait(&bar.q_ready[split ? 0 : t], 0, status) && k_ready(t, 0, s0);
          if (ok) {
            tc_fence_after();
            issue_qk(t, s0);
            umma_commit(&bar.k_empty[s0]);
          }
          for (int j = 0; ok && j < nk; ++j) {
            const int gv = load_index(t, j), sv = gv % C::NS;
            if (j + 1 < nk) {
              int sk = 0;
              if (!mbar_wait(&bar.s_free[t], j & 1, status) || !k_ready(t, j + 1, sk)) break;
              tc_fence_after();
              issue_qk(t, sk);
              umma_commit(&bar.k_empty[sk]);
            }
            if (!mbar_wait(&bar.v_full[sv], (gv / C::NS) & 1, status)) break;
            if (gv == n_load - 1 && n_load * kBN > Lk && !mbar_wait(&bar.v_fix, 0, status)) break;
            if (!mbar_wait(&bar.p_full[t], j & 1, status)) break;
            tc_fence_after();
            issue_pv(t, j, sv);
            umma_commit(&bar.pv_done[t]);
            umma_commit(&bar.v_empty[sv]);
            if (j + 1 == nk) umma_commit(&bar.o_full[t]);
          }
        };
        if (nkv(t_lo) > 0) {
          if (t_lo == 0) run_group(std::integral_constant<int, 0>{});
          else run_group(std::integral_constant<int, 1>{});
        }
      } else {
        // one thread, both groups in turn; P over S, so a group's next QK^T follows its P.V
        bool ok = mbar_wait(&bar.q_ready[0], 0, status);
        if (ok && has_b && !split) ok = mbar_wait(&bar.q_ready[1], 0, status);
        tc_fence_after();
        if (split) {
          // each group walks its own cache tiles; slots follow the producer's load order
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            int s0 = 0;
            if (!ok || n_kv[t] == 0) continue;
            ok = k_ready(t, 0, s0);
            tc_fence_after();
            if (ok) {
              issue_qk(t, s0);
              umma_commit(&bar.k_empty[s0]);
            }
          }
          const int steps = max(n_kv[0], n_kv[1]);
          for (int j = 0; ok && j < steps; ++j) {
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              if (!ok || j >= n_kv[t]) continue;
              const int gv = load_index(t, j), sv = gv % C::NS;
              const bool next = j + 1 < n_kv[t];
              int sk = 0;
              if (!mbar_wait(&bar.v_full[sv], (gv / C::NS) & 1, status)) { ok = false; break; }
              if (gv == n_load - 1 && n_load * kBN > Lk && !mbar_wait(&bar.v_fix, 0, status)) { ok = false; break; }
              if (next && !k_ready(t, j + 1, sk)) { ok = false; break; }
              if (!mbar_wait(&bar.p_full[t], j & 1, status)) { ok = false; break; }
              tc_fence_after();
              issue_pv(t, j, sv);
              umma_commit(&bar.v_empty[sv]);
              if (next) {
                issue_qk(t, sk);
                umma_commit(&bar.k_empty[sk]);
              } else {
                umma_commit(&bar.o_full[t]);
              }
            }
          }
        } else {
          // pair mode: both groups read cache tile j from the same ring slot
          if (ok && n_load > 0) {
            ok = mbar_wait(&bar.k_full[0], 0, status);
            tc_fence_after();
            if (ok && n_kv[0] > 0) issue_qk(0, 0);
            if (ok && n_kv[1] > 0) issue_qk(1, 0);
            if (ok) umma_commit(&bar.k_empty[0]);
          }
          for (int j = 0; ok && j < n_load; ++j) {
            const int s = j % C::NS;
            const int s1 = (j + 1) % C::NS;
            // operands first (normally long resident), then the softmax hand-offs
            if (!mbar_wait(&bar.v_full[s], (j / C::NS) & 1, status)) { ok = false; break; }
            if (j == n_load - 1 && n_load * kBN > Lk && !mbar_wait(&bar.v_fix, 0, status)) { ok = false; break; }
            if (j + 1 < n_load && !mbar_wait(&bar.k_full[s1], ((j + 1) / C::NS) & 1, status)) { ok = false; break; }
            tc_fence_after();
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              if (j >= n_kv[t]) continue;
              if (!mbar_wait(&bar.p_full[t], j & 1, status)) { ok = false; break; }
              tc_fence_after();
              issue_pv(t, j, s);
              if (j + 1 < n_kv[t]) issue_qk(t, s1);
              else umma_commit(&bar.o_full[t]);
            }
            if (!ok) break;
            umma_commit(&bar.v_empty[s]);
            if (j + 1 < n_load) umma_commit(&bar.k_empty[s1]);
          }
        }
      }
    }
    }
  } else {
    regs_alloc<kRegsSoftmax>();
    // ------------------------------------------------------------------ softmax groups
    const int t = warp >= 8 ? 1 : 0;
    const int quarter = warp & 3;
    const int r = quarter * 32 + lane;  // query row within the tile == TMEM lane
    const uint32_t lane_base = static_cast<uint32_t>(quarter * 32) << 16;
    const int nk = t ? n_kv[1] : n_kv[0];
    const int kv_first = t ? kv_lo[1] : 0;
    const int q0 = (t ? qt[1] : qt[0]) * kBM;
    uint8_t* const q_tile = split || t == 0 ? q_s[0] : q_s[1];
    const int32_t qpos = start + q0 + r;      // absolute position of this query row
    const int32_t limit = min(qpos, Lk - 1);  // last visible cache row
    const bool active = t == 0 || has_b;
    bool ok = true;
    if (active) {
      // In split mode both groups share Q tile A and each rotates half of its pairs.
      const int qb = split ? 0 : t;
      ok = mbar_wait(&bar.q_full, 0, status);
      if (ok && a.rope_mode != AIHOST_ROPE_NONE) {
        // whole 16-byte chunks of the swizzled row (8 consecutive elements): a quarter-warp's
        // 8 rows hit 8 distinct bank groups. In split mode each group rotates half the chunks.
        const float pos = static_cast<float>(qpos);
        auto rot = [&](uint32_t& w1, uint32_t& w2, int pair) {  // w1 / w2: the pair's two halves
          float sn, cs;
          sincos_reduced(pos * a.freqs.f[pair], &sn, &cs);
          const float x1 = __half2float(*reinterpret_cast<const __half*>(&w1));
          const float x2 = __half2float(*reinterpret_cast<const __half*>(&w2));
          const __half y1 = __float2half_rn(x1 * cs - x2 * sn), y2 = __float2half_rn(x1 * sn + x2 * cs);
          w1 = __half_as_ushort(y1);
          w2 = __half_as_ushort(y2);
        };
        constexpr int NC = D / 8;  // 16-byte chunks per row
        if (a.rope_mode == AIHOST_ROPE_NEOX) {  // chunk c pairs with chunk c + NC/2, element by element
          const int c0 = split ? t * (NC / 4) : 0, c1 = split ? c0 + NC / 4 : NC / 2;
          for (int c = c0; c < c1; ++c) {
            uint4* pa = reinterpret_cast<uint4*>(q_tile + sw128_off(r, 8 * c, kBM));
            uint4* pb = reinterpret_cast<uint4*>(q_tile + sw128_off(r, 8 * (c + NC / 2), kBM));
            uint4 va = *pa, vb = *pb;
            uint32_t* ua = reinterpret_cast<uint32_t*>(&va);
            uint32_t* ub = reinterpret_cast<uint32_t*>(&vb);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              uint32_t a0 = ua[k] & 0xffffu, a1 = ua[k] >> 16, b0 = ub[k] & 0xffffu, b1 = ub[k] >> 16;
              rot(a0, b0, 8 * c + 2 * k);
              rot(a1, b1, 8 * c + 2 * k + 1);
              ua[k] = a0 | (a1 << 16);
              ub[k] = b0 | (b1 << 16);
            }
            *pa = va;
            *pb = vb;
          }
        } else {  // interleaved: the 4 pairs (2i, 2i + 1) of a chunk sit in its four 32-bit words
          const int c0 = split ? t * (NC / 2) : 0, c1 = split ? c0 + NC / 2 : NC;
          for (int c = c0; c < c1; ++c) {
            uint4* pc = reinterpret_cast<uint4*>(q_tile + sw128_off(r, 8 * c, kBM));
            uint4 v = *pc;
            uint32_t* u = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
            for (int k = 0; k < 4; ++k) {
              uint32_t lo = u[k] & 0xffffu, hi = u[k] >> 16;
              rot(lo, hi, 4 * c + k);
              u[k] = lo | (hi << 16);
            }
            *pc = v;
          }
        }
      }
      fence_proxy_async_smem();
      mbar_arrive(&bar.q_ready[qb]);
    }

    const float sl2 = a.scale * kLog2e;
    float m = -1e30f, l = 0.0f;  // running max (log2 units) and denominator
    const uint32_t s_tmem = tmem + lane_base + C::s_col(t);
    const uint32_t o_tmem = tmem + lane_base + C::o_col(t);
    const uint32_t p_tmem = tmem + lane_base + C::p_col(t);
    for (int j = 0; active && ok && j < nk; ++j) {
      if (!mbar_wait(&bar.s_full[t], j & 1, status)) { ok = false; break; }
      tc_fence_after();
      uint32_t sr[4][32];
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_ld32(s_tmem + c * 32, sr[c]);
      tmem_wait_ld();
      if constexpr (C::P_SEP) {  // S is in registers: the next QK^T may overwrite it
        tc_fence_before();
        mbar_arrive(&bar.s_free[t]);
      }
      const int kv0 = (kv_first + j) * kBN;
      const bool need_mask = __any_sync(0xffffffffu, kv0 + kBN - 1 > limit);
      if (need_mask) {
#pragma unroll
        for (int c = 0; c < 4; ++c)
#pragma unroll
          for (int i = 0; i < 32; ++i)
            if (kv0 + c * 32 + i > limit) sr[c][i] = __float_as_uint(-INFINITY);
      }
      // row max: three-input maxima into independent partials (instruction-level parallelism)
      float mxp[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mxp[i] = -INFINITY;
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 16; ++i)
          mxp[i & 7] = fmax3(mxp[i & 7], __uint_as_float(sr[c][2 * i]), __uint_as_float(sr[c][2 * i + 1]));
      const float mx = fmax3(fmax3(mxp[0], mxp[1], mxp[2]), fmax3(mxp[3], mxp[4], mxp[5]), fmaxf(mxp[6], mxp[7]));
      const float m_new = fmaxf(m, mx * sl2);
      const bool resc = m_new > m + kRescaleThreshold;
      const float f = resc ? ex2_approx(m - m_new) : 1.0f;
      if (resc) {
        l *= f;
        m = m_new;
      }
      // P = 2^(s*scale*log2e - m) in fp16 (masked entries: 2^-inf = 0), from S in registers; the
      // scale-and-subtract and the row sums run on packed fp32 pairs
      const float2 sl2x2 = make_float2(sl2, sl2), neg_m2 = make_float2(-m, -m);
      float2 rsp[4] = {make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f), make_float2(0.0f, 0.0f),
                       make_float2(0.0f, 0.0f)};
      uint32_t pk[4][16];
#pragma unroll
      for (int c = 0; c < 4; ++c)
#pragma unroll
        for (int i = 0; i < 16; ++i) {
          const float2 x = ffma2(make_float2(__uint_as_float(sr[c][2 * i]), __uint_as_float(sr[c][2 * i + 1])), sl2x2,
                                 neg_m2);
          const float2 pp = make_float2(ex2_approx(x.x), ex2_approx(x.y));
          rsp[i & 3] = fadd2(rsp[i & 3], pp);
          pk[c][i] = pack_half2(pp.x, pp.y);
        }
      l += ((rsp[0].x + rsp[0].y) + (rsp[1].x + rsp[1].y)) + ((rsp[2].x + rsp[2].y) + (rsp[3].x + rsp[3].y));
      // O and the separate P of the previous tile: the previous P.V may still be running (the next
      // QK^T was issued ahead of it), so wait for it; with P over S, this tile's S was committed
      // after it, which already orders it.
      if constexpr (C::P_SEP) {
        if (j > 0 && !mbar_wait(&bar.pv_done[t], (j - 1) & 1, status)) { ok = false; break; }
        tc_fence_after();
      }
      // The vote keeps the tcgen05.ld/st warp-collective; rows that keep their max use f = 1.
      if (j > 0 && __any_sync(0xffffffffu, resc)) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o[32];
          tmem_ld32(o_tmem + c * 32, o);
          tmem_wait_ld();
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * f);
          tmem_st32(o_tmem + c * 32, o);
        }
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) tmem_st16(p_tmem + c * 16, pk[c]);
      tmem_wait_st();  // the O rescale and P complete before the next P.V reads them
      tc_fence_before();
      mbar_arrive(&bar.p_full[t]);
    }
    // ---- epilogue: O / l -> out[b][q0 + r][h][:]
    const bool valid = q0 + r < a.n_new;
    const int64_t orow = ((static_cast<int64_t>(b) * a.n_new + q0 + r) * a.n_q_heads + h) * D;
    auto store32 = [&](int c, const float (&o)[32]) {
      if (!valid) return;
      if (a.out_dtype == AIHOST_F16) {
        uint4* dst = reinterpret_cast<uint4*>(static_cast<__half*>(a.out) + orow + c * 32);
#pragma unroll
        for (int v = 0; v < 4; ++v)
          dst[v] = make_uint4(pack_half2(o[8 * v], o[8 * v + 1]), pack_half2(o[8 * v + 2], o[8 * v + 3]),
                              pack_half2(o[8 * v + 4], o[8 * v + 5]), pack_half2(o[8 * v + 6], o[8 * v + 7]));
      } else {
        float4* dst = reinterpret_cast<float4*>(static_cast<float*>(a.out) + orow + c * 32);
#pragma unroll
        for (int v = 0; v < 8; ++v) dst[v] = make_float4(o[4 * v], o[4 * v + 1], o[4 * v + 2], o[4 * v + 3]);
      }
    };
    if (split) {
      // Merge the two groups' partial softmax states of the same rows: (m, l) through shared
      // memory (Q tile B's space, unused in this mode), O from both TMEM blocks. Each group writes
      // half of the output columns.
      float* ml = reinterpret_cast<float*>(q_s[1]);
      ml[(t * kBM + r) * 2] = m;
      ml[(t * kBM + r) * 2 + 1] = l;
      asm volatile("bar.sync 1, 256;" ::: "memory");
      bool ready = ok;
      if (ready && n_kv[0] > 0) ready = mbar_wait(&bar.o_full[0], 0, status);
      if (ready) ready = mbar_wait(&bar.o_full[1], 0, status);
      if (__all_sync(0xffffffffu, ready)) {
        tc_fence_after();
        const float mA = ml[r * 2], lA = ml[r * 2 + 1];
        const float mB = ml[(kBM + r) * 2], lB = ml[(kBM + r) * 2 + 1];
        const float mm = fmaxf(mA, mB);
        const float aA = n_kv[0] > 0 ? ex2_approx(mA - mm) : 0.0f;
        const float aB = ex2_approx(mB - mm);
        const float L = lA * aA + lB * aB;
        const float inv = L > 0.0f ? 1.0f / L : 0.0f;
        const float fA = aA * inv, fB = aB * inv;
        const uint32_t oa_tmem = tmem + lane_base + C::o_col(0), ob_tmem = tmem + lane_base + C::o_col(1);
#pragma unroll
        for (int cc = 0; cc < D / 64; ++cc) {
          const int c = t * (D / 64) + cc;
          uint32_t ob[32], oa[32];
          tmem_ld32(ob_tmem + c * 32, ob);
          if (n_kv[0] > 0) tmem_ld32(oa_tmem + c * 32, oa);
          tmem_wait_ld();
          float o[32];
#pragma unroll
          for (int i = 0; i < 32; ++i)
            o[i] = __uint_as_float(ob[i]) * fB + (n_kv[0] > 0 ? __uint_as_float(oa[i]) * fA : 0.0f);
          store32(c, o);
        }
      }
    } else if (active && ok && nk > 0 && mbar_wait(&bar.o_full[t], 0, status)) {
      tc_fence_after();
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t ou[32];
        tmem_ld32(o_tmem + c * 32, ou);
        tmem_wait_ld();
        float o[32];
#pragma unroll
        for (int i = 0; i < 32; ++i) o[i] = __uint_as_float(ou[i]) * inv;
        store32(c, o);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    __syncwarp();
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
  const int n_qt = (a.n_new + kBM - 1) / kBM;
  // programmatic launch: the CTAs' set-up overlaps the tail of the kernel before (append or
  // staging), which signals griddepcontrol.launch_dependents; the producer waits for it in full
  // before reading the cache
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(a.n_q_heads * a.batch, a.split_kv ? n_qt : (n_qt + 1) / 2, 1);
  cfg.blockDim = dim3(kThreads);
  cfg.dynamicSmemBytes = C::SMEM;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, a);
}

}  // namespace

bool prefill_supported(int32_t head_dim) { return head_dim == 64 || head_dim == 128; }

bool prefill_split_kv(int32_t batch, int32_t n_new, int32_t n_q_heads, int32_t num_sms) {
  const int64_t n_qt = (n_new + kBM - 1) / kBM;
  const int64_t pair_ctas = (n_qt + 1) / 2 * n_q_heads * static_cast<int64_t>(batch);
  return pair_ctas < 2LL * num_sms;
}

cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t st) {
  return a.head_dim == 64 ? launch_d<64>(a, st) : launch_d<128>(a, st);
}

}  // namespace aihost
