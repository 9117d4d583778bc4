// rows.cuh — one cache row (one token of one KV head) held by a warp: RoPE and the conversion
// into the cache's storage type. Shared by the append kernel and the decode kernels that append
// the new token themselves, so both produce identical cache bytes.
//
// Lane l holds elements [l*E, l*E + E) of the row, E = head_dim / 32.
#pragma once

#include "common.cuh"
#include "kernels.h"

namespace aihost {

// Rotation with explicitly rounded multiplies/adds (no FMA contraction), so a kernel and a CPU
// restatement that see the same cos/sin produce the same bits.
__device__ __forceinline__ void rotate_pair(float& x1, float& x2, float c, float s) {
  const float a = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
  const float b = __fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c));
  x1 = a;
  x2 = b;
}

__device__ __forceinline__ float freq_at(const RopeFreqs& f, int i) { return f.f[i]; }
__device__ __forceinline__ float freq_at(const float* f, int i) { return f[i]; }

// RoPE of the row at position `pos` (ComputeShaders.cs:517-543). Interleaved pairs (2i, 2i+1)
// sit in one lane; NEOX pairs (i, i + D/2) sit in lanes l and l ^ 16. `freqs` is the kernel's
// RopeFreqs or a copy of it in shared memory; the lanes read different pairs, and divergent
// reads of kernel parameters serialise per address, so hot kernels pass the shared copy.
template <int E, typename F>
__device__ __forceinline__ void rope_row_warp(float (&x)[E], int32_t lane, float pos, int32_t rope_mode,
                                              const F& freqs) {
  if (rope_mode == AIHOST_ROPE_INTERLEAVED) {
#pragma unroll
    for (int e = 0; e < E; e += 2) {
      const int pair = (lane * E + e) >> 1;
      float sn, cs;
      sincosf(__fmul_rn(pos, freq_at(freqs, pair)), &sn, &cs);
      rotate_pair(x[e], x[e + 1], cs, sn);
    }
  } else if (rope_mode == AIHOST_ROPE_NEOX) {
    const bool lo = lane < 16;
#pragma unroll
    for (int e = 0; e < E; ++e) {
      const float other = __shfl_xor_sync(0xffffffffu, x[e], 16);
      const int pair = (lane & 15) * E + e;
      float sn, cs;
      sincosf(__fmul_rn(pos, freq_at(freqs, pair)), &sn, &cs);
      float x1 = lo ? x[e] : other, x2 = lo ? other : x[e];
      rotate_pair(x1, x2, cs, sn);
      x[e] = lo ? x1 : x2;
    }
  }
}

// This lane's E elements of an fp32 or fp16 row as floats.
template <int E>
__device__ __forceinline__ void load_row_warp(const void* row, int32_t dtype, int32_t lane, float (&x)[E]) {
  if (dtype == AIHOST_F32) {
    const float* p = static_cast<const float*>(row) + lane * E;
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = p[e];
  } else {
    const __half* p = static_cast<const __half*>(row) + lane * E;
#pragma unroll
    for (int e = 0; e < E; ++e) x[e] = __half2float(p[e]);
  }
}

// Store the row at `dst` in the cache dtype: fp32 copy, fp16 round-to-nearest-even, or GGUF
// Q8_0 with ggml's reference quantiser (d = amax / 127, q = roundf(x * (1/d)), d stored as fp16;
// ggml quantize_row_q8_0_ref).
template <int E>
__device__ __forceinline__ void store_row_warp(const float (&x)[E], int32_t lane, uint8_t* dst, int32_t dtype) {
  if (dtype == AIHOST_F32) {
    float* d = reinterpret_cast<float*>(dst) + lane * E;
#pragma unroll
    for (int e = 0; e < E; ++e) d[e] = x[e];
  } else if (dtype == AIHOST_F16) {
    __half* d = reinterpret_cast<__half*>(dst) + lane * E;
#pragma unroll
    for (int e = 0; e < E; ++e) d[e] = __float2half_rn(x[e]);
  } else {  // Q8_0: 32 values per block = 32/E lanes
    constexpr int LPB = 32 / E;
    float amax = 0.0f;
#pragma unroll
    for (int e = 0; e < E; ++e) amax = fmaxf(amax, fabsf(x[e]));
#pragma unroll
    for (int off = 1; off < LPB; off <<= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
    const float dsc = __fdiv_rn(amax, 127.0f);
    const float id = dsc != 0.0f ? __frcp_rn(dsc) : 0.0f;
    const int blk = lane / LPB, sub = lane % LPB;
    // Every field is stored with 16-bit stores: the row base, the 34-byte block stride and the
    // 2-byte scale are all even, so each pair of bytes is 2-byte aligned.
    uint16_t* bp = reinterpret_cast<uint16_t*>(dst + blk * 34);
    if (sub == 0) bp[0] = __half_as_ushort(__float2half_rn(dsc));
#pragma unroll
    for (int e = 0; e < E; e += 2) {
      const uint32_t q0 = static_cast<uint8_t>(static_cast<int8_t>(roundf(__fmul_rn(x[e], id))));
      const uint32_t q1 = static_cast<uint8_t>(static_cast<int8_t>(roundf(__fmul_rn(x[e + 1], id))));
      bp[1 + (sub * E + e) / 2] = static_cast<uint16_t>(q0 | (q1 << 8));
    }
  }
}

}  // namespace aihost
