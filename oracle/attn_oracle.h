/*
 * attn_oracle.h — CPU restatement of AIHost's attention hot path.
 *
 * TEST INFRASTRUCTURE ONLY. Nothing in the product (libaihost_attn.so, aihost_b200/) links or
 * calls this code; only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg do,
 * as the checker and as the timed CPU reference.
 *
 * Restates, in plain C, the GLSL compute shaders and the C# host sequencing of the reference:
 *   RoPE            AIHost/AIHost/Compute/ComputeShaders.cs:517-543, ComputeOps.cs:959-979
 *   KV append       Inference/InferenceEngine.cs:598-622 (Concat axis 0, ComputeShaders.cs:353-381)
 *   decode          ComputeShaders.cs:656-733 (fused_mha_generate), ComputeOps.cs:1015-1043
 *   prefill         ComputeOps.cs:1076-1101: MatMul (ComputeShaders.cs:172-208), Scale (:487-497),
 *                   CausalMask (:545-561), RowwiseSoftmax (:429-485), MatMul, ScatterCols
 *   call order      ComputeOps.cs:1279-1304 (RoPE Q, RoPE K, KVCache.Add, Get, MultiHeadAttention)
 *
 * Modes:
 *   ORACLE_FAITHFUL (0): fp32 arithmetic in the shaders' order (256-way strided partial sums
 *     with a tree reduction for the softmax denominator, k-ascending dot products, j-ascending
 *     P.V), unfused multiply/add, the same constants (-1e38 mask / max seed, 1e-6 decode floor).
 *     Pinned bit-exactly against the reference's own shader source compiled for the CPU
 *     (oracle/ref_glsl).
 *   ORACLE_EXACT (1): the same math with double accumulation; the tolerance anchor.
 * Q8_0 follows the GGUF/ggml block format (ggml is not vendored by the reference; the
 * reference pins only the 34-byte block size, GGUF/GGUFTensorInfo.cs:64): ggml's reference
 * quantiser quantize_row_q8_0_ref (ggml 0.9.x): d = amax/127, id = d ? 1/d : 0,
 * q = roundf(x*id), scale stored as fp16(d).
 */
#ifndef AIHOST_ATTN_ORACLE_H
#define AIHOST_ATTN_ORACLE_H

#include <stdint.h>
#include "../include/aihost_attn.h"

#ifdef __cplusplus
extern "C" {
#endif

enum { ORACLE_FAITHFUL = 0, ORACLE_EXACT = 1 };

int32_t oracle_num_threads(void);
void oracle_set_num_threads(int32_t n); /* OpenMP threads of later calls (n > 0) */

/* IEEE binary16 <-> binary32, round-to-nearest-even. */
float oracle_f16_to_f32(uint16_t h);
uint16_t oracle_f32_to_f16(float f);
void oracle_f16_to_f32_n(const uint16_t* src, float* dst, int64_t n);
void oracle_f32_to_f16_n(const float* src, uint16_t* dst, int64_t n);

/* GGUF Q8_0: n % 32 == 0, blocks = n/32 * 34 bytes. */
void oracle_q8_0_quantize(const float* x, int64_t n, uint8_t* blocks);
void oracle_q8_0_dequantize(const uint8_t* blocks, int64_t n, float* x);

/* RoPE frequency of pair i: 1 / powf(theta, (float)(2i) / (float)head_dim) (ComputeShaders.cs:536). */
float oracle_rope_freq(float theta, int32_t pair, int32_t head_dim);
/* ApplyRoPEFull on x [seq, n_heads*head_dim] fp32, positions start_pos + s. */
void oracle_rope_full(float* x, int32_t seq, int32_t n_heads, int32_t head_dim, int32_t start_pos,
                      float theta, int32_t rope_mode);

/* Qwen TypeB Q/K prologue (Compute/Formats/QwenHybridFormat.cs:141-142): ComputeOps.LayerNorm
 * (ComputeOps.cs:517-542, shader ComputeShaders.cs:249-277) of each token row of x
 * [seq, n_heads*head_dim] over the whole row, with the per-head weight w [head_dim] tiled over the
 * heads (TransformerBase.cs:301-319), then ApplyRoPEFull at start_pos. The sum of squares follows
 * the shader's order: 256 strided partial sums, then a halving tree. */
void oracle_qk_norm_rope(float* x, int32_t seq, int32_t n_heads, int32_t head_dim, const float* w, float eps,
                         int32_t start_pos, float theta, int32_t rope_mode);

/* MultiHeadAttention over fp32 K/V that are already rotated.
 * q [n_q, Hq*d], out [n_q, Hq*d]; k/v row r, head h at k[r*kv_row_stride + h*d].
 * n_q == 1: FusedMHAGenerate; n_q > 1: per-head causal chain with j > start_pos + i masked. */
int32_t oracle_mha(const float* q, const float* k, const float* v, int64_t kv_row_stride,
                   int32_t n_q, int32_t n_kv, int32_t n_q_heads, int32_t n_kv_heads,
                   int32_t head_dim, int32_t start_pos, float scale, int32_t mode, float* out);

/* The fused forward of aihost_attn_forward on host memory with identical argument meaning:
 * RoPE(q), RoPE(k_new), append into the caches (converted / quantised to kv_dtype), then
 * attention over rows [0, seq_len[b] + n_new). Caches are modified. Returns 0 on success. */
int32_t oracle_attn_forward(const aihost_attn_desc* desc, int32_t batch, int32_t n_new,
                            const void* q, const void* k_new, const void* v_new, void* k_cache,
                            void* v_cache, const int32_t* seq_len, void* out, int32_t mode);

/* Same, restricted to query heads [h0, h1) and sequences [b0, b1) (bounded CPU-baseline
 * samples); caches are still appended for the KV heads those query heads use. */
int32_t oracle_attn_forward_part(const aihost_attn_desc* desc, int32_t batch, int32_t n_new,
                                 const void* q, const void* k_new, const void* v_new,
                                 void* k_cache, void* v_cache, const int32_t* seq_len, void* out,
                                 int32_t mode, int32_t b0, int32_t b1, int32_t h0, int32_t h1);
/* As oracle_attn_forward_part, attending only query rows [r0, r1) of every selected sequence and
 * head (the append still covers all n_new rows): samples of long prefills. */
int32_t oracle_attn_forward_rows(const aihost_attn_desc* desc, int32_t batch, int32_t n_new,
                                 const void* q, const void* k_new, const void* v_new,
                                 void* k_cache, void* v_cache, const int32_t* seq_len, void* out,
                                 int32_t mode, int32_t b0, int32_t b1, int32_t h0, int32_t h1,
                                 int32_t r0, int32_t r1);

/* GGUF K-quant weights (kind = AIHost DataType ordinal: Q2_K 8, Q3_K 9, Q4_K 10, Q5_K 11, Q6_K 12):
 * bytes per 256-value block, and n values (a multiple of 256) dequantised to fp32 with the
 * reference shaders' formulas (QuantizationFormats.cs). */
int32_t oracle_kquant_block_bytes(int32_t kind);
int32_t oracle_dequantize(int32_t kind, const uint8_t* blocks, int64_t n, float* out);
/* ComputeOps.MatMulWeights: C [M, N] = A [M, K] . W with W given as w[n * K + k] (GGUF
 * column-major); mode ORACLE_FAITHFUL (fp32, k ascending) or ORACLE_EXACT (double). */
int32_t oracle_matmul_weights(const float* a, int32_t M, int32_t K, const float* w, int32_t N, float* c, int32_t mode);

#ifdef __cplusplus
}
#endif

#endif
