// kernels.h — host-side launch interface between the C-ABI layer (api.cu) and the kernels.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace aihost {

constexpr int kMaxHeadDim = 256;

// RoPE frequencies of one call, computed on the host as 1 / powf(theta, 2i / d) so that every
// kernel uses bit-identical angles (ComputeShaders.cs:536); passed by value.
struct RopeFreqs {
  float f[kMaxHeadDim / 2];
};

// Resolved cache geometry (bytes).
struct KvLayout {
  int64_t seq_stride, token_stride, head_stride;
  int32_t capacity;
  int32_t dtype;  // aihost_dtype
  // Paged cache (block_table non-NULL): row t of sequence b lives in the shared pool at row
  // block_table[b * max_pages + t / page_rows] * page_rows + t % page_rows; seq_stride unused.
  const int32_t* block_table;
  int32_t max_pages, page_rows, n_pages;
};

#ifdef __CUDACC__
// Pool row of (sequence b, row t) for a paged cache; t itself otherwise.
__device__ __forceinline__ int32_t kv_phys_row(const KvLayout& kv, int b, int32_t t) {
  return kv.block_table ? kv.block_table[static_cast<int64_t>(b) * kv.max_pages + t / kv.page_rows] * kv.page_rows +
                              t % kv.page_rows
                        : t;
}
// False when a paged cache's block table maps (b, t) outside the pool (the writers then skip the
// row and record a status bit; TMA reads of such rows return zeros).
__device__ __forceinline__ bool kv_row_ok(const KvLayout& kv, int b, int32_t t) {
  if (!kv.block_table) return true;
  const int32_t pg = kv.block_table[static_cast<int64_t>(b) * kv.max_pages + t / kv.page_rows];
  return pg >= 0 && pg < kv.n_pages;
}
// Byte offset of (sequence b, row t, head 0) from the cache base.
__device__ __forceinline__ int64_t kv_row_offset(const KvLayout& kv, int b, int32_t t) {
  return kv.block_table ? static_cast<int64_t>(kv_phys_row(kv, b, t)) * kv.token_stride
                        : b * kv.seq_stride + static_cast<int64_t>(t) * kv.token_stride;
}
#endif

// ---------------------------------------------------------------- rope_append.cu
// In-place RoPE of x [seq, n_heads, head_dim] (ApplyRoPEFull).
cudaError_t launch_rope_full(void* x, int32_t dtype, int32_t seq, int32_t n_heads, int32_t head_dim,
                             int32_t start_pos, int32_t rope_mode, const RopeFreqs& freqs, cudaStream_t st);

// In-place RMS norm of each row of x [seq, n_heads * head_dim] over the whole row (weight w
// [head_dim] device fp32, tiled over the heads), then RoPE at start_pos + s (Qwen TypeB prologue).
cudaError_t launch_qk_norm_rope(void* x, int32_t dtype, int32_t seq, int32_t n_heads, int32_t head_dim,
                                const float* w, float eps, int32_t start_pos, int32_t rope_mode, const RopeFreqs& freqs,
                                cudaStream_t st);

// Append k_new/v_new [batch][n_new][Hkv][d] into cache rows [seq_len[b], seq_len[b]+n_new),
// rotating K when rope_mode != NONE at position seq_len[b] + s, or rope_pos[b] + s when rope_pos
// (device, per sequence) is given. Records kStatusBadLength when a row would exceed capacity.
cudaError_t launch_kv_append(const void* k_new, const void* v_new, int32_t in_dtype, void* k_cache,
                             void* v_cache, const KvLayout& kv, const int32_t* seq_len, int32_t batch,
                             int32_t n_new, int32_t n_kv_heads, int32_t head_dim, int32_t rope_mode,
                             const RopeFreqs& freqs, int32_t* status, cudaStream_t st,
                             const int32_t* rope_pos = nullptr);

// fp16 staging for the prefill: q [batch][n_q][Hq][d] fp32 -> fp16, rotated at start_b + s
// (start_b = seq_len[b], or start_scalar when seq_len is NULL) unless rope_mode is NONE.
cudaError_t launch_stage_q(const float* q, __half* dst, const int32_t* seq_len, int32_t start_scalar, int32_t batch,
                           int32_t n_q, int32_t n_heads, int32_t head_dim, int32_t rope_mode, const RopeFreqs& freqs,
                           cudaStream_t st);
// Cache rows [0, start_b + len_offset) (at most `rows`) of an fp32 / Q8_0 cache -> dense fp16
// [batch][rows][Hkv][d] copies of K and V.
cudaError_t launch_stage_kv(const void* k_cache, const void* v_cache, const KvLayout& kv, __half* k_dst,
                            __half* v_dst, int32_t rows, const int32_t* seq_len, int32_t start_scalar,
                            int32_t len_offset, int32_t batch, int32_t n_kv_heads, int32_t head_dim, cudaStream_t st);

// ---------------------------------------------------------------- decode.cu
struct DecodeArgs {
  const void* q;            // [batch][Hq][d], q_dtype
  int32_t q_dtype;
  const void* k_cache;
  const void* v_cache;
  KvLayout kv;
  const int32_t* seq_len;   // device; NULL -> every sequence starts at start_scalar
  int32_t start_scalar;
  int32_t len_offset;       // attended rows = start + len_offset
  int32_t rope_pos_offset;  // q position = seq_len[b] + rope_pos_offset
  int32_t batch, n_q_heads, n_kv_heads, head_dim;
  float scale;
  int32_t rope_mode;
  RopeFreqs freqs;
  int32_t chunk;            // tokens per split
  int32_t max_splits;       // grid.x
  float* part_o;            // [batch][Hq][max_splits][d]   (scratch)
  float* part_ml;           // [batch][Hq][max_splits][2]   (scratch)
  void* out;                // [batch][Hq][d], out_dtype
  int32_t out_dtype;
  int32_t* status;
  // The new token's rows (forward decode): k_new / v_new [batch][Hkv][d] of new_dtype, appended at
  // row seq_len[b] (K rotated). NULL when the cache is already complete (mha).
  const void* k_new;
  const void* v_new;
  int32_t new_dtype;
  int32_t fuse_append;          // set by launch_decode_any: the kernel appends the rows itself
  // Fused combine (tensor-core kernels): per (sequence, blockIdx.y) arrival counters tagged with
  // the call's epoch; the last split to arrive merges the partials. NULL: combine kernel.
  unsigned long long* counters;
  uint32_t epoch;
  // Optional: q position per sequence (device; NULL -> seq_len[b] + rope_pos_offset), and
  // lse[b][h] = ln sum_j exp(scale * q.k_j) over the attended rows, written with the output.
  const int32_t* q_pos;
  float* lse;
  // Q8_0 caches, head groups of <= 8, batch <= 512: the stream-K schedule (one wave
  // of 2 CTAs per SM over the flattened cache tiles); part_o then holds q8_stream_k_bytes of
  // per-CTA partial slots. Set by the host (launch_decode_any keeps it only for TMA-able caches).
  int32_t stream_k;
  int32_t num_sms;
};
constexpr float kLn2 = 0.6931471805599453f;
// Arrival counters a fused combine may use (per (sequence, KV head, head group)).
constexpr int64_t kMaxSplitCounters = 1 << 16;
size_t decode_scratch_bytes(int32_t batch, int32_t n_q_heads, int32_t head_dim, int32_t max_splits);
// Split kernel; writes the output directly for sequences that fit in one split.
cudaError_t launch_decode(const DecodeArgs& a, cudaStream_t st);
// Merge of the per-split partials (only needed when max_splits > 1).
cudaError_t launch_decode_combine(const DecodeArgs& a, cudaStream_t st);
// Merge of n_parts normalised partial outputs of the same query rows over disjoint key sets:
// out[r] = sum_p o_p[r] * exp(lse_p[r] - lse[r]), lse[r] = ln sum_p exp(lse_p[r]).
// o_parts [n_parts][rows][head_dim] and out [rows][head_dim] of dtype (F32 / F16).
cudaError_t launch_merge_partials(int32_t n_parts, int64_t rows, int32_t head_dim, int32_t dtype,
                                  const void* o_parts, const float* lse_parts, void* out, float* lse_out,
                                  cudaStream_t st);

// ---------------------------------------------------------------- decode_mma.cu
// fp16-cache decode on the tensor cores: K/V maps over the cache with 64-row boxes.
struct DecodeMmaArgs {
  DecodeArgs base;
  CUtensorMap k_map;  // dims {d, Hkv, capacity, batch}, box {64, 1, 64, 1}, 128-byte swizzle
  CUtensorMap v_map;
};
cudaError_t launch_decode_mma(const DecodeMmaArgs& a, cudaStream_t st);
// Scratch of the stream-K Q8_0 decode: three per-warp partial slots of 8 heads per CTA (2 CTAs
// per SM).
size_t q8_stream_k_bytes(int32_t head_dim, int32_t num_sms);
constexpr int32_t kQ8StreamKMaxUnits = 512;
// Width in 32-bit words of the TMA box that holds one (token, head) slice of a Q8_0 cache whose
// heads are head_stride bytes apart (the narrowest 16-byte multiple every head offset fits).
uint32_t q8_box_words(int32_t head_dim, int64_t head_stride);

}  // namespace aihost
struct aihost_attn_ctx;
namespace aihost {
// Decode with whichever kernel fits the cache: the tensor-core kernels for fp16 / Q8_0 caches
// with TMA-compatible strides, the CUDA-core split kernel otherwise. Includes the new rows'
// append (when a.k_new is set) and the split merge, both fused into the tensor-core kernels when
// a group of query heads fits one CTA. Launches are timed by the context's profiler when ctx is
// non-NULL; the context also supplies the merge counters and epoch (with ctx NULL the caller
// sets a.counters / a.epoch, or leaves counters NULL for the combine kernel). Defined in api.cu.
cudaError_t launch_decode_any(DecodeArgs a, cudaStream_t st, aihost_attn_ctx* ctx);

// ---------------------------------------------------------------- prefill_sm100.cu
struct PrefillArgs {
  const void* q;            // [batch][S][Hq][d] fp16
  CUtensorMap q_map;        // dims {d, Hq, S, batch}
  CUtensorMap k_map;        // dims {d, Hkv, capacity, batch} over the cache
  CUtensorMap v_map;
  const int32_t* seq_len;   // device: rows cached before this call (start position)
  int32_t start_scalar;     // used when seq_len is NULL
  int32_t len_offset;       // attended rows = seq_len[b] + len_offset (n_new for forward, 0 for mha)
  int32_t batch, n_new, n_q_heads, n_kv_heads, head_dim;
  float scale;
  int32_t rope_mode;        // applied to Q inside the kernel
  RopeFreqs freqs;
  void* out;                // [batch][S][Hq][d]
  int32_t out_dtype;
  int32_t* status;
  int32_t split_kv;         // 1: the CTA's two softmax groups split one query tile's cache range
  int32_t q_early;          // 1: q is not written by the kernel launched just before this one
  // Paged cache (block_table non-NULL; page_rows a multiple of 128): k_map / v_map cover the
  // pool as one sequence, and cache tile j of sequence b is pool row
  // block_table[b * max_pages + j * 128 / page_rows] * page_rows + (j * 128) % page_rows.
  const int32_t* block_table;
  int32_t max_pages, page_rows;
};
bool prefill_supported(int32_t head_dim);
// Split mode pays off when pairing query tiles would leave SMs idle (about one wave or less).
bool prefill_split_kv(int32_t batch, int32_t n_new, int32_t n_q_heads, int32_t num_sms);
cudaError_t launch_prefill(const PrefillArgs& a, cudaStream_t st);

// ---------------------------------------------------------------- matmul_sm100.cu
// C[M, N] = A[M, K] . W[N, K]^T on the tensor cores (fp16 operands, fp32 accumulation).
struct GemmArgs {
  CUtensorMap a_map;   // fp16 A: dims {part_cols, M, n_parts}, box {64, 128 (BN when swapped), 1}, 128-byte swizzle
  CUtensorMap b_map;   // fp16 W: dims {K, N}, box {64, BN (128 when swapped)}, 128-byte swizzle
  int32_t M, N, K, part_cols;
  // K range split over the k_splits CTAs of a thread-block cluster (1: no split, persistent grid)
  int32_t k_splits;
  void* out;           // [M][ldc] in out_dtype
  int32_t out_dtype;
  int64_t ldc;
  int32_t* status;
  // AIHOST_F16: W through b_map. Q4_K / Q5_K: W's raw GGUF rows through w_raw_map (uint8 dims
  // {row bytes, N}, box {one super-block, 128 rows}), dequantised inside the GEMM (swapped form)
  int32_t w_type;
  CUtensorMap w_raw_map;
};
// Bytes of one 256-element GGUF block of a K-quant type (0 for other types).
int32_t weight_block_bytes(int32_t wt);
// GGUF K-quant blocks -> n_elems values (a multiple of 256) in out_dtype (F16 or F32).
cudaError_t launch_dequant(const void* w, int32_t wt, int64_t n_elems, void* out, int32_t out_dtype, cudaStream_t st);
cudaError_t launch_f32_to_f16(const float* x, __half* y, int64_t n, int32_t num_sms, cudaStream_t st);
// Output-tile width the GEMM uses for this shape: 256 when the tiles fill the SMs, else 64; for
// at most 128 rows of A, -64 / -128: the swapped form (weight rows in the MMA's M, BN rows of A).
int32_t gemm_block_n(int32_t M, int32_t N, int32_t num_sms);
// Output tiles of that shape and width.
int64_t gemm_tiles(int32_t M, int32_t N, int32_t block_n);
// True when a weight of this type is dequantised inside the GEMM for this output-tile width.
bool gemm_fuses_dequant(int32_t w_dtype, int32_t block_n);
cudaError_t launch_gemm(const GemmArgs& a, int32_t block_n, int32_t num_sms, cudaStream_t st);

}  // namespace aihost
