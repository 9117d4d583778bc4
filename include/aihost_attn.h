/*
 * aihost_attn.h — C ABI of libaihost_attn.so, the B200 (sm_100a) attention op for AIHost.
 *
 * This library replaces, for one hot path, what AIHost's C# compute layer does through
 * `ComputeOps` on a GPU backend:
 *
 *   ApplyRoPEFull(Q) ; ApplyRoPEFull(K) ; KVCache.Add(layer, K, V) ; KVCache.Get(layer) ;
 *   MultiHeadAttention(Q, cachedK, cachedV, numHeads, position)
 *
 * (AIHost/AIHost/Compute/ComputeOps.cs:1279-1304, Formats/CombinedQKVFormat.cs:52-67,
 *  Formats/QwenHybridFormat.cs:141-145). The reference dispatches these as GLSL compute shaders
 * through Vulkan; its CUDA backend (ICompute/CUDA/CudaComputeCommandQueue.cs:56-61) cannot
 * dispatch at all. A C# host binds the functions below with [DllImport("aihost_attn")].
 *
 * Conventions (mirroring ICompute/CUDA/CudaApi.cs:11-92, where every native call returns an
 * error enum that the caller checks):
 *   - every function returns an aihost_status; no exception or abort crosses the ABI;
 *   - aihost_attn_last_error() gives a thread-local message for the last failure;
 *   - all tensor pointers are raw device pointers (CUdeviceptr, IComputeBuffer.GetPointer()),
 *     owned by the caller; the library never frees or retains them past the call;
 *   - work is enqueued on the caller's cudaStream_t (passed as void*, NULL = legacy stream);
 *     calls are asynchronous with respect to the host, like Dispatch() before Flush();
 *   - the library allocates nothing inside the attention calls: split-K scratch is owned by
 *     the context and sized once by aihost_attn_reserve().
 *
 * Layouts (reference KVCache, Inference/InferenceEngine.cs:582-625, is one fp32 tensor
 * [rows, n_kv_heads*head_dim] per layer for K and one for V, token-major):
 *   q, out          [batch][n_new][n_q_heads][head_dim]      (= reference [S, Hq*d] per sequence)
 *   k_new, v_new    [batch][n_new][n_kv_heads][head_dim]
 *   k_cache,v_cache element (b, t, h, i) at byte offset
 *                     b*kv_seq_stride + t*kv_token_stride + h*kv_head_stride + bytes(i)
 *                   defaults (strides 0): token-major, kv_capacity rows per sequence.
 *   Q8_0 caches hold GGUF blocks {fp16 d; int8 qs[32]} (34 bytes per 32 values,
 *   GGUF/GGUFTensorInfo.cs:64), head_dim/32 blocks per (token, head).
 */
#ifndef AIHOST_ATTN_H
#define AIHOST_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define AIHOST_ATTN_ABI_VERSION 1

typedef enum {
  AIHOST_OK = 0,
  AIHOST_EINVAL = 1,        /* bad argument: null pointer, bad dims, misaligned pointer, ... */
  AIHOST_ENOMEM = 2,        /* context reservation failed, or scratch too small for a call */
  AIHOST_ECUDA = 3,         /* a CUDA runtime/driver call failed */
  AIHOST_ETIMEOUT = 4,      /* a bounded device-side wait expired (status word set by a kernel) */
  AIHOST_EUNSUPPORTED = 5,  /* valid request this build does not implement (e.g. head_dim 96) */
  AIHOST_ENCCL = 6          /* a collective failed */
} aihost_status;

/* Element types; the numeric values are AIHost's DataType ordinals
 * (ICompute/IComputeBuffer.cs:57-76: F32=0, F16=1, Q8_0=6, Q2_K=8 ... Q6_K=12). The K-quant
 * types are GGUF weight blocks of 256 values (QuantizationFormats.cs header: Q2_K 84 bytes,
 * Q3_K 110, Q4_K 144, Q5_K 176, Q6_K 210) and are accepted as weights only. */
typedef enum {
  AIHOST_F32 = 0, AIHOST_F16 = 1, AIHOST_Q8_0 = 6,
  AIHOST_Q2_K = 8, AIHOST_Q3_K = 9, AIHOST_Q4_K = 10, AIHOST_Q5_K = 11, AIHOST_Q6_K = 12
} aihost_dtype;

/* RoPE pairing. INTERLEAVED is the reference's (x[2i], x[2i+1]) pairing used by every
 * architecture in AIHost (Compute/ComputeShaders.cs:517-543). NEOX pairs (x[i], x[i+d/2]).
 * NONE skips rotation (inputs already rotated). */
typedef enum { AIHOST_ROPE_INTERLEAVED = 0, AIHOST_ROPE_NEOX = 1, AIHOST_ROPE_NONE = 2 } aihost_rope_mode;

/* One attention layer's static description. The fields are the GGUF metadata the reference
 * reads in Compute/TransformerBase.cs:72-80 (head_count, head_count_kv, rope.freq_base). */
typedef struct {
  int32_t n_q_heads;        /* Hq */
  int32_t n_kv_heads;       /* Hkv; Hq % Hkv == 0, Q head h uses KV head h / (Hq/Hkv) */
  int32_t head_dim;         /* d: 64 or 128 in this build */
  float rope_theta;         /* frequency base; LlamaFormat passes none and gets 10000 */
  int32_t rope_mode;        /* aihost_rope_mode */
  float scale;              /* 0 -> 1/sqrtf(head_dim), as ComputeOps.cs:1065 */
  int32_t q_dtype;          /* dtype of q, k_new, v_new: F32 or F16 */
  int32_t kv_dtype;         /* cache dtype: F32, F16 or Q8_0 */
  int32_t out_dtype;        /* F32 or F16 */
  int32_t kv_capacity;      /* rows allocated per sequence in the cache */
  int64_t kv_seq_stride;    /* bytes between sequences; 0 -> kv_capacity * kv_token_stride */
  int64_t kv_token_stride;  /* bytes between tokens;    0 -> n_kv_heads * kv_head_stride */
  int64_t kv_head_stride;   /* bytes between heads;     0 -> bytes of one head row */
} aihost_attn_desc;

typedef struct aihost_attn_ctx aihost_attn_ctx;

/* Library version and the thread-local message of the last failing call on this thread. */
int32_t aihost_attn_abi_version(void);
const char* aihost_attn_last_error(void);

/* Context: binds a CUDA device, owns split-K scratch and cached TMA descriptors.
 * Replaces the per-call buffer creation of ComputeOps.FusedMHAGenerate (ComputeOps.cs:1015-1043). */
aihost_status aihost_attn_create(int32_t device, aihost_attn_ctx** out_ctx);
aihost_status aihost_attn_destroy(aihost_attn_ctx* ctx);

/* Bytes of device scratch a forward (or mha, with batch = 1 and n_new = n_q) call with these
 * arguments needs (0 if none): split partials for decode; for prefill, fp16 copies of an fp32 q
 * and of an fp32 / Q8_0 cache (kv_capacity rows), which the tensor-core kernel reads. */
aihost_status aihost_attn_workspace_size(const aihost_attn_desc* desc, int32_t batch, int32_t n_new,
                                         size_t* out_bytes);
/* Grow the context's scratch to at least `bytes` (the only allocating call besides create). */
aihost_status aihost_attn_reserve(aihost_attn_ctx* ctx, size_t bytes);

/* The fused op: RoPE(q) and RoPE(k_new) at positions seq_len[b] + s, append the rotated k_new
 * and v_new into cache rows [seq_len[b], seq_len[b] + n_new), then attention of the n_new
 * query rows over cache rows [0, seq_len[b] + n_new) with the causal rule j <= seq_len[b] + i
 * (ComputeShaders.cs:545-561). n_new == 1 is decode (ComputeOps.cs:1069-1073, split-K kernel);
 * n_new > 1 is prefill (ComputeOps.cs:1076-1101, tcgen05 kernel; fp32 q and fp32 / Q8_0 caches
 * are converted to fp16 in the context's scratch first, with fp32 accumulation throughout).
 *   seq_len     device int32[batch]: rows already cached per sequence (= start position).
 *   h_seq_len   optional host copy of seq_len (NULL allowed): only used to size the grid.
 * q, k_new, v_new are not modified (the reference rotates Q and K in place; here the rotated
 * values live only in registers and in the cache). */
aihost_status aihost_attn_forward(aihost_attn_ctx* ctx, const aihost_attn_desc* desc, int32_t batch,
                                  int32_t n_new, const void* q, const void* k_new, const void* v_new,
                                  void* k_cache, void* v_cache, const int32_t* seq_len,
                                  const int32_t* h_seq_len, void* out, void* stream);

/* aihost_attn_forward over a paged cache instead of one contiguous cache per sequence: the
 * preallocated manager that replaces KVCache.Add's per-token Concat (InferenceEngine.cs:598-622).
 * k_pool / v_pool hold n_pages pages of page_rows rows (a positive multiple of 128) in the layout
 * desc gives per row (kv_token_stride / kv_head_stride; kv_seq_stride is ignored). Row t of
 * sequence b is pool row block_table[b * max_pages + t / page_rows] * page_rows + t % page_rows
 * (block_table: device int32[batch][max_pages]; entries for the pages that rows [0, seq_len[b] +
 * n_new) touch must be valid page indices, distinct across sequences). desc->kv_capacity, the
 * per-sequence row limit, is at most max_pages * page_rows. kv_dtype F32, F16 or Q8_0 (fp16 and
 * Q8_0 pools must be TMA-describable, as for the tensor-core decode of a contiguous cache). */
aihost_status aihost_attn_forward_paged(aihost_attn_ctx* ctx, const aihost_attn_desc* desc, int32_t batch,
                                        int32_t n_new, const void* q, const void* k_new, const void* v_new,
                                        void* k_pool, void* v_pool, int32_t n_pages, int32_t page_rows,
                                        const int32_t* block_table, int32_t max_pages, const int32_t* seq_len,
                                        const int32_t* h_seq_len, void* out, void* stream);

/* ComputeOps.MultiHeadAttention(Q, K, V, numHeads, startPosition) (ComputeOps.cs:1055-1102):
 * attention only, for one sequence, over K/V rows [0, n_kv) that are already rotated.
 * q/out [n_q, Hq*d]; k/v laid out as desc (kv_capacity >= n_kv). rope_mode is ignored.
 * n_q == 1 -> FusedMHAGenerate semantics (no mask); n_q > 1 -> causal j <= start_pos + i. */
aihost_status aihost_attn_mha(aihost_attn_ctx* ctx, const aihost_attn_desc* desc, int32_t n_q,
                              int32_t n_kv, int32_t start_pos, const void* q, const void* k,
                              const void* v, void* out, void* stream);

/* ComputeOps.ApplyRoPEFull(tensor, startPosition, numHeads, headDim, theta)
 * (ComputeOps.cs:959-979): in-place rotation of x [seq, n_heads*head_dim] (F32 or F16). */
aihost_status aihost_rope_full(void* x, int32_t dtype, int32_t seq, int32_t n_heads,
                               int32_t head_dim, int32_t start_pos, float theta, int32_t rope_mode,
                               void* stream);

/* Qwen TypeB Q/K prologue (Compute/Formats/QwenHybridFormat.cs:141-142) in one pass, in place on
 * x [seq, n_heads*head_dim] (F32 or F16): ComputeOps.LayerNorm (ComputeOps.cs:517-542) of each
 * token row over the whole row, all heads together (rms = sqrt(mean(x^2) + eps), x = x / rms *
 * w[i % head_dim], the head_dim weight tiled over the heads as TransformerBase.cs:301-319 does),
 * then ApplyRoPEFull at start_pos + s. weight: device fp32 [head_dim]; the reference's eps is
 * 1e-5. Call it on Q and on the new K before aihost_attn_forward with rope_mode NONE. */
aihost_status aihost_qk_norm_rope(void* x, int32_t dtype, int32_t seq, int32_t n_heads, int32_t head_dim,
                                  const float* weight, float eps, int32_t start_pos, float theta, int32_t rope_mode,
                                  void* stream);

/* KVCache.Add(layer, K, V) (Inference/InferenceEngine.cs:598-622) without the per-token
 * reallocation: copies (and converts / Q8_0-quantises) k_new, v_new [batch][n_new][Hkv][d]
 * into cache rows [seq_len[b], seq_len[b] + n_new). No rotation. */
aihost_status aihost_kv_append(aihost_attn_ctx* ctx, const aihost_attn_desc* desc, int32_t batch, int32_t n_new,
                               const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                               const int32_t* seq_len, void* stream);

/* Device-time profiler, the GPU-side counterpart of the reference's GlobalProfiler
 * (AIHost/Compute/ComputeProfiler.cs:16-97, host Stopwatch totals by name). While enabled,
 * every kernel the context launches is bracketed by CUDA events on the caller's stream;
 * aihost_attn_profiler_read synchronises those events and returns the launch count and
 * total device milliseconds of one kernel kind since the last reset. */
typedef enum {
  AIHOST_KERNEL_APPEND = 0,   /* RoPE(K) + cache append */
  AIHOST_KERNEL_DECODE = 1,   /* split-K decode */
  AIHOST_KERNEL_COMBINE = 2,  /* split merge */
  AIHOST_KERNEL_PREFILL = 3,  /* tcgen05 prefill */
  AIHOST_KERNEL_CONVERT = 4,  /* fp16 staging of fp32 / Q8_0 prefill operands, weight dequantisation */
  AIHOST_KERNEL_MATMUL = 5,   /* tcgen05 weight product (aihost_matmul_weights) */
  AIHOST_KERNEL_COUNT = 6
} aihost_kernel;
aihost_status aihost_attn_profiler_enable(aihost_attn_ctx* ctx, int32_t enable);
aihost_status aihost_attn_profiler_read(aihost_attn_ctx* ctx, int32_t kernel, int64_t* launches, double* total_ms);
aihost_status aihost_attn_profiler_reset(aihost_attn_ctx* ctx);

/* No counterpart in the reference. The one-token decode step of aihost_attn_forward
 * (n_new == 1: RoPE, KV append, split-K attention, split merge) for hosts that cannot allocate
 * device memory when they decode (their allocator is taken by a pool, or may not be entered on
 * the token path). It needs no context and allocates nothing: the split scratch is a static
 * 8 MiB array (plus 512 KiB of split-merge counters) that every GPU loading this library holds
 * until the process exits. Calls whose
 * split scratch, batch * n_q_heads * splits * (head_dim + 2) * 4 bytes, exceeds 8 MiB return
 * AIHOST_ENOMEM. Runs on the current CUDA device. The first call on each device looks up the
 * array's device address: make it before any stream capture. All calls share the array, so
 * calls that overlap on the GPU race; serialise them. Results equal aihost_attn_forward's.
 * Errors the kernels find on the device (a seq_len past kv_capacity, a bounded wait that ran
 * out) are collected in a status word of the array; read them with the call below. */
aihost_status aihost_attn_decode_noalloc(const aihost_attn_desc* desc, int32_t batch, const void* q,
                                         const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                                         const int32_t* seq_len, const int32_t* h_seq_len, void* out,
                                         void* stream);
/* No counterpart in the reference. The status read of aihost_attn_decode_noalloc, which has no
 * context and so no aihost_attn_sync_status: waits for `stream` (the stream of the decode calls),
 * then reads and clears the current device's no-alloc status word, which holds the error bits of
 * every no-alloc call since the last read. Returns AIHOST_EINVAL for a device-side length past
 * kv_capacity, AIHOST_ETIMEOUT for an expired wait, else AIHOST_OK; *out_bits (may be NULL)
 * receives the raw bits. Allocates nothing. */
aihost_status aihost_attn_noalloc_sync_status(void* stream, int32_t* out_bits);

/* ---- KV-head sharding across GPUs (one process per GPU, NCCL over NVLink). Replaces the
 * reference's layer split with host staging (Inference/MultiGPUTransformer.cs:48-183).
 * Rank r of N owns KV heads [r*Hkv/N, (r+1)*Hkv/N) and their query heads, and a cache holding only
 * those heads. NCCL is loaded at run time (libnccl.so.2); AIHOST_EUNSUPPORTED when absent. */
typedef struct aihost_attn_dist aihost_attn_dist;
/* One rank creates the 128-byte NCCL id and the host hands it to every rank. */
aihost_status aihost_attn_dist_unique_id(void* out_id);
/* Collective over all ranks: returns once every rank has called it, or after timeout_ms with
 * AIHOST_ETIMEOUT (a rank that never joins; the half-built communicator is aborted and nothing is
 * returned). The communicator is nonblocking: every NCCL wait of this library is a bounded host
 * poll, never an unbounded block. No counterpart in the reference, whose waits are unbounded
 * (ICompute/Vulkan/VulkanComputeCommandQueue.cs:287). */
aihost_status aihost_attn_dist_init_bounded(int32_t world, int32_t rank, const void* nccl_id, int32_t device,
                                            int32_t timeout_ms, aihost_attn_dist** out);
/* aihost_attn_dist_init_bounded with the limit AIHOST_NCCL_TIMEOUT_MS from the environment
 * (default 300000 ms). */
aihost_status aihost_attn_dist_init(int32_t world, int32_t rank, const void* nccl_id, int32_t device,
                                    aihost_attn_dist** out);
aihost_status aihost_attn_dist_destroy(aihost_attn_dist* dist);
/* Waits at most timeout_ms for everything enqueued on `stream` (this rank's kernels and
 * collectives) to finish. AIHOST_ETIMEOUT when it does not (a peer that stopped taking part) and
 * AIHOST_ENCCL on an asynchronous NCCL error; in both cases the communicator is aborted, which
 * ends its in-flight collectives, and later sharded calls on it return AIHOST_ENCCL. The host's
 * replacement for a Flush() fence wait (ComputeOps.cs:115-140) on the sharded path. */
aihost_status aihost_attn_dist_sync(aihost_attn_dist* dist, void* stream, int32_t timeout_ms);
/* aihost_attn_forward of this rank's heads (`local`: n_q_heads = Hq/N, n_kv_heads = Hkv/N and the
 * local cache layout), written into this rank's slot of out_gathered, then one in-place
 * all-gather on `stream`: out_gathered is [N][batch][n_new][Hq/N][head_dim] (rank-major) on every
 * rank. Every rank must make the same calls in the same order. ctx and dist must be on the same
 * device (AIHOST_EINVAL otherwise). */
aihost_status aihost_attn_forward_sharded(aihost_attn_dist* dist, aihost_attn_ctx* ctx,
                                          const aihost_attn_desc* local, int32_t batch, int32_t n_new,
                                          const void* q, const void* k_new, const void* v_new,
                                          void* k_cache, void* v_cache, const int32_t* seq_len,
                                          const int32_t* h_seq_len, void* out_gathered, void* stream);

/* ---- Context parallelism for decode (layers with fewer KV heads than ranks). No counterpart
 * in the reference, which decodes a sequence on one device (ComputeOps.cs:1015-1043). Each rank
 * holds a contiguous chunk of every sequence's cached rows; it attends its chunk with
 * aihost_attn_decode_partial, the ranks exchange (out, lse) with their own collective, and
 * aihost_attn_merge_partials combines them into the unsharded result.
 *
 * One query row per sequence over this part's cache rows with every row visible. seq_len
 * (device int32[batch]) holds this part's cached rows per sequence. With k_new / v_new
 * [batch][Hkv][d] (the part that stores the new token; both or neither), the new rows are
 * appended at row seq_len[b] first, K rotated at q_pos[b], and rows [0, seq_len[b] + 1) are
 * attended; without them rows [0, seq_len[b]). q [batch][Hq][d]: rotated in the kernel at
 * position q_pos[b] (device int32[batch], the token's global position) when q_pos is non-NULL
 * and desc->rope_mode is not NONE, else used as given (q_pos is required with k_new). out
 * [batch][Hq][d] in out_dtype, normalised over this part's rows; lse (device float[batch][Hq],
 * may be NULL) receives ln sum_j exp(scale * q.k_j) over those rows. */
aihost_status aihost_attn_decode_partial(aihost_attn_ctx* ctx, const aihost_attn_desc* desc, int32_t batch,
                                         const void* q, const void* k_new, const void* v_new, void* k_cache,
                                         void* v_cache, const int32_t* seq_len, const int32_t* q_pos, void* out,
                                         float* lse, void* stream);
/* out[r] = sum_p o_parts[p][r] * exp(lse_parts[p][r] - lse[r]), lse[r] = ln sum_p exp(lse_parts[p][r]),
 * for rows r < rows (= batch * Hq) of head_dim elements; o_parts [n_parts][rows][head_dim] and
 * out in dtype (F32 or F16), lse_parts [n_parts][rows] fp32 (a part with lse = -inf adds
 * nothing). lse_out (may be NULL) receives lse. */
aihost_status aihost_attn_merge_partials(aihost_attn_ctx* ctx, int32_t n_parts, int32_t rows, int32_t head_dim,
                                         int32_t dtype, const void* o_parts, const float* lse_parts, void* out,
                                         float* lse_out, void* stream);

/* ---- The weight products around the op: C[rows, n_out] = A[rows, k] . W, with W a GGUF weight
 * ("column-major" in GGUF terms: element (k, n) at n * k_total + k, i.e. n_out rows of k values,
 * K-quant blocks running along k). Replaces ComputeOps.MatMulWeights (ComputeOps.cs:275-313) at
 * its calls beside attention: the Q/K/V projections that feed the op (ComputeOps.cs:1274-1276,
 * weights dequantised per call by TransformerBase.TempF32 / ComputeOps.DequantizeInto,
 * ComputeOps.cs:761-861) and the output projection right after it (ComputeOps.cs:1317).
 * A is given as n_parts column blocks stored one after another, [n_parts][rows][k / n_parts]
 * (n_parts = 1: plain row-major [rows][k]); with n_parts = N this is the rank-major
 * [N][batch][n_new][Hq/N][head_dim] buffer aihost_attn_forward_sharded gathers, read in place.
 * fp16 operands on the tensor cores (fp32 A is rounded to fp16 first; K-quant weights are
 * dequantised with the reference shaders' formulas, then rounded once to fp16), fp32
 * accumulation. With at most 128 rows, Q4_K and Q5_K weights are dequantised inside the one GEMM
 * launch; other K-quant and fp32 weights are first copied to fp16 in the context's scratch. Needs
 * aihost_matmul_workspace_size bytes of that scratch (0 for fp16 A with fp16, or in-GEMM, weights). */
typedef struct {
  int32_t rows;       /* M: rows of A and of the output */
  int32_t k;          /* K: a multiple of 64 (of 256 for K-quant weights); k / n_parts a multiple of 64 */
  int32_t n_out;      /* N: output columns, a multiple of 8 */
  int32_t n_parts;    /* column blocks of A (>= 1) */
  int32_t a_dtype;    /* F16 or F32 */
  int32_t w_dtype;    /* F16, F32, Q2_K, Q3_K, Q4_K, Q5_K or Q6_K */
  int32_t out_dtype;  /* F16 or F32 */
} aihost_matmul_desc;
aihost_status aihost_matmul_workspace_size(const aihost_matmul_desc* desc, size_t* out_bytes);
aihost_status aihost_matmul_weights(aihost_attn_ctx* ctx, const aihost_matmul_desc* desc, const void* a,
                                    const void* w, void* out, void* stream);
/* ComputeOps.DequantizeInto (ComputeOps.cs:761-861) with the reference's own formulas
 * (QuantizationFormats.cs): n_elems (a multiple of 256) values of a K-quant tensor into out, F32
 * (the reference's target type; equal to its shader's result) or F16 (that value rounded once). */
aihost_status aihost_dequantize(const void* w, int32_t w_dtype, int64_t n_elems, void* out, int32_t out_dtype,
                                void* stream);

/* Synchronise the context's device and read-and-clear the device status word that kernels
 * set when a bounded wait expired (AIHOST_ETIMEOUT) or a device-side length exceeded
 * kv_capacity (AIHOST_EINVAL). *out_bits receives the raw bits (may be NULL). */
aihost_status aihost_attn_sync_status(aihost_attn_ctx* ctx, int32_t* out_bits);

#ifdef __cplusplus
}
#endif

#endif /* AIHOST_ATTN_H */
