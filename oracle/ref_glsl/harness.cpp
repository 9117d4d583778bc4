// harness.cpp — the host side of AIHost's attention path, driving the reference's own shaders
// (compiled for the CPU by build_ref.py) in the order and with the parameters that
// AIHost/AIHost/Compute/ComputeOps.cs uses. TEST INFRASTRUCTURE ONLY: pins the C oracle.
//
// Vulkan's Dispatch(kernel, {x, y}) launches x*y workgroups (VulkanComputeCommandQueue.cs
// records vkCmdDispatch with these counts); the same counts are used here.
#include <cmath>
#include <cstdint>
#include <cstring>
#include <vector>

namespace glsl {
typedef unsigned int uint;
}
#define AIHOST_SHADER(name)                     \
  namespace sh_##name {                         \
  void bind(int binding, void* ptr);            \
  void run(glsl::uint gx, glsl::uint gy, glsl::uint gz); \
  }
AIHOST_SHADER(rope_full)
AIHOST_SHADER(concat_axis0)
AIHOST_SHADER(fused_mha_generate)
AIHOST_SHADER(matmul)
AIHOST_SHADER(transpose)
AIHOST_SHADER(scale)
AIHOST_SHADER(causal_mask)
AIHOST_SHADER(rowwise_softmax)
AIHOST_SHADER(slice_cols)
AIHOST_SHADER(scatter_cols)
AIHOST_SHADER(layernorm)
AIHOST_SHADER(matmul_weights)
AIHOST_SHADER(dequant_q2k)
AIHOST_SHADER(dequant_q3k)
AIHOST_SHADER(dequant_q4k)
AIHOST_SHADER(dequant_q5k)
AIHOST_SHADER(dequant_q6k)
#undef AIHOST_SHADER

namespace {

using Vec = std::vector<float>;

uint32_t fbits(float f) {
  uint32_t u;
  std::memcpy(&u, &f, 4);
  return u;
}

// ApplyRoPEFull (ComputeOps.cs:959-979): params {seqLen, numHeads, headDim, startPosition, theta}.
void ApplyRoPEFull(float* x, int seqLen, int numHeads, int headDim, uint32_t start, float theta) {
  uint32_t p[5] = {uint32_t(seqLen), uint32_t(numHeads), uint32_t(headDim), start, fbits(theta)};
  sh_rope_full::bind(0, x);
  sh_rope_full::bind(1, p);
  const uint32_t total = uint32_t(seqLen * numHeads * headDim / 2);
  sh_rope_full::run((total + 255u) / 256u, 1, 1);
}

// LayerNorm (ComputeOps.cs:517-542): params {rows, cols, eps}, one workgroup per row.
void LayerNorm(float* x, int rows, int cols, const float* w, float eps) {
  uint32_t p[3] = {uint32_t(rows), uint32_t(cols), fbits(eps)};
  sh_layernorm::bind(0, x);
  sh_layernorm::bind(1, const_cast<float*>(w));
  sh_layernorm::bind(2, p);
  sh_layernorm::run(uint32_t(rows), 1, 1);
}

// Concat axis 0 (ComputeOps.cs:424-453): params {rows_a, rows_b, cols}.
Vec ConcatAxis0(const float* a, int rows_a, const float* b, int rows_b, int cols) {
  Vec r(size_t(rows_a + rows_b) * cols);
  uint32_t p[3] = {uint32_t(rows_a), uint32_t(rows_b), uint32_t(cols)};
  sh_concat_axis0::bind(0, const_cast<float*>(a));
  sh_concat_axis0::bind(1, const_cast<float*>(b));
  sh_concat_axis0::bind(2, r.data());
  sh_concat_axis0::bind(3, p);
  sh_concat_axis0::run(uint32_t((r.size() + 255) / 256), 1, 1);
  return r;
}

// FusedMHAGenerate (ComputeOps.cs:1015-1043): one workgroup per Q head.
Vec FusedMHAGenerate(const float* Q, const float* K, const float* V, int kvSeqLen, int Hq, int Hkv, int d,
                     float scale) {
  Vec out(size_t(Hq) * d);
  uint32_t p[5] = {uint32_t(Hq), uint32_t(Hkv), uint32_t(d), uint32_t(kvSeqLen), fbits(scale)};
  sh_fused_mha_generate::bind(0, const_cast<float*>(Q));
  sh_fused_mha_generate::bind(1, const_cast<float*>(K));
  sh_fused_mha_generate::bind(2, const_cast<float*>(V));
  sh_fused_mha_generate::bind(3, out.data());
  sh_fused_mha_generate::bind(4, p);
  sh_fused_mha_generate::run(uint32_t(Hq), 1, 1);
  return out;
}

// MatMul (ComputeOps.cs:315-351): C[M x N] = A[M x K] B[K x N], 16x16 workgroups.
Vec MatMul(const Vec& A, const Vec& B, int M, int K, int N) {
  Vec C(size_t(M) * N);
  uint32_t p[3] = {uint32_t(M), uint32_t(K), uint32_t(N)};
  sh_matmul::bind(0, const_cast<float*>(A.data()));
  sh_matmul::bind(1, const_cast<float*>(B.data()));
  sh_matmul::bind(2, C.data());
  sh_matmul::bind(3, p);
  sh_matmul::run(uint32_t((N + 15) / 16), uint32_t((M + 15) / 16), 1);
  return C;
}

// Transpose (ComputeOps.cs:880-904).
Vec Transpose(const Vec& A, int rows, int cols) {
  Vec B(size_t(rows) * cols);
  uint32_t p[2] = {uint32_t(rows), uint32_t(cols)};
  sh_transpose::bind(0, const_cast<float*>(A.data()));
  sh_transpose::bind(1, B.data());
  sh_transpose::bind(2, p);
  sh_transpose::run(uint32_t((cols + 15) / 16), uint32_t((rows + 15) / 16), 1);
  return B;
}

// Scale (ComputeOps.cs:935-953): params {size, scale}.
void Scale(Vec& t, float s) {
  uint32_t p[2] = {uint32_t(t.size()), fbits(s)};
  sh_scale::bind(0, t.data());
  sh_scale::bind(1, p);
  sh_scale::run(uint32_t((t.size() + 255) / 256), 1, 1);
}

// ApplyCausalMask (ComputeOps.cs:986-1007): skipped when seqLen_q <= 1.
void ApplyCausalMask(Vec& scores, int seq_q, int seq_k, uint32_t start) {
  if (seq_q <= 1) return;
  uint32_t p[3] = {uint32_t(seq_q), uint32_t(seq_k), start};
  sh_causal_mask::bind(0, scores.data());
  sh_causal_mask::bind(1, p);
  sh_causal_mask::run(uint32_t((size_t(seq_q) * seq_k + 255) / 256), 1, 1);
}

// RowwiseSoftmax (ComputeOps.cs:909-930): one workgroup per row.
void RowwiseSoftmax(Vec& t, int rows, int cols) {
  uint32_t p[2] = {uint32_t(rows), uint32_t(cols)};
  sh_rowwise_softmax::bind(0, t.data());
  sh_rowwise_softmax::bind(1, p);
  sh_rowwise_softmax::run(uint32_t(rows), 1, 1);
}

// SliceCols (ComputeOps.cs:1107-1121).
Vec SliceCols(const float* src, int rows, int srcCols, int colStart, int colCount) {
  Vec r(size_t(rows) * colCount);
  uint32_t p[4] = {uint32_t(rows), uint32_t(srcCols), uint32_t(colStart), uint32_t(colCount)};
  sh_slice_cols::bind(0, const_cast<float*>(src));
  sh_slice_cols::bind(1, r.data());
  sh_slice_cols::bind(2, p);
  sh_slice_cols::run(uint32_t((r.size() + 255) / 256), 1, 1);
  return r;
}

// ScatterCols (ComputeOps.cs:1124-1136).
void ScatterCols(float* dst, int dstCols, const Vec& src, int rows, int colStart, int colCount) {
  uint32_t p[4] = {uint32_t(rows), uint32_t(dstCols), uint32_t(colStart), uint32_t(colCount)};
  sh_scatter_cols::bind(0, const_cast<float*>(src.data()));
  sh_scatter_cols::bind(1, dst);
  sh_scatter_cols::bind(2, p);
  sh_scatter_cols::run(uint32_t((size_t(rows) * colCount + 255) / 256), 1, 1);
}

// MultiHeadAttention (ComputeOps.cs:1055-1102).
Vec MultiHeadAttention(const float* Q, int seqLen, int dModelQ, const float* K, const float* V, int kvSeqLen,
                       int kvDim, int numHeads, uint32_t startPosition) {
  const int headDim = dModelQ / numHeads;
  const int numKvHeads = kvDim / headDim;
  const float scale = 1.0f / std::sqrt(static_cast<float>(headDim));
  if (seqLen == 1) return FusedMHAGenerate(Q, K, V, kvSeqLen, numHeads, numKvHeads, headDim, scale);
  Vec out(size_t(seqLen) * dModelQ, 0.0f);
  for (int h = 0; h < numHeads; ++h) {
    const int kvHead = h / (numHeads / numKvHeads);
    Vec Qh = SliceCols(Q, seqLen, dModelQ, h * headDim, headDim);
    Vec Kh = SliceCols(K, kvSeqLen, kvDim, kvHead * headDim, headDim);
    Vec Vh = SliceCols(V, kvSeqLen, kvDim, kvHead * headDim, headDim);
    Vec KTh = Transpose(Kh, kvSeqLen, headDim);
    Vec scores = MatMul(Qh, KTh, seqLen, headDim, kvSeqLen);
    Scale(scores, scale);
    ApplyCausalMask(scores, seqLen, kvSeqLen, startPosition);
    RowwiseSoftmax(scores, seqLen, kvSeqLen);
    Vec oh = MatMul(scores, Vh, seqLen, kvSeqLen, headDim);
    ScatterCols(out.data(), dModelQ, oh, seqLen, h * headDim, headDim);
  }
  return out;
}

}  // namespace

extern "C" {

// ApplyRoPEFull on x [seq, n_heads * head_dim] in place.
int ref_rope_full(float* x, int seq, int n_heads, int head_dim, int start, float theta) {
  ApplyRoPEFull(x, seq, n_heads, head_dim, uint32_t(start), theta);
  return 0;
}

// Qwen TypeB Q/K prologue (QwenHybridFormat.cs:141-142): LayerNorm of each row of
// x [seq, n_heads * head_dim] with the head_dim weight tiled over the heads
// (TransformerBase.GetOrBuildTiledNorm), then ApplyRoPEFull at start.
int ref_qk_norm_rope(float* x, int seq, int n_heads, int head_dim, const float* w_head, float eps, int start,
                     float theta) {
  std::vector<float> tiled(size_t(n_heads) * head_dim);
  for (int h = 0; h < n_heads; ++h) std::memcpy(tiled.data() + size_t(h) * head_dim, w_head, sizeof(float) * head_dim);
  LayerNorm(x, seq, n_heads * head_dim, tiled.data(), eps);
  ApplyRoPEFull(x, seq, n_heads, head_dim, uint32_t(start), theta);
  return 0;
}

// MultiHeadAttention(Q [seq, Hq*d], K/V [kv_len, Hkv*d], numHeads, startPosition).
int ref_mha(const float* q, int seq, const float* k, const float* v, int kv_len, int n_q_heads, int n_kv_heads,
            int head_dim, int start, float* out) {
  Vec o = MultiHeadAttention(q, seq, n_q_heads * head_dim, k, v, kv_len, n_kv_heads * head_dim, n_q_heads,
                             uint32_t(start));
  std::memcpy(out, o.data(), o.size() * 4);
  return 0;
}

// One layer's attention step as TransformerLayer runs it (ComputeOps.cs:1282-1304):
// RoPE(Q), RoPE(K) at `pos`, KVCache.Add (InferenceEngine.cs:598-622: the first Add owns the
// new rows, later Adds Concat old and new), Get, MultiHeadAttention(Q, K, V, numHeads, pos).
// k_cached / v_cached hold `pos` rows (ignored when pos == 0); k_all / v_all receive the
// pos + S cached rows after the append.
int ref_layer_attention(const float* q, const float* k_new, const float* v_new, int S, const float* k_cached,
                        const float* v_cached, int pos, int n_q_heads, int n_kv_heads, int head_dim, float theta,
                        float* out, float* k_all, float* v_all) {
  const int dq = n_q_heads * head_dim, dkv = n_kv_heads * head_dim;
  Vec Q(q, q + size_t(S) * dq), K(k_new, k_new + size_t(S) * dkv), V(v_new, v_new + size_t(S) * dkv);
  ApplyRoPEFull(Q.data(), S, n_q_heads, head_dim, uint32_t(pos), theta);
  ApplyRoPEFull(K.data(), S, n_kv_heads, head_dim, uint32_t(pos), theta);
  Vec Kc, Vc;
  if (pos == 0) {
    Kc = K;
    Vc = V;
  } else {
    Kc = ConcatAxis0(k_cached, pos, K.data(), S, dkv);
    Vc = ConcatAxis0(v_cached, pos, V.data(), S, dkv);
  }
  Vec o = MultiHeadAttention(Q.data(), S, dq, Kc.data(), Vc.data(), pos + S, dkv, n_q_heads, uint32_t(pos));
  std::memcpy(out, o.data(), o.size() * 4);
  std::memcpy(k_all, Kc.data(), Kc.size() * 4);
  std::memcpy(v_all, Vc.data(), Vc.size() * 4);
  return 0;
}

// ComputeOps.Dequantize (ComputeOps.cs:733-745 -> DequantizeQ2K..DequantizeQ6K): one dispatch of
// ceil(n / 256) workgroups, element offset 0 (DequantizeInto's chunked dispatches differ only in
// that offset, and every invocation is independent). kind = AIHost DataType ordinal (Q2_K = 8 ..
// Q6_K = 12); blocks hold n / 256 GGUF blocks.
int ref_dequantize(int kind, const void* blocks, int n, float* out) {
  uint32_t zero = 0;
  void (*bind)(int, void*) = nullptr;
  void (*run)(glsl::uint, glsl::uint, glsl::uint) = nullptr;
  switch (kind) {
    case 8: bind = sh_dequant_q2k::bind; run = sh_dequant_q2k::run; break;
    case 9: bind = sh_dequant_q3k::bind; run = sh_dequant_q3k::run; break;
    case 10: bind = sh_dequant_q4k::bind; run = sh_dequant_q4k::run; break;
    case 11: bind = sh_dequant_q5k::bind; run = sh_dequant_q5k::run; break;
    case 12: bind = sh_dequant_q6k::bind; run = sh_dequant_q6k::run; break;
    default: return 1;
  }
  bind(0, const_cast<void*>(blocks));
  bind(1, out);
  bind(2, &zero);
  run((uint32_t(n) + 255u) / 256u, 1, 1);
  return 0;
}

// ComputeOps.MatMulWeights (ComputeOps.cs:275-313): C [M, N] = A [M, K] . B with B a GGUF
// column-major weight (element (k, n) at n * K + k); params {M, K, N}; workgroups of 16 x 16
// over {ceil(N / 16), ceil(M / 16)}.
int ref_matmul_weights(const float* a, int M, int K, const float* b, int N, float* c) {
  uint32_t p[3] = {uint32_t(M), uint32_t(K), uint32_t(N)};
  sh_matmul_weights::bind(0, const_cast<float*>(a));
  sh_matmul_weights::bind(1, const_cast<float*>(b));
  sh_matmul_weights::bind(2, c);
  sh_matmul_weights::bind(3, p);
  sh_matmul_weights::run((uint32_t(N) + 15u) / 16u, (uint32_t(M) + 15u) / 16u, 1);
  return 0;
}

}  // extern "C"
