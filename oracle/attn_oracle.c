/*
 * attn_oracle.c — CPU restatement of AIHost's attention hot path (TEST INFRASTRUCTURE ONLY).
 *
 * Only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline leg load this code, as the
 * checker and as the timed CPU reference. The product library never links it.
 * Build: oracle/Makefile (-O3 -fopenmp -ffp-contract=off; see attn_oracle.h for the modes).
 */
#include "attn_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

int32_t oracle_num_threads(void) {
#ifdef _OPENMP
  return (int32_t)omp_get_max_threads();
#else
  return 1;
#endif
}

void oracle_set_num_threads(int32_t n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* ---------------------------------------------------------------- fp16 <-> fp32 (IEEE RNE) */

float oracle_f16_to_f32(uint16_t h) {
  uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu;
  uint32_t m = h & 0x3ffu;
  uint32_t bits;
  if (e == 0) {
    if (m == 0) {
      bits = sign;
    } else { /* subnormal: value m * 2^-24, renormalise */
      int32_t ee = -14;
      while ((m & 0x400u) == 0) { m <<= 1; ee--; }
      m &= 0x3ffu;
      bits = sign | ((uint32_t)(ee + 127) << 23) | (m << 13);
    }
  } else if (e == 31) {
    bits = sign | 0x7f800000u | (m << 13);
  } else {
    bits = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

uint16_t oracle_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0u));
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to inf */
  if (ax < 0x38800000u) {                                    /* below 2^-14: subnormal or zero */
    if (ax < 0x33000000u) return (uint16_t)sign;             /* below 2^-25 */
    uint32_t e = ax >> 23, m = (ax & 0x7fffffu) | 0x800000u;
    uint32_t shift = 126u - e; /* value / 2^-24 = m >> shift */
    uint32_t q = m >> shift, rem = m & ((1u << shift) - 1u), half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t h = (((ax >> 23) - 112u) << 10) | ((ax & 0x7fffffu) >> 13);
  uint32_t rem = ax & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
  return (uint16_t)(sign | h);
}

static float g_f16_lut[65536];
static int g_f16_lut_ready = 0;

static void f16_lut_init(void) {
  if (g_f16_lut_ready) return;
  for (uint32_t i = 0; i < 65536u; ++i) g_f16_lut[i] = oracle_f16_to_f32((uint16_t)i);
  g_f16_lut_ready = 1;
}

void oracle_f16_to_f32_n(const uint16_t* src, float* dst, int64_t n) {
  f16_lut_init();
  for (int64_t i = 0; i < n; ++i) dst[i] = g_f16_lut[src[i]];
}

void oracle_f32_to_f16_n(const float* src, uint16_t* dst, int64_t n) {
  for (int64_t i = 0; i < n; ++i) dst[i] = oracle_f32_to_f16(src[i]);
}

/* ---------------------------------------------------------------- GGUF Q8_0 */

static void q8_0_quantize_block(const float* x, uint8_t* blk) {
  float amax = 0.0f;
  for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(x[j]));
  const float d = amax / 127.0f;
  const float id = d != 0.0f ? 1.0f / d : 0.0f;
  uint16_t dh = oracle_f32_to_f16(d);
  blk[0] = (uint8_t)(dh & 0xffu);
  blk[1] = (uint8_t)(dh >> 8);
  for (int j = 0; j < 32; ++j) blk[2 + j] = (uint8_t)(int8_t)roundf(x[j] * id);
}

static void q8_0_dequantize_block(const uint8_t* blk, float* x) {
  f16_lut_init();
  const float d = g_f16_lut[(uint16_t)(blk[0] | (blk[1] << 8))];
  for (int j = 0; j < 32; ++j) x[j] = d * (float)(int8_t)blk[2 + j];
}

void oracle_q8_0_quantize(const float* x, int64_t n, uint8_t* blocks) {
  for (int64_t b = 0; b < n / 32; ++b) q8_0_quantize_block(x + 32 * b, blocks + 34 * b);
}

void oracle_q8_0_dequantize(const uint8_t* blocks, int64_t n, float* x) {
  for (int64_t b = 0; b < n / 32; ++b) q8_0_dequantize_block(blocks + 34 * b, x + 32 * b);
}

/* ---------------------------------------------------------------- RoPE (ComputeShaders.cs:517-543) */

float oracle_rope_freq(float theta, int32_t pair, int32_t head_dim) {
  return 1.0f / powf(theta, (float)(pair * 2) / (float)head_dim);
}

static void rope_row(float* x, int32_t head_dim, int32_t pos, float theta, int32_t rope_mode) {
  const int32_t half = head_dim / 2;
  for (int32_t i = 0; i < half; ++i) {
    const float freq = oracle_rope_freq(theta, i, head_dim);
    const float angle = (float)pos * freq;
    const float c = cosf(angle), s = sinf(angle);
    const int32_t i1 = rope_mode == AIHOST_ROPE_NEOX ? i : 2 * i;
    const int32_t i2 = rope_mode == AIHOST_ROPE_NEOX ? i + half : 2 * i + 1;
    const float x1 = x[i1], x2 = x[i2];
    x[i1] = x1 * c - x2 * s;
    x[i2] = x1 * s + x2 * c;
  }
}

void oracle_qk_norm_rope(float* x, int32_t seq, int32_t n_heads, int32_t head_dim, const float* w, float eps,
                         int32_t start_pos, float theta, int32_t rope_mode) {
  const int32_t cols = n_heads * head_dim;
  for (int32_t s = 0; s < seq; ++s) {
    float* row = x + (int64_t)s * cols;
    float part[256];
    for (int t = 0; t < 256; ++t) {  /* thread t of the workgroup: elements t, t + 256, ... */
      float acc = 0.0f;
      for (int32_t i = t; i < cols; i += 256) acc += row[i] * row[i];
      part[t] = acc;
    }
    for (int h = 128; h > 0; h >>= 1)
      for (int t = 0; t < h; ++t) part[t] += part[t + h];
    const float rms = sqrtf(part[0] / (float)cols + eps);
    for (int32_t i = 0; i < cols; ++i) row[i] = (row[i] / rms) * w[i % head_dim];
  }
  oracle_rope_full(x, seq, n_heads, head_dim, start_pos, theta, rope_mode);
}

void oracle_rope_full(float* x, int32_t seq, int32_t n_heads, int32_t head_dim, int32_t start_pos,
                      float theta, int32_t rope_mode) {
  if (rope_mode == AIHOST_ROPE_NONE) return;
  for (int32_t s = 0; s < seq; ++s)
    for (int32_t h = 0; h < n_heads; ++h)
      rope_row(x + ((int64_t)s * n_heads + h) * head_dim, head_dim, start_pos + s, theta, rope_mode);
}

/* RoPE of rows [s0, s1) and heads [h0, h1) of x [seq, n_heads * head_dim] (rows rotated at
 * start_pos + s): the same per-element operations as oracle_rope_full, restricted to the part a
 * sampled call attends or appends. */
static void rope_part(float* x, int32_t n_heads, int32_t head_dim, int32_t start_pos, float theta, int32_t rope_mode,
                      int32_t s0, int32_t s1, int32_t h0, int32_t h1) {
  if (rope_mode == AIHOST_ROPE_NONE) return;
#pragma omp parallel for schedule(static)
  for (int32_t s = s0; s < s1; ++s)
    for (int32_t h = h0; h < h1; ++h)
      rope_row(x + ((int64_t)s * n_heads + h) * head_dim, head_dim, start_pos + s, theta, rope_mode);
}

/* ---------------------------------------------------------------- attention row */

/* K/V row access: fp32 rows, fp16 rows or Q8_0 rows, dequantised into dst[head_dim]. */
typedef struct {
  const uint8_t* base;
  int32_t dtype;
  int64_t row_stride;  /* bytes between rows (tokens) */
  int64_t head_stride; /* bytes between heads */
} kv_view;

static inline void kv_load(const kv_view* v, int64_t row, int32_t head, int32_t head_dim, float* dst) {
  const uint8_t* p = v->base + row * v->row_stride + (int64_t)head * v->head_stride;
  if (v->dtype == AIHOST_F32) {
    memcpy(dst, p, (size_t)head_dim * 4);
  } else if (v->dtype == AIHOST_F16) {
    const uint16_t* h = (const uint16_t*)p;
    for (int32_t i = 0; i < head_dim; ++i) dst[i] = g_f16_lut[h[i]];
  } else {
    for (int32_t blk = 0; blk < head_dim / 32; ++blk) q8_0_dequantize_block(p + 34 * blk, dst + 32 * blk);
  }
}

/* One query row of one head against visible rows [0, n_vis) of n_kv (masked rows are
 * j >= n_vis). Faithful: the order of fused_mha_generate / rowwise_softmax; is_decode adds the
 * 1e-6 denominator floor (ComputeShaders.cs:716). Scratch: n_kv floats + 2*head_dim floats. */
static void attend_row(const float* qrow, const kv_view* kv_k, const kv_view* kv_v, int32_t kvh,
                       int32_t n_vis, int32_t head_dim, float scale, int32_t mode, int32_t is_decode,
                       float* scores, float* rowbuf, float* out) {
  if (mode == ORACLE_FAITHFUL) {
    for (int32_t j = 0; j < n_vis; ++j) {
      kv_load(kv_k, j, kvh, head_dim, rowbuf);
      float s = 0.0f;
      for (int32_t t = 0; t < head_dim; ++t) s += qrow[t] * rowbuf[t];
      scores[j] = s * scale;
    }
    /* masked entries hold -1e38 in the reference; exp(-1e38 - max) is exactly 0 and adds
     * nothing to any partial sum or P.V accumulator, so they are skipped below. */
    float mx = -1e38f;
    for (int32_t j = 0; j < n_vis; ++j) mx = fmaxf(mx, scores[j]);
    float partial[256];
    for (int32_t t = 0; t < 256; ++t) partial[t] = 0.0f;
    for (int32_t j = 0; j < n_vis; ++j) {
      const float e = expf(scores[j] - mx);
      scores[j] = e;
      partial[j & 255] += e;
    }
    for (int32_t st = 128; st > 0; st >>= 1)
      for (int32_t t = 0; t < st; ++t) partial[t] += partial[t + st];
    float sum = partial[0];
    if (is_decode) sum = fmaxf(sum, 0.000001f);
    for (int32_t j = 0; j < n_vis; ++j) scores[j] /= sum;
    float* acc = rowbuf + head_dim;
    for (int32_t t = 0; t < head_dim; ++t) acc[t] = 0.0f;
    for (int32_t j = 0; j < n_vis; ++j) {
      kv_load(kv_v, j, kvh, head_dim, rowbuf);
      const float p = scores[j];
      for (int32_t t = 0; t < head_dim; ++t) acc[t] += p * rowbuf[t];
    }
    for (int32_t t = 0; t < head_dim; ++t) out[t] = acc[t];
  } else {
    double* ds = (double*)scores; /* caller sized scratch for doubles */
    double mx = -1e300;
    for (int32_t j = 0; j < n_vis; ++j) {
      kv_load(kv_k, j, kvh, head_dim, rowbuf);
      double s = 0.0;
      for (int32_t t = 0; t < head_dim; ++t) s += (double)qrow[t] * (double)rowbuf[t];
      ds[j] = s * (double)scale;
      if (ds[j] > mx) mx = ds[j];
    }
    double sum = 0.0;
    for (int32_t j = 0; j < n_vis; ++j) {
      ds[j] = exp(ds[j] - mx);
      sum += ds[j];
    }
    double acc[256];
    for (int32_t t = 0; t < head_dim; ++t) acc[t] = 0.0;
    for (int32_t j = 0; j < n_vis; ++j) {
      kv_load(kv_v, j, kvh, head_dim, rowbuf);
      const double p = ds[j] / sum;
      for (int32_t t = 0; t < head_dim; ++t) acc[t] += p * (double)rowbuf[t];
    }
    for (int32_t t = 0; t < head_dim; ++t) out[t] = (float)acc[t];
  }
}

int32_t oracle_mha(const float* q, const float* k, const float* v, int64_t kv_row_stride,
                   int32_t n_q, int32_t n_kv, int32_t n_q_heads, int32_t n_kv_heads,
                   int32_t head_dim, int32_t start_pos, float scale, int32_t mode, float* out) {
  if (!q || !k || !v || !out || n_q < 1 || n_kv < 1 || n_q_heads < 1 || n_kv_heads < 1 ||
      n_q_heads % n_kv_heads || head_dim < 2 || head_dim > 256 || head_dim % 2)
    return 1;
  f16_lut_init();
  const int32_t group = n_q_heads / n_kv_heads;
  const kv_view kk = {(const uint8_t*)k, AIHOST_F32, kv_row_stride * 4, (int64_t)head_dim * 4};
  const kv_view vv = {(const uint8_t*)v, AIHOST_F32, kv_row_stride * 4, (int64_t)head_dim * 4};
  int32_t err = 0;
#pragma omp parallel
  {
    float* scores = (float*)malloc(sizeof(double) * (size_t)n_kv);
    float* rowbuf = (float*)malloc(sizeof(float) * 2 * (size_t)head_dim);
    if (!scores || !rowbuf) {
#pragma omp atomic write
      err = 2;
    } else {
#pragma omp for collapse(2) schedule(dynamic, 1)
      for (int32_t h = 0; h < n_q_heads; ++h)
        for (int32_t i = 0; i < n_q; ++i) {
          /* decode sees every row; prefill masks j > start_pos + i (ComputeShaders.cs:557) */
          int32_t n_vis = n_q == 1 ? n_kv : start_pos + i + 1;
          if (n_vis > n_kv) n_vis = n_kv;
          attend_row(q + ((int64_t)i * n_q_heads + h) * head_dim, &kk, &vv, h / group, n_vis,
                     head_dim, scale, mode, n_q == 1, scores, rowbuf,
                     out + ((int64_t)i * n_q_heads + h) * head_dim);
        }
    }
    free(scores);
    free(rowbuf);
  }
  return err;
}

/* ---------------------------------------------------------------- fused forward */

static int64_t dtype_row_bytes(int32_t dtype, int32_t head_dim) {
  if (dtype == AIHOST_F32) return 4LL * head_dim;
  if (dtype == AIHOST_F16) return 2LL * head_dim;
  return 34LL * (head_dim / 32);
}

static void to_f32(const void* src, int32_t dtype, int64_t n, float* dst) {
  if (dtype == AIHOST_F32) memcpy(dst, src, (size_t)n * 4);
  else oracle_f16_to_f32_n((const uint16_t*)src, dst, n);
}

static void store_row(uint8_t* dst, int32_t dtype, const float* x, int32_t head_dim) {
  if (dtype == AIHOST_F32) memcpy(dst, x, (size_t)head_dim * 4);
  else if (dtype == AIHOST_F16) oracle_f32_to_f16_n(x, (uint16_t*)dst, head_dim);
  else oracle_q8_0_quantize(x, head_dim, dst);
}

int32_t oracle_attn_forward_rows(const aihost_attn_desc* desc, int32_t batch, int32_t n_new,
                                 const void* q, const void* k_new, const void* v_new,
                                 void* k_cache, void* v_cache, const int32_t* seq_len, void* out,
                                 int32_t mode, int32_t b0, int32_t b1, int32_t h0, int32_t h1,
                                 int32_t r0, int32_t r1) {
  if (!desc || !q || !k_new || !v_new || !k_cache || !v_cache || !seq_len || !out) return 1;
  if (r0 < 0 || r1 > n_new || r0 >= r1) return 1;
  const int32_t Hq = desc->n_q_heads, Hkv = desc->n_kv_heads, D = desc->head_dim;
  if (batch < 1 || n_new < 1 || Hq < 1 || Hkv < 1 || Hq % Hkv || D < 2 || D % 2 || D > 256) return 1;
  if (desc->kv_dtype == AIHOST_Q8_0 && D % 32) return 1;
  if (b0 < 0 || b1 > batch || b0 >= b1 || h0 < 0 || h1 > Hq || h0 >= h1) return 1;
  f16_lut_init();
  const int32_t group = Hq / Hkv;
  const float scale = desc->scale != 0.0f ? desc->scale : 1.0f / sqrtf((float)D);
  const int64_t head_stride = desc->kv_head_stride ? desc->kv_head_stride : dtype_row_bytes(desc->kv_dtype, D);
  const int64_t tok_stride = desc->kv_token_stride ? desc->kv_token_stride : head_stride * Hkv;
  const int64_t seq_stride = desc->kv_seq_stride ? desc->kv_seq_stride : tok_stride * desc->kv_capacity;
  const int64_t qe = (int64_t)n_new * Hq * D, ke = (int64_t)n_new * Hkv * D;
  const int64_t in_es = desc->q_dtype == AIHOST_F32 ? 4 : 2;
  const int64_t out_es = desc->out_dtype == AIHOST_F32 ? 4 : 2;
  const int32_t kvh0 = h0 / group, kvh1 = (h1 - 1) / group + 1;

  float* qf = (float*)malloc(sizeof(float) * (size_t)qe * (size_t)(b1 - b0));
  float* kf = (float*)malloc(sizeof(float) * (size_t)ke);
  float* vf = (float*)malloc(sizeof(float) * (size_t)ke);
  if (!qf || !kf || !vf) { free(qf); free(kf); free(vf); return 2; }

  /* 1. RoPE(Q), RoPE(K), KVCache.Add — ComputeOps.cs:1282-1296 */
  for (int32_t b = b0; b < b1; ++b) {
    const int32_t P = seq_len[b];
    if (P < 0 || P + n_new > desc->kv_capacity) { free(qf); free(kf); free(vf); return 1; }
    float* qb = qf + (int64_t)(b - b0) * qe;
    to_f32((const uint8_t*)q + (int64_t)b * qe * in_es, desc->q_dtype, qe, qb);
    to_f32((const uint8_t*)k_new + (int64_t)b * ke * in_es, desc->q_dtype, ke, kf);
    to_f32((const uint8_t*)v_new + (int64_t)b * ke * in_es, desc->q_dtype, ke, vf);
    /* only the query rows and heads this call attends, and the KV heads it appends */
    rope_part(qb, Hq, D, P, desc->rope_theta, desc->rope_mode, r0, r1, h0, h1);
    rope_part(kf, Hkv, D, P, desc->rope_theta, desc->rope_mode, 0, n_new, kvh0, kvh1);
    for (int32_t s = 0; s < n_new; ++s)
      for (int32_t h = kvh0; h < kvh1; ++h) {
        const int64_t off = (int64_t)b * seq_stride + (int64_t)(P + s) * tok_stride + (int64_t)h * head_stride;
        store_row((uint8_t*)k_cache + off, desc->kv_dtype, kf + ((int64_t)s * Hkv + h) * D, D);
        store_row((uint8_t*)v_cache + off, desc->kv_dtype, vf + ((int64_t)s * Hkv + h) * D, D);
      }
  }
  free(kf);
  free(vf);

  /* 2. MultiHeadAttention(Q, cachedK, cachedV, numHeads, position) — ComputeOps.cs:1304 */
  int32_t max_kv = 0;
  for (int32_t b = b0; b < b1; ++b) max_kv = seq_len[b] + n_new > max_kv ? seq_len[b] + n_new : max_kv;
  int32_t err = 0;
#pragma omp parallel
  {
    float* scores = (float*)malloc(sizeof(double) * (size_t)max_kv);
    float* rowbuf = (float*)malloc(sizeof(float) * 2 * (size_t)D);
    float* orow = (float*)malloc(sizeof(float) * (size_t)D);
    if (!scores || !rowbuf || !orow) {
#pragma omp atomic write
      err = 2;
    } else {
#pragma omp for collapse(3) schedule(dynamic, 1)
      for (int32_t b = b0; b < b1; ++b)
        for (int32_t h = h0; h < h1; ++h)
          for (int32_t i = r0; i < r1; ++i) {
            const int32_t P = seq_len[b];
            const kv_view kk = {(const uint8_t*)k_cache + (int64_t)b * seq_stride, desc->kv_dtype, tok_stride, head_stride};
            const kv_view vv = {(const uint8_t*)v_cache + (int64_t)b * seq_stride, desc->kv_dtype, tok_stride, head_stride};
            const int32_t n_vis = n_new == 1 ? P + 1 : P + i + 1;
            attend_row(qf + (int64_t)(b - b0) * qe + ((int64_t)i * Hq + h) * D, &kk, &vv, h / group, n_vis, D,
                       scale, mode, n_new == 1, scores, rowbuf, orow);
            const int64_t oidx = (int64_t)b * qe + ((int64_t)i * Hq + h) * D;
            if (desc->out_dtype == AIHOST_F32) memcpy((float*)out + oidx, orow, (size_t)D * 4);
            else oracle_f32_to_f16_n(orow, (uint16_t*)out + oidx, D);
          }
    }
    free(scores);
    free(rowbuf);
    free(orow);
  }
  (void)out_es;
  free(qf);
  return err;
}

int32_t oracle_attn_forward_part(const aihost_attn_desc* desc, int32_t batch, int32_t n_new,
                                 const void* q, const void* k_new, const void* v_new,
                                 void* k_cache, void* v_cache, const int32_t* seq_len, void* out,
                                 int32_t mode, int32_t b0, int32_t b1, int32_t h0, int32_t h1) {
  return oracle_attn_forward_rows(desc, batch, n_new, q, k_new, v_new, k_cache, v_cache, seq_len, out, mode, b0, b1,
                                  h0, h1, 0, n_new);
}

int32_t oracle_attn_forward(const aihost_attn_desc* desc, int32_t batch, int32_t n_new,
                            const void* q, const void* k_new, const void* v_new, void* k_cache,
                            void* v_cache, const int32_t* seq_len, void* out, int32_t mode) {
  if (!desc) return 1;
  return oracle_attn_forward_part(desc, batch, n_new, q, k_new, v_new, k_cache, v_cache, seq_len, out,
                                  mode, 0, batch, 0, desc->n_q_heads);
}

/* ------------------------------------------------------------------ weights beside the op
 * GGUF K-quant dequantisation, restated from the reference's shaders (the inline sources the
 * reference runs: QuantizationFormats.cs DequantizeQ2K_Correct .. DequantizeQ6K_Correct, chosen
 * by ComputeShaders.cs:12-16 since no dequant .glsl is deployed). Each value is evaluated in the
 * shader's order, one fp32 rounding per operation (this file is built without contraction). */
static float kq_f16(const uint8_t* p) { return oracle_f16_to_f32((uint16_t)(p[0] | (p[1] << 8))); }

static void kq_scale_min_k4(int j, const uint8_t* q, float* sc, float* mn) { /* get_scale_min_k4 */
  if (j < 4) {
    *sc = (float)(q[j] & 63);
    *mn = (float)(q[j + 4] & 63);
  } else {
    *sc = (float)((q[j + 4] & 0xF) | ((q[j - 4] >> 6) << 4));
    *mn = (float)((q[j + 4] >> 4) | ((q[j] >> 6) << 4));
  }
}

static float kq_value(int32_t kind, const uint8_t* b, int e) {
  switch (kind) {
    case 8: { /* Q2_K: scales[16] | qs[64] | d | dmin — QuantizationFormats.cs:20-56 */
      const uint8_t sc = b[e / 16];
      const int chunk = e / 128, local = e % 128;
      const int qv = (b[16 + chunk * 32 + local % 32] >> ((local / 32) * 2)) & 3;
      const float d = kq_f16(b + 80), dmin = kq_f16(b + 82);
      const float t = d * (float)(sc & 0xF);
      return t * (float)qv - dmin * (float)((sc >> 4) & 0xF);
    }
    case 9: { /* Q3_K: hmask[32] | qs[64] | scales[12] | d — QuantizationFormats.cs:65-128 */
      const int chunk = e / 128, local = e % 128;
      const int low2 = (b[32 + chunk * 32 + local % 32] >> ((local / 32) * 2)) & 3;
      const int high1 = (b[local % 32] >> (chunk * 4 + local / 32)) & 1;
      const int qval = (low2 | (high1 << 2)) - 4;
      const int is = e / 16, k = is % 4, ag = is / 4;
      const uint8_t* sc = b + 96;
      const int tmp = sc[8 + k];
      int sb;
      if (ag == 0) sb = (sc[k] & 0xF) | (((tmp >> 0) & 3) << 4);
      else if (ag == 1) sb = (sc[k + 4] & 0xF) | (((tmp >> 2) & 3) << 4);
      else if (ag == 2) sb = ((sc[k] >> 4) & 0xF) | (((tmp >> 4) & 3) << 4);
      else sb = ((sc[k + 4] >> 4) & 0xF) | (((tmp >> 6) & 3) << 4);
      const float dl = kq_f16(b + 108) * (float)(sb - 32);
      return dl * (float)qval;
    }
    case 10: { /* Q4_K: d | dmin | scales[12] | qs[128] — QuantizationFormats.cs:140-197 */
      const int group = e / 64, within = e % 64, upper = within >= 32;
      float sc, mn;
      kq_scale_min_k4(group * 2 + upper, b + 4, &sc, &mn);
      const int q = (b[16 + group * 32 + within % 32] >> (upper * 4)) & 0xF;
      const float t = kq_f16(b) * sc;
      return t * (float)q - kq_f16(b + 2) * mn;
    }
    case 11: { /* Q5_K: d | dmin | scales[12] | qh[32] | qs[128] — QuantizationFormats.cs:204-257 */
      float sc, mn;
      kq_scale_min_k4(e / 32, b + 4, &sc, &mn);
      const int j = e / 64, local = e % 64, upper = local >= 32, l = local % 32;
      const int ql = (b[48 + j * 32 + l] >> (upper * 4)) & 0xF;
      const int qh = (b[16 + j * 32 + l] >> (j * 2 + upper)) & 1;
      const float t = kq_f16(b) * sc;
      return t * (float)(ql | (qh << 4)) - kq_f16(b + 2) * mn;
    }
    case 12: { /* Q6_K: ql[128] | qh[64] | scales[16] | d — QuantizationFormats.cs:264-315 */
      const int half = e / 128, w = e % 128, quarter = w / 32, wq = w % 32;
      const int ql_extra = (quarter == 1 || quarter == 3) ? 32 : 0;
      const int upper = quarter >= 2;
      const int lower4 = (b[half * 64 + ql_extra + wq] >> (upper * 4)) & 0xF;
      const int upper2 = (b[128 + half * 32 + wq] >> (quarter * 2)) & 3;
      const int q = lower4 | (upper2 << 4);
      const float sc = (float)(int8_t)b[192 + e / 16];
      const float t = kq_f16(b + 208) * sc;
      return t * ((float)q - 32.0f);
    }
    default:
      return 0.0f;
  }
}

int32_t oracle_kquant_block_bytes(int32_t kind) {
  switch (kind) {
    case 8: return 84;
    case 9: return 110;
    case 10: return 144;
    case 11: return 176;
    case 12: return 210;
    default: return 0;
  }
}

int32_t oracle_dequantize(int32_t kind, const uint8_t* blocks, int64_t n, float* out) {
  const int32_t bb = oracle_kquant_block_bytes(kind);
  if (!bb || !blocks || !out || n < 0 || n % 256) return 1;
  f16_lut_init();
#pragma omp parallel for schedule(static)
  for (int64_t blk = 0; blk < n / 256; ++blk)
    for (int e = 0; e < 256; ++e) out[blk * 256 + e] = kq_value(kind, blocks + blk * bb, e);
  return 0;
}

/* ComputeOps.MatMulWeights (ComputeOps.cs:275-313; shader _inlineMatMulWeights in
 * ComputeShaders.cs): C [M, N] = A [M, K] . B, B GGUF column-major, element (k, n) at
 * w[n * K + k]. FAITHFUL: one fp32 accumulator per output, k ascending, as the shader's 16-wide
 * tiles visit them; EXACT: double accumulation. */
int32_t oracle_matmul_weights(const float* a, int32_t M, int32_t K, const float* w, int32_t N, float* c, int32_t mode) {
  if (!a || !w || !c || M < 1 || K < 1 || N < 1) return 1;
#pragma omp parallel for collapse(2) schedule(static)
  for (int32_t m = 0; m < M; ++m)
    for (int32_t n = 0; n < N; ++n) {
      const float* ar = a + (int64_t)m * K;
      const float* wr = w + (int64_t)n * K;
      if (mode == ORACLE_EXACT) {
        double acc = 0.0;
        for (int32_t k = 0; k < K; ++k) acc += (double)ar[k] * (double)wr[k];
        c[(int64_t)m * N + n] = (float)acc;
      } else {
        float acc = 0.0f;
        for (int32_t k = 0; k < K; ++k) acc += ar[k] * wr[k];
        c[(int64_t)m * N + n] = acc;
      }
    }
  return 0;
}
