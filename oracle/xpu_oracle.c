/*
 * xpu_oracle.c - CPU oracle for the xpu_playground decode hot path.
 *
 * TEST INFRASTRUCTURE ONLY. This file restates, in plain C, the reference's
 * CPU-side algorithms so that tests/, __graft_entry__.smoke() and the
 * cpu_baseline leg of bench.py can check (and time) the CUDA library. Nothing
 * in the product (libxpu_cuda.so, its C++ host programs) links or calls it.
 *
 * Sources restated (paths inside DanielSawczuk/xpu_playground):
 *   - bf16 codecs: qwen3/model.cpp:497-508; fp16 codecs: level_zero/peak_l0.cpp:740-785
 *   - GEMV host check: gemv.cpp:191-199 and level_zero/peak_l0.cpp:866-881
 *     (FP32 accumulation over decoded 16-bit inputs, in column order)
 *   - benchmark input generators: gemv.cpp:156-167, peak_mem_2d.cpp:36-47
 *   - Qwen3 operators: qwen3/kernels.hpp:24-246 (reference kernel semantics)
 *   - Qwen3 model step: qwen3/reference.py:11-45, i.e. the transformers
 *     Qwen3ForCausalLM eager/bf16 forward (third-party; its rounding points
 *     are restated in orc_qwen3_decode below)
 * The GEMM has no host reference in the reference (gemm.cpp:109-117 checks a
 * closed form only); orc_gemm is a plain FP32 triple loop.
 *
 * Build: oracle/build.py (gcc -O2 -fopenmp -ffp-contract=off). FP
 * contraction is off so that a*b+c rounds twice, like the separate
 * multiply/add the restated code performs.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------ codecs ---- */

/* Round-to-nearest-even fp32 -> bf16 (qwen3/model.cpp:497-502). */
uint16_t orc_f32_to_bf16(float value) {
  uint32_t bits;
  memcpy(&bits, &value, 4);
  if ((bits & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((bits >> 16) | 0x40u); /* keep NaN a NaN */
  bits += 0x7fffu + ((bits >> 16) & 1u);
  return (uint16_t)(bits >> 16);
}

float orc_bf16_to_f32(uint16_t v) { /* qwen3/model.cpp:503-508 */
  uint32_t bits = (uint32_t)v << 16;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static inline float rb(float v) { return orc_bf16_to_f32(orc_f32_to_bf16(v)); }

/* RNE fp32 -> fp16 with subnormals and overflow (level_zero/peak_l0.cpp:740-764). */
uint16_t orc_f32_to_f16(float value) {
  uint32_t bits;
  memcpy(&bits, &value, 4);
  const uint32_t sign = (bits >> 16) & 0x8000u;
  const uint32_t absbits = bits & 0x7fffffffu;
  if (absbits > 0x7f800000u) return (uint16_t)(sign | 0x7e00u);
  int exponent = (int)((bits >> 23) & 0xffu) - 127 + 15;
  uint32_t mantissa = bits & 0x7fffffu;
  if (exponent <= 0) {
    if (exponent < -10) return (uint16_t)sign;
    mantissa = (mantissa | 0x800000u);
    const int shift = 14 - exponent;
    const uint32_t half = 1u << (shift - 1);
    const uint32_t rest = mantissa & ((1u << shift) - 1u);
    uint32_t result = mantissa >> shift;
    if (rest > half || (rest == half && (result & 1u))) ++result;
    return (uint16_t)(sign | result);
  }
  if (exponent >= 31) return (uint16_t)(sign | 0x7c00u);
  mantissa += 0xfffu + ((mantissa >> 13) & 1u);
  if (mantissa & 0x800000u) {
    mantissa = 0;
    if (++exponent >= 31) return (uint16_t)(sign | 0x7c00u);
  }
  return (uint16_t)(sign | ((uint32_t)exponent << 10) | (mantissa >> 13));
}

float orc_f16_to_f32(uint16_t value) { /* level_zero/peak_l0.cpp:766-785 */
  const uint32_t sign = (uint32_t)(value & 0x8000u) << 16;
  uint32_t exponent = (value >> 10) & 0x1fu;
  uint32_t mantissa = value & 0x3ffu;
  uint32_t bits;
  if (exponent == 0) {
    if (mantissa == 0) {
      bits = sign;
    } else {
      int shift = 0;
      while ((mantissa & 0x400u) == 0) { mantissa <<= 1; ++shift; }
      mantissa &= 0x3ffu;
      bits = sign | ((uint32_t)(127 - 14 - shift) << 23) | (mantissa << 13);
    }
  } else if (exponent == 31) {
    bits = sign | 0x7f800000u | (mantissa << 13);
  } else {
    bits = sign | ((exponent + 112u) << 23) | (mantissa << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

static inline float dec16(uint16_t v, int fp16) { return fp16 ? orc_f16_to_f32(v) : orc_bf16_to_f32(v); }
static inline uint16_t enc16(float v, int fp16) { return fp16 ? orc_f32_to_f16(v) : orc_f32_to_bf16(v); }

void orc_encode16(const float *in, uint16_t *out, uint64_t n, int fp16) {
  for (uint64_t i = 0; i < n; ++i) out[i] = enc16(in[i], fp16);
}
void orc_decode16(const uint16_t *in, float *out, uint64_t n, int fp16) {
  for (uint64_t i = 0; i < n; ++i) out[i] = dec16(in[i], fp16);
}

/* ------------------------------------------------------- generators ---- */

/* The reference's integer hash (gemv.cpp:157-162, peak_mem_2d.cpp:94-99). */
uint32_t orc_hash_u32(uint32_t bits) {
  bits ^= bits >> 16;
  bits *= 0x7feb352du;
  bits ^= bits >> 15;
  bits *= 0x846ca68bu;
  bits ^= bits >> 16;
  return bits;
}

/* GEMV benchmark matrix / vector values (gemv.cpp:163, 166-167). */
void orc_gemv_bench_inputs(uint16_t *matrix, uint16_t *vector, uint32_t m, uint32_t k, int fp16) {
  for (uint64_t i = 0; i < (uint64_t)m * k; ++i)
    matrix[i] = enc16(0.25f + (float)(orc_hash_u32((uint32_t)i) & 255u) / 1024.0f, fp16);
  for (uint32_t i = 0; i < k; ++i) {
    const uint32_t bits = i * 747796405u;
    vector[i] = enc16(0.5f + (float)((bits >> 16) & 127u) / 512.0f, fp16);
  }
}

/* peak_mem_2d.cpp:93-101 */
float orc_peak_mem_value(uint64_t index) {
  return 1.0f + (float)(orc_hash_u32((uint32_t)index) & 0xffffu) * (1.0f / 65536.0f);
}

/* splitmix64 finaliser: the seeded generators below (shared bit-for-bit with
 * the device generators in libxpu_cuda's synthetic-data kernels). */
static inline uint64_t mix64(uint64_t z) {
  z += 0x9E3779B97F4A7C15ull;
  z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
  z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
  return z ^ (z >> 31);
}

uint64_t orc_stream_base(uint64_t seed, uint64_t tag) { return mix64(seed ^ (tag * 0xD1B54A32D192ED03ull)); }

/* uniform[-1, 1) on a 2^-23 grid, then rounded to bf16/fp16 */
void orc_fill_uniform16(uint16_t *out, uint64_t n, uint64_t seed, uint64_t tag, int fp16) {
  const uint64_t base = orc_stream_base(seed, tag);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (int64_t)n; ++i) {
    const uint64_t h = mix64(base + (uint64_t)i);
    const float u = (float)((int32_t)(h >> 40) - 8388608) * (1.0f / 8388608.0f);
    out[i] = enc16(u, fp16);
  }
}

/* Approximately N(0, std^2): the Irwin-Hall sum of twelve 10-bit uniforms,
 * centred and scaled (variance of the sum is 1024^2 - 1), rounded to bf16. */
void orc_fill_normal_bf16(uint16_t *out, uint64_t n, uint64_t seed, uint64_t tag, float std) {
  const uint64_t base = orc_stream_base(seed, tag);
  const float scale = std * (1.0f / 1024.0f);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < (int64_t)n; ++i) {
    const uint64_t h1 = mix64(base + 2 * (uint64_t)i), h2 = mix64(base + 2 * (uint64_t)i + 1);
    int32_t sum = 0;
    for (int j = 0; j < 6; ++j) sum += (int32_t)((h1 >> (10 * j)) & 1023u) + (int32_t)((h2 >> (10 * j)) & 1023u);
    out[i] = orc_f32_to_bf16((float)(sum - 6138) * scale);
  }
}

/* ------------------------------------------------------- GEMV / GEMM ---- */

/* y[r] = sum_c A[r,c] * x[c], FP32, column order (gemv.cpp:191-196). */
void orc_gemv(const uint16_t *A, const uint16_t *x, float *y, uint32_t m, uint32_t k, int fp16) {
  float *xf = (float *)malloc(sizeof(float) * k);
  for (uint32_t c = 0; c < k; ++c) xf[c] = dec16(x[c], fp16);
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < (int64_t)m; ++r) {
    const uint16_t *row = A + (uint64_t)r * k;
    float acc = 0.0f;
    for (uint32_t c = 0; c < k; ++c) acc += dec16(row[c], fp16) * xf[c];
    y[r] = acc;
  }
  free(xf);
}

/* C[m,n] = sum_k A[m,k] B[k,n] in FP32 (row-major). Rows of C are split
 * across threads; each accumulates over k in order. */
void orc_gemm(const uint16_t *A, const uint16_t *B, float *C, uint32_t m, uint32_t n, uint32_t k,
              int fp16) {
  float *bf = (float *)malloc(sizeof(float) * (uint64_t)k * n);
  for (uint64_t i = 0; i < (uint64_t)k * n; ++i) bf[i] = dec16(B[i], fp16);
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < (int64_t)m; ++r) {
    float *crow = C + (uint64_t)r * n;
    for (uint32_t j = 0; j < n; ++j) crow[j] = 0.0f;
    for (uint32_t kk = 0; kk < k; ++kk) {
      const float a = dec16(A[(uint64_t)r * k + kk], fp16);
      const float *brow = bf + (uint64_t)kk * n;
      for (uint32_t j = 0; j < n; ++j) crow[j] += a * brow[j];
    }
  }
  free(bf);
}

int orc_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

void orc_set_num_threads(int n) {
#ifdef _OPENMP
  omp_set_num_threads(n);
#else
  (void)n;
#endif
}

/* ------------------------------- Qwen3 operators (kernels.hpp semantics) ---- */

#define HD 128u

void orc_embedding(const uint16_t *table, uint16_t *out, uint32_t token, uint32_t width) {
  memcpy(out, table + (uint64_t)token * width, (size_t)width * 2); /* kernels.hpp:29-33 */
}

/* kernels.hpp:43-55: out = bf16(x * w * rsqrt(sum/width + eps)) */
void orc_rms_norm(const uint16_t *in, const uint16_t *w, uint16_t *out, uint32_t width, float eps) {
  float sum = 0.0f;
  for (uint32_t i = 0; i < width; ++i) {
    const float v = orc_bf16_to_f32(in[i]);
    sum += v * v;
  }
  const float scale = 1.0f / sqrtf(sum / (float)width + eps);
  for (uint32_t i = 0; i < width; ++i)
    out[i] = orc_f32_to_bf16(orc_bf16_to_f32(in[i]) * orc_bf16_to_f32(w[i]) * scale);
}

static void head_norm_ref(uint16_t *v, const uint16_t *w) {
  float sum = 0.0f;
  for (uint32_t i = 0; i < HD; ++i) {
    const float x = orc_bf16_to_f32(v[i]);
    sum += x * x;
  }
  const float scale = 1.0f / sqrtf(sum / (float)HD + 1.0e-6f);
  for (uint32_t i = 0; i < HD; ++i) v[i] = orc_f32_to_bf16(orc_bf16_to_f32(v[i]) * orc_bf16_to_f32(w[i]) * scale);
}

static void head_rope_ref(const uint16_t *in, uint16_t *out, const uint16_t *c, const uint16_t *s) {
  for (uint32_t i = 0; i < HD / 2; ++i) {
    const float a = orc_bf16_to_f32(in[i]), b = orc_bf16_to_f32(in[i + 64]);
    const float ca = orc_bf16_to_f32(c[i]), sa = orc_bf16_to_f32(s[i]);
    const float cb = orc_bf16_to_f32(c[i + 64]), sb = orc_bf16_to_f32(s[i + 64]);
    out[i] = orc_f32_to_bf16(a * ca - b * sa);
    out[i + 64] = orc_f32_to_bf16(b * cb + a * sb);
  }
}

/* kernels.hpp:71-154 (generic head counts) */
void orc_qkv_rope_cache(uint16_t *query, uint16_t *key, const uint16_t *value, const uint16_t *qn,
                        const uint16_t *kn, const uint16_t *cos_t, const uint16_t *sin_t,
                        uint16_t *key_cache, uint16_t *value_cache, uint32_t position,
                        uint32_t max_seq, uint32_t q_heads, uint32_t kv_heads) {
  if (position >= max_seq) return;
  const uint16_t *c = cos_t + (uint64_t)position * HD, *s = sin_t + (uint64_t)position * HD;
  uint16_t tmp[HD];
  for (uint32_t h = 0; h < q_heads; ++h) {
    uint16_t *q = query + (uint64_t)h * HD;
    head_norm_ref(q, qn);
    head_rope_ref(q, tmp, c, s);
    memcpy(q, tmp, sizeof(tmp));
  }
  for (uint32_t h = 0; h < kv_heads; ++h) {
    uint16_t *k = key + (uint64_t)h * HD;
    const uint64_t slot = ((uint64_t)position * kv_heads + h) * HD;
    head_norm_ref(k, kn);
    head_rope_ref(k, key_cache + slot, c, s);
    memcpy(value_cache + slot, value + (uint64_t)h * HD, HD * 2);
  }
}

/* kernels.hpp:164-191: serial online softmax per head, scale 1/sqrt(128) */
void orc_attention(const uint16_t *query, const uint16_t *key_cache, const uint16_t *value_cache,
                   uint16_t *out, uint32_t position, uint32_t q_heads, uint32_t kv_heads) {
  const float scale = 0.08838834764831845f;
  const uint32_t group = q_heads / kv_heads;
  for (uint32_t h = 0; h < q_heads; ++h) {
    const uint32_t kvh = h / group;
    float q[HD], acc[HD];
    for (uint32_t i = 0; i < HD; ++i) { q[i] = orc_bf16_to_f32(query[(uint64_t)h * HD + i]); acc[i] = 0.0f; }
    float maximum = -INFINITY, denom = 0.0f;
    for (uint32_t t = 0; t <= position; ++t) {
      const uint64_t off = ((uint64_t)t * kv_heads + kvh) * HD;
      float score = 0.0f;
      for (uint32_t i = 0; i < HD; ++i) score += q[i] * orc_bf16_to_f32(key_cache[off + i]);
      score *= scale;
      const float nm = maximum > score ? maximum : score;
      const float old_scale = expf(maximum - nm), new_scale = expf(score - nm);
      for (uint32_t i = 0; i < HD; ++i) acc[i] = acc[i] * old_scale + orc_bf16_to_f32(value_cache[off + i]) * new_scale;
      denom = denom * old_scale + new_scale;
      maximum = nm;
    }
    for (uint32_t i = 0; i < HD; ++i) out[(uint64_t)h * HD + i] = orc_f32_to_bf16(acc[i] / denom);
  }
}

void orc_add(uint16_t *left, const uint16_t *right, uint32_t width) { /* kernels.hpp:198-206 */
  for (uint32_t i = 0; i < width; ++i) left[i] = orc_f32_to_bf16(orc_bf16_to_f32(left[i]) + orc_bf16_to_f32(right[i]));
}

void orc_silu_multiply(uint16_t *gate, const uint16_t *up, uint32_t width) { /* kernels.hpp:213-222 */
  for (uint32_t i = 0; i < width; ++i) {
    const float g = orc_bf16_to_f32(gate[i]);
    gate[i] = orc_f32_to_bf16(g / (1.0f + expf(-g)) * orc_bf16_to_f32(up[i]));
  }
}

uint32_t orc_argmax(const uint16_t *values, uint32_t width) { /* kernels.hpp:229-245 */
  float best = -INFINITY;
  uint32_t best_index = 0;
  for (uint32_t i = 0; i < width; ++i) {
    const float v = orc_bf16_to_f32(values[i]);
    if (v != v || v == INFINITY || v == -INFINITY) return 0xffffffffu;
    if (v > best) { best = v; best_index = i; }
  }
  return best_index;
}

/* ----------------------------------- Qwen3 decode step (transformers) ---- */
/*
 * One greedy decode step of Qwen3ForCausalLM in bf16 with eager attention,
 * with the rounding points of the transformers modelling code that
 * qwen3/reference.py runs:
 *   RMSNorm:  t = bf16(x * RN(1/RN(sqrt(mean(x^2) + eps)))), out = bf16(w * t)
 *   Linear:   bf16(FP32 dot product)
 *   RoPE:     bf16(bf16(q*cos) + bf16(rotate_half(q)*sin)), cos/sin bf16 tables
 *   scores:   bf16(bf16(q.k) * scale), softmax in FP32, probabilities -> bf16,
 *             output bf16(sum p*v)
 *   MLP:      bf16(bf16(silu(bf16 g)) * bf16 u); residual adds in bf16.
 * Tensor order in `w`: embed, final_norm, lm_head, then per layer:
 * input_norm, post_norm, q, k, v, o, q_norm, k_norm, gate, up, down.
 */
typedef struct {
  uint32_t hidden, intermediate, q_heads, kv_heads, layers, vocab, max_seq;
  float eps;
} orc_qwen3_config;

static void rms_hf(const uint16_t *x, const uint16_t *w, uint16_t *out, uint32_t n, float eps) {
  float sum = 0.0f;
  for (uint32_t i = 0; i < n; ++i) {
    const float v = orc_bf16_to_f32(x[i]);
    sum += v * v;
  }
  const float r = 1.0f / sqrtf(sum / (float)n + eps);
  for (uint32_t i = 0; i < n; ++i) {
    const float t = rb(orc_bf16_to_f32(x[i]) * r);
    out[i] = orc_f32_to_bf16(orc_bf16_to_f32(w[i]) * t);
  }
}

static void linear_bf16(const uint16_t *W, const uint16_t *x, uint16_t *y, uint32_t rows, uint32_t cols) {
#pragma omp parallel for schedule(static)
  for (int64_t r = 0; r < (int64_t)rows; ++r) {
    const uint16_t *row = W + (uint64_t)r * cols;
    float acc = 0.0f;
    for (uint32_t c = 0; c < cols; ++c) acc += orc_bf16_to_f32(row[c]) * orc_bf16_to_f32(x[c]);
    y[r] = orc_f32_to_bf16(acc);
  }
}

static void rope_hf(uint16_t *v, const uint16_t *c, const uint16_t *s) {
  uint16_t out[HD];
  for (uint32_t i = 0; i < HD / 2; ++i) {
    const float a = orc_bf16_to_f32(v[i]), b = orc_bf16_to_f32(v[i + 64]);
    const float lo = rb(a * orc_bf16_to_f32(c[i])) + rb(-b * orc_bf16_to_f32(s[i]));
    const float hi = rb(b * orc_bf16_to_f32(c[i + 64])) + rb(a * orc_bf16_to_f32(s[i + 64]));
    out[i] = orc_f32_to_bf16(lo);
    out[i + 64] = orc_f32_to_bf16(hi);
  }
  memcpy(v, out, sizeof(out));
}

/* RoPE tables as transformers' default rope builds them: inv_freq in FP32 as
 * 1 / theta^(2i/128), angle = FP32(position * inv_freq), cos/sin in FP32,
 * rounded to bf16; dimension d uses frequency d % 64. */
void orc_rope_tables(uint16_t *cos_t, uint16_t *sin_t, uint32_t max_seq, float theta) {
  float inv[HD / 2];
  for (uint32_t i = 0; i < HD / 2; ++i) inv[i] = 1.0f / powf(theta, (float)(2 * i) / (float)HD);
  for (uint32_t p = 0; p < max_seq; ++p)
    for (uint32_t d = 0; d < HD; ++d) {
      const float angle = (float)p * inv[d % (HD / 2)];
      cos_t[(uint64_t)p * HD + d] = orc_f32_to_bf16(cosf(angle));
      sin_t[(uint64_t)p * HD + d] = orc_f32_to_bf16(sinf(angle));
    }
}

/* Returns the greedy token (0xffffffff on NaN/Inf logits). logits (vocab,
 * bf16) may be NULL. key/value caches: [layers][max_seq][kv_heads][128]. */
uint32_t orc_qwen3_decode(const orc_qwen3_config *cfg, const uint16_t *const *w, uint16_t *key_cache,
                          uint16_t *value_cache, const uint16_t *cos_t, const uint16_t *sin_t,
                          uint32_t token, uint32_t position, uint16_t *logits) {
  const uint32_t H = cfg->hidden, I = cfg->intermediate, QH = cfg->q_heads, KVH = cfg->kv_heads;
  const uint32_t G = QH / KVH;
  const float scale = 0.08838834764831845f;
  uint16_t *x = malloc(H * 2), *xn = malloc(H * 2), *q = malloc(QH * HD * 2), *k = malloc(KVH * HD * 2);
  uint16_t *v = malloc(KVH * HD * 2), *att = malloc(QH * HD * 2), *y = malloc(H * 2);
  uint16_t *g = malloc((size_t)I * 2), *u = malloc((size_t)I * 2);
  float *scores = malloc(sizeof(float) * (position + 1));
  uint16_t *lg = logits ? logits : malloc((size_t)cfg->vocab * 2);
  memcpy(x, w[0] + (uint64_t)token * H, H * 2);
  const uint16_t *c = cos_t + (uint64_t)position * HD, *s = sin_t + (uint64_t)position * HD;
  for (uint32_t l = 0; l < cfg->layers; ++l) {
    const uint16_t *const *L = w + 3 + 11 * l;
    uint16_t *kc = key_cache + (uint64_t)l * cfg->max_seq * KVH * HD;
    uint16_t *vc = value_cache + (uint64_t)l * cfg->max_seq * KVH * HD;
    rms_hf(x, L[0], xn, H, cfg->eps);
    linear_bf16(L[2], xn, q, QH * HD, H);
    linear_bf16(L[3], xn, k, KVH * HD, H);
    linear_bf16(L[4], xn, v, KVH * HD, H);
    for (uint32_t h = 0; h < QH; ++h) { rms_hf(q + h * HD, L[6], q + h * HD, HD, cfg->eps); rope_hf(q + h * HD, c, s); }
    for (uint32_t h = 0; h < KVH; ++h) {
      rms_hf(k + h * HD, L[7], k + h * HD, HD, cfg->eps);
      rope_hf(k + h * HD, c, s);
      memcpy(kc + ((uint64_t)position * KVH + h) * HD, k + h * HD, HD * 2);
      memcpy(vc + ((uint64_t)position * KVH + h) * HD, v + h * HD, HD * 2);
    }
    for (uint32_t h = 0; h < QH; ++h) {
      const uint32_t kvh = h / G;
      float maximum = -INFINITY;
      for (uint32_t t = 0; t <= position; ++t) {
        const uint16_t *kr = kc + ((uint64_t)t * KVH + kvh) * HD;
        float dot = 0.0f;
        for (uint32_t i = 0; i < HD; ++i) dot += orc_bf16_to_f32(q[h * HD + i]) * orc_bf16_to_f32(kr[i]);
        scores[t] = rb(rb(dot) * scale);
        if (scores[t] > maximum) maximum = scores[t];
      }
      float sum = 0.0f;
      for (uint32_t t = 0; t <= position; ++t) { scores[t] = expf(scores[t] - maximum); sum += scores[t]; }
      float acc[HD];
      for (uint32_t i = 0; i < HD; ++i) acc[i] = 0.0f;
      for (uint32_t t = 0; t <= position; ++t) {
        const float p = rb(scores[t] / sum);
        const uint16_t *vr = vc + ((uint64_t)t * KVH + kvh) * HD;
        for (uint32_t i = 0; i < HD; ++i) acc[i] += p * orc_bf16_to_f32(vr[i]);
      }
      for (uint32_t i = 0; i < HD; ++i) att[h * HD + i] = orc_f32_to_bf16(acc[i]);
    }
    linear_bf16(L[5], att, y, H, QH * HD);
    for (uint32_t i = 0; i < H; ++i) x[i] = orc_f32_to_bf16(orc_bf16_to_f32(x[i]) + orc_bf16_to_f32(y[i]));
    rms_hf(x, L[1], xn, H, cfg->eps);
    linear_bf16(L[8], xn, g, I, H);
    linear_bf16(L[9], xn, u, I, H);
    for (uint32_t i = 0; i < I; ++i) {
      const float gv = orc_bf16_to_f32(g[i]);
      const float act = rb(gv / (1.0f + expf(-gv)));
      g[i] = orc_f32_to_bf16(act * orc_bf16_to_f32(u[i]));
    }
    linear_bf16(L[10], g, y, H, I);
    for (uint32_t i = 0; i < H; ++i) x[i] = orc_f32_to_bf16(orc_bf16_to_f32(x[i]) + orc_bf16_to_f32(y[i]));
  }
  rms_hf(x, w[1], xn, H, cfg->eps);
  linear_bf16(w[2], xn, lg, cfg->vocab, H);
  const uint32_t next = orc_argmax(lg, cfg->vocab);
  free(x); free(xn); free(q); free(k); free(v); free(att); free(y); free(g); free(u); free(scores);
  if (!logits) free(lg);
  return next;
}
