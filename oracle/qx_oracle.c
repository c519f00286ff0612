/*
 * qx_oracle.c — CPU restatement of qx's GQA attention path.
 *
 * TEST INFRASTRUCTURE ONLY: the parity checker for qx_b200's CUDA kernels
 * and the timed CPU baseline. The product never links or calls this file.
 *
 * Parity is pinned by the reference's own golden bits (exp, rsqrt, RoPE
 * sin/cos from crates/qx-consensus-math/src/lib.rs:267-330) and its unit
 * tests (crates/qx-runtime/src/lib.rs:2873-2902); tests/golden holds them.
 *
 * Compile with -O2 -ffp-contract=off (no fast-math): every `a * b` and
 * `a + b` below must round separately, as in the Rust source.
 */
#include "qx_oracle.h"

#include <float.h>
#include <math.h>
#include <stdlib.h>
#include <string.h>
#include <pthread.h>

/* Minimal parallel-for over [0, n) on `threads` POSIX threads with an atomic
 * work counter (the image has no OpenMP runtime). */
typedef void (*qxo_body)(void* ctx, int index);
typedef struct {
  qxo_body body;
  void* ctx;
  int n;
  int next;
} qxo_pool;
static void* qxo_worker(void* arg) {
  qxo_pool* pool = (qxo_pool*)arg;
  for (;;) {
    int i = __atomic_fetch_add(&pool->next, 1, __ATOMIC_RELAXED);
    if (i >= pool->n) break;
    pool->body(pool->ctx, i);
  }
  return NULL;
}
static void qxo_parallel_for(int n, int threads, qxo_body body, void* ctx) {
  qxo_pool pool = {body, ctx, n, 0};
  if (threads > n) threads = n;
  if (threads <= 1) {
    qxo_worker(&pool);
    return;
  }
  pthread_t* tids = (pthread_t*)malloc(sizeof(pthread_t) * (size_t)(threads - 1));
  int started = 0;
  for (int t = 0; t < threads - 1; ++t)
    if (pthread_create(&tids[t], NULL, qxo_worker, &pool) == 0) ++started;
  qxo_worker(&pool);
  for (int t = 0; t < started; ++t) pthread_join(tids[t], NULL);
  free(tids);
}

/* Granite shape constants, crates/qx-model/src/lib.rs:9-25. */
#define G_HIDDEN 1024
#define G_HEADS 16
#define G_KV_HEADS 8
#define G_HEAD_DIM 64
#define G_MAX_CONTEXT 4096
#define G_ATTENTION_MULTIPLIER 0.015625f

/* Qwen3-30B-A3B attention shape, tools/qx-qwen-parity/src/main.rs:1218-1224. */
#define Q_HEADS 32
#define Q_KV_HEADS 4
#define Q_HEAD_DIM 128

static inline float fb(uint32_t bits) {
  float f;
  memcpy(&f, &bits, 4);
  return f;
}
static inline uint32_t bf(float f) {
  uint32_t b;
  memcpy(&b, &f, 4);
  return b;
}

/* crates/qx-consensus-math/src/lib.rs:28-61 */
static const uint32_t INVFREQ_BITS[32] = {
    0x3f800000, 0x3f3ff911, 0x3f0ff59a, 0x3ed7e89b, 0x3ea1e89b, 0x3e72d424,
    0x3e361887, 0x3e088d77, 0x3dcccccd, 0x3d99940e, 0x3d6655c3, 0x3d2cba15,
    0x3d0186e2, 0x3cc24350, 0x3c91ad39, 0x3c5a7bf1, 0x3c23d70a, 0x3bf5b9b0,
    0x3bb8449c, 0x3b8a2e77, 0x3b4f3e37, 0x3b1b690d, 0x3ae91528, 0x3aaec98e,
    0x3a83126f, 0x3a44948c, 0x3a136a16, 0x39dd1726, 0x39a5cb5f, 0x3978a814,
    0x393a7753, 0x390bd472};

uint32_t qxo_granite_inverse_frequency_bits(uint32_t pair) {
  return pair < 32 ? INVFREQ_BITS[pair] : 0u;
}

/* exp_f32, crates/qx-consensus-math/src/lib.rs:70-110. Returns 0 for None. */
int qxo_exp_f32(float x, float* out) {
  if (!isfinite(x)) return 0;
  if (x < -87.0f) {
    *out = 0.0f;
    return 1;
  }
  if (x > 88.0f) {
    *out = FLT_MAX;
    return 1;
  }
  float scaled = fmaf(x, fb(0x3fb8aa3b), 0.0f);
  float rounded = scaled >= 0.0f ? scaled + 0.5f : scaled - 0.5f;
  int32_t exponent = (int32_t)rounded; /* truncation toward zero */
  float exponent_f32 = (float)exponent;
  float reduced = fmaf(-exponent_f32, fb(0x3f317200), x);
  reduced = fmaf(-exponent_f32, fb(0x35bfbe8e), reduced);
  float p = fb(0x39500d01);
  p = fmaf(p, reduced, fb(0x3ab60b61));
  p = fmaf(p, reduced, fb(0x3c088889));
  p = fmaf(p, reduced, fb(0x3d2aaaab));
  p = fmaf(p, reduced, fb(0x3e2aaaab));
  p = fmaf(p, reduced, fb(0x3f000000));
  p = fmaf(p, reduced, 1.0f);
  p = fmaf(p, reduced, 1.0f);
  float power_of_two = fb((uint32_t)(exponent + 127) << 23);
  float result = p * power_of_two;
  if (!isfinite(result)) return 0;
  *out = result;
  return 1;
}

/* rsqrt_f32, crates/qx-consensus-math/src/lib.rs:114-128. */
int qxo_rsqrt_f32(float x, float* out) {
  if (!isfinite(x) || x <= 0.0f) return 0;
  float half = x * 0.5f;
  float estimate = fb(0x5f375a86u - (bf(x) >> 1));
  for (int i = 0; i < 4; ++i) {
    float square = estimate * estimate;
    float correction = fmaf(-half, square, 1.5f);
    estimate = estimate * correction;
  }
  if (!isfinite(estimate)) return 0;
  *out = estimate;
  return 1;
}

/* sin_cos_f32, crates/qx-consensus-math/src/lib.rs:148-189. */
int qxo_sin_cos_f32(float angle, float* s, float* c) {
  if (!isfinite(angle) || fabsf(angle) > 4096.0f) return 0;
  float scaled = fmaf(angle, fb(0x3e22f983), 0.0f);
  float rounded = scaled >= 0.0f ? scaled + 0.5f : scaled - 0.5f;
  int32_t turns = (int32_t)rounded;
  float turns_f32 = (float)turns;
  float reduced = fmaf(-turns_f32, fb(0x40c90fdb), angle);
  reduced = fmaf(-turns_f32, fb(0xb43bbd2e), reduced);
  float cosine_sign = 1.0f;
  if (reduced > fb(0x3fc90fdb)) {
    reduced = fb(0x40490fdb) - reduced;
    cosine_sign = -1.0f;
  } else if (reduced < -fb(0x3fc90fdb)) {
    reduced = -fb(0x40490fdb) - reduced;
    cosine_sign = -1.0f;
  }
  float square = reduced * reduced;
  float sp = fb(0x2f309231);
  sp = fmaf(sp, square, fb(0xb2d7322b));
  sp = fmaf(sp, square, fb(0x3638ef1d));
  sp = fmaf(sp, square, fb(0xb9500d01));
  sp = fmaf(sp, square, fb(0x3c088889));
  sp = fmaf(sp, square, fb(0xbe2aaaab));
  float sine = fmaf(sp * square, reduced, reduced);
  float cp = fb(0x310f76c7);
  cp = fmaf(cp, square, fb(0xb493f27e));
  cp = fmaf(cp, square, fb(0x37d00d01));
  cp = fmaf(cp, square, fb(0xbab60b61));
  cp = fmaf(cp, square, fb(0x3d2aaaab));
  cp = fmaf(cp, square, fb(0xbf000000));
  float cosine = fmaf(cp, square, 1.0f) * cosine_sign;
  *s = sine;
  *c = cosine;
  return 1;
}

/* granite_rope_sin_cos, crates/qx-consensus-math/src/lib.rs:192-195. */
int qxo_granite_rope_sin_cos(uint32_t position, uint32_t pair, float* s,
                             float* c) {
  if (pair >= 32) return 0;
  float inverse = fb(INVFREQ_BITS[pair]);
  return qxo_sin_cos_f32((float)position * inverse, s, c);
}

/* granite_rope_pair, crates/qx-consensus-math/src/lib.rs:199-207. */
int qxo_granite_rope_pair(uint32_t position, uint32_t pair, float left,
                          float right, float* first, float* second) {
  if (!isfinite(left) || !isfinite(right)) return 0;
  float s, c;
  if (!qxo_granite_rope_sin_cos(position, pair, &s, &c)) return 0;
  float a = fmaf(-right, s, left * c);
  float b = fmaf(right, c, left * s);
  if (!isfinite(a) || !isfinite(b)) return 0;
  *first = a;
  *second = b;
  return 1;
}

/* reduce_simd32, crates/qx-runtime/src/lib.rs:2298-2306. */
float qxo_reduce_simd32(const float* in) {
  float lanes[32];
  memcpy(lanes, in, sizeof(lanes));
  for (int offset = 16; offset >= 1; offset >>= 1)
    for (int lane = 0; lane < offset; ++lane) lanes[lane] += lanes[lane + offset];
  return lanes[0];
}

/* Error sweeps of the consensus-math tests (:217-236, :239-254, :298-311);
 * the native references are the double-rounded libm values. */
float qxo_exp_worst_relative_error(void) {
  float worst = 0.0f;
  for (int step = -87000; step <= 88000; ++step) {
    float input = (float)step / 1000.0f;
    float actual = 0.0f;
    qxo_exp_f32(input, &actual);
    float reference = expf(input);
    float rel = fabsf((actual - reference) / reference);
    if (rel > worst) worst = rel;
  }
  return worst;
}

float qxo_rsqrt_worst_relative_error(void) {
  float worst = 0.0f;
  for (int e = -20; e <= 20; ++e)
    for (int m = 1; m <= 1000; ++m) {
      float input = ((float)m / 1000.0f) * ldexpf(1.0f, e);
      float actual = 0.0f;
      qxo_rsqrt_f32(input, &actual);
      float reference = 1.0f / sqrtf(input);
      float rel = fabsf((actual - reference) / reference);
      if (rel > worst) worst = rel;
    }
  return worst;
}

float qxo_rope_worst_absolute_error(void) {
  float worst = 0.0f;
  for (uint32_t position = 0; position < 4096; ++position)
    for (uint32_t pair = 0; pair < 32; ++pair) {
      float angle = (float)position * fb(INVFREQ_BITS[pair]);
      float s = 0.0f, c = 0.0f;
      qxo_granite_rope_sin_cos(position, pair, &s, &c);
      float ds = fabsf(s - sinf(angle)), dc = fabsf(c - cosf(angle));
      if (ds > worst) worst = ds;
      if (dc > worst) worst = dc;
    }
  return worst;
}

/* ---- element conversions ---- */
uint16_t qxo_f32_to_bf16(float f) {
  uint32_t u = bf(f);
  if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
  u += 0x7fffu + ((u >> 16) & 1u);
  return (uint16_t)(u >> 16);
}
float qxo_bf16_to_f32(uint16_t b) { return fb((uint32_t)b << 16); }
uint16_t qxo_f32_to_f16(float f) {
  _Float16 h = (_Float16)f; /* IEEE RNE, as half::f16::from_f32 */
  uint16_t bits;
  memcpy(&bits, &h, 2);
  return bits;
}
float qxo_f16_to_f32(uint16_t bits) {
  _Float16 h;
  memcpy(&h, &bits, 2);
  return (float)h;
}

static inline float load_elem(const void* base, size_t index, int dtype) {
  switch (dtype) {
    case QXO_BF16: return qxo_bf16_to_f32(((const uint16_t*)base)[index]);
    case QXO_F16: return qxo_f16_to_f32(((const uint16_t*)base)[index]);
    default: return ((const float*)base)[index];
  }
}
static inline void store_elem(void* base, size_t index, int dtype, float v) {
  switch (dtype) {
    case QXO_BF16: ((uint16_t*)base)[index] = qxo_f32_to_bf16(v); break;
    case QXO_F16: ((uint16_t*)base)[index] = qxo_f32_to_f16(v); break;
    default: ((float*)base)[index] = v; break;
  }
}

/* rotate_heads, crates/qx-runtime/src/lib.rs:2439-2453. */
int qxo_rotate_heads(float* values, int heads, uint32_t position) {
  for (int head = 0; head < heads; ++head) {
    int start = head * G_HEAD_DIM;
    for (int pair = 0; pair < G_HEAD_DIM / 2; ++pair) {
      float left = values[start + pair];
      float right = values[start + G_HEAD_DIM / 2 + pair];
      float first, second;
      if (!qxo_granite_rope_pair(position, (uint32_t)pair, left, right, &first,
                                 &second))
        return QXO_ERR_NONFINITE;
      values[start + pair] = first;
      values[start + G_HEAD_DIM / 2 + pair] = second;
    }
  }
  return QXO_OK;
}

/* cpu_rotate_heads, crates/qx-runtime-v2/src/lib.rs:4957-4970: the V2 CPU
 * twin's RoPE. Same sin/cos as rotate_heads, but the pair is rotated as
 * left*cos - right*sin and left*sin + right*cos with every product and sum
 * rounded on its own (no fma), so it differs from rotate_heads in the last
 * bits. The reference expects a registered coordinate (a panic otherwise). */
int qxo_cpu_rotate_heads(float* values, int heads, uint32_t position) {
  for (int head = 0; head < heads; ++head) {
    int start = head * G_HEAD_DIM;
    for (int pair = 0; pair < G_HEAD_DIM / 2; ++pair) {
      float s, c;
      if (!qxo_granite_rope_sin_cos(position, (uint32_t)pair, &s, &c)) return QXO_ERR_NONFINITE;
      const float left = values[start + pair];
      const float right = values[start + G_HEAD_DIM / 2 + pair];
      const float lc = left * c, rs = right * s, ls = left * s, rc = right * c;
      values[start + pair] = lc - rs;
      values[start + G_HEAD_DIM / 2 + pair] = ls + rc;
    }
  }
  return QXO_OK;
}

/* Rust's f32::max: a NaN operand yields the other operand. */
static inline float rust_max(float a, float b) {
  if (isnan(a)) return b;
  if (isnan(b)) return a;
  return a > b ? a : b;
}

/* granite_attention_decode_with_profile, crates/qx-runtime/src/lib.rs:464-552
 * (KvCache::append :382-405 inlined). With cpu_twin the query and key are
 * rotated by cpu_rotate_heads instead of apply_granite_rope: with
 * hierarchical set, that is the V2 CPU twin CpuQ4Cache::attend
 * (crates/qx-runtime-v2/src/lib.rs:4791-4863), whose scores, pinned exp,
 * 256-thread / reduce_simd32 sum and 16 x 32 value chunks are the V1
 * hierarchical variant's, in the same order. */
static int granite_decode_impl(const float* query_in, const float* key_in, const float* value, int position,
                               void* keys, void* values, int key_dtype, int value_dtype, int* length,
                               int max_context, int hierarchical, int cpu_twin, float* output) {
  float query[G_HIDDEN];
  float key[G_KV_HEADS * G_HEAD_DIM];
  memcpy(query, query_in, sizeof(query));
  memcpy(key, key_in, sizeof(key));
  if (position < 0) return QXO_ERR_POSITION;
  if (cpu_twin) {
    /* CpuQ4Reference::step, qx-runtime-v2 lib.rs:4691-4692 */
    if (qxo_cpu_rotate_heads(query, G_HEADS, (uint32_t)position) != QXO_OK ||
        qxo_cpu_rotate_heads(key, G_KV_HEADS, (uint32_t)position) != QXO_OK)
      return QXO_ERR_NONFINITE;
  } else if (qxo_rotate_heads(query, G_HEADS, (uint32_t)position) != QXO_OK ||
             qxo_rotate_heads(key, G_KV_HEADS, (uint32_t)position) != QXO_OK) {
    /* apply_granite_rope :434-442 */
    return QXO_ERR_NONFINITE;
  }
  /* KvCache::append :382-405 */
  if (position != *length) return QXO_ERR_POSITION;
  if (position >= max_context) return QXO_ERR_POSITION;
  const size_t width = G_KV_HEADS * G_HEAD_DIM;
  for (size_t i = 0; i < width; ++i) {
    store_elem(keys, (size_t)position * width + i, key_dtype, key[i]);
    store_elem(values, (size_t)position * width + i, value_dtype, value[i]);
  }
  *length += 1;
  const int len = *length;
  if (len > G_MAX_CONTEXT) return QXO_ERR_INVALID_ARG; /* exponentials[MAX_CONTEXT] */
  if (hierarchical && len > 512) return QXO_ERR_INVALID_ARG; /* partials[..16] */

  float* scores = (float*)malloc(sizeof(float) * (size_t)len);
  float* exponentials = (float*)malloc(sizeof(float) * (size_t)len);
  int status = QXO_OK;
  const int groups = G_HEADS / G_KV_HEADS;
  for (int qh = 0; qh < G_HEADS && status == QXO_OK; ++qh) {
    const int kvh = qh / groups;
    const float* qv = query + qh * G_HEAD_DIM;
    for (int p = 0; p < len; ++p) {
      float score = 0.0f;
      size_t base = ((size_t)p * G_KV_HEADS + kvh) * G_HEAD_DIM;
      for (int j = 0; j < G_HEAD_DIM; ++j)
        score = fmaf(qv[j], load_elem(keys, base + j, key_dtype), score);
      scores[p] = score * G_ATTENTION_MULTIPLIER;
    }
    float max_score = -INFINITY;
    for (int p = 0; p < len; ++p) max_score = rust_max(max_score, scores[p]);
    for (int p = 0; p < len; ++p) {
      if (!qxo_exp_f32(scores[p] - max_score, &exponentials[p])) {
        status = QXO_ERR_NONFINITE;
        break;
      }
    }
    if (status != QXO_OK) break;
    float normalizer;
    if (hierarchical) {
      float threads[256];
      for (int t = 0; t < 256; ++t) {
        float sum = 0.0f;
        for (int p = t; p < len; p += 256) sum += exponentials[p];
        threads[t] = sum;
      }
      float groups8[8];
      for (int g = 0; g < 8; ++g) groups8[g] = qxo_reduce_simd32(threads + g * 32);
      normalizer = 0.0f;
      for (int g = 0; g < 8; ++g) normalizer += groups8[g];
    } else {
      normalizer = 0.0f;
      for (int p = 0; p < len; ++p) normalizer += exponentials[p];
    }
    for (int p = 0; p < len; ++p) scores[p] = exponentials[p] / normalizer;
    float* out = output + qh * G_HEAD_DIM;
    if (hierarchical) {
      const int chunks = (len + 31) / 32;
      for (int d = 0; d < G_HEAD_DIM; ++d) {
        float partials[16] = {0};
        for (int c = 0; c < 16; ++c) {
          int begin = c * 32, end = len < begin + 32 ? len : begin + 32;
          for (int p = begin; p < end; ++p)
            partials[c] = fmaf(scores[p],
                               load_elem(values, ((size_t)p * G_KV_HEADS + kvh) *
                                                         G_HEAD_DIM + d,
                                         value_dtype),
                               partials[c]);
        }
        float sum = 0.0f;
        for (int c = 0; c < chunks; ++c) sum += partials[c];
        out[d] = sum;
      }
    } else {
      for (int d = 0; d < G_HEAD_DIM; ++d) out[d] = 0.0f;
      for (int p = 0; p < len; ++p) {
        float w = scores[p];
        size_t base = ((size_t)p * G_KV_HEADS + kvh) * G_HEAD_DIM;
        for (int d = 0; d < G_HEAD_DIM; ++d)
          out[d] = fmaf(w, load_elem(values, base + d, value_dtype), out[d]);
      }
    }
  }
  free(scores);
  free(exponentials);
  return status;
}

int qxo_granite_attention_decode(const float* query_in, const float* key_in, const float* value, int position,
                                 void* keys, void* values, int key_dtype, int value_dtype, int* length,
                                 int max_context, int hierarchical, float* output) {
  return granite_decode_impl(query_in, key_in, value, position, keys, values, key_dtype, value_dtype, length,
                             max_context, hierarchical, 0, output);
}

typedef struct {
  const float* const* query;
  const float* const* key;
  const float* const* value;
  const int* positions;
  void* const* keys;
  void* const* values;
  int key_dtype, value_dtype;
  int* lengths;
  int max_context, hierarchical;
  float* const* output;
  int* statuses;
} many_ctx;

static void many_body(void* vctx, int u) {
  many_ctx* c = (many_ctx*)vctx;
  c->statuses[u] = qxo_granite_attention_decode(
      c->query[u], c->key[u], c->value[u], c->positions[u], c->keys[u],
      c->values[u], c->key_dtype, c->value_dtype, &c->lengths[u],
      c->max_context, c->hierarchical, c->output[u]);
}

int qxo_granite_attention_decode_many(
    int n_units, const float* const* query, const float* const* key,
    const float* const* value, const int* positions, void* const* keys,
    void* const* values, int key_dtype, int value_dtype, int* lengths,
    int max_context, int hierarchical, float* const* output, int threads,
    int* statuses) {
  int* local = statuses ? statuses : (int*)calloc((size_t)n_units, sizeof(int));
  many_ctx c = {query,   key,         value,       positions, keys,
                values,  key_dtype,   value_dtype, lengths,   max_context,
                hierarchical, output, local};
  qxo_parallel_for(n_units, threads, many_body, &c);
  int worst = QXO_OK;
  for (int u = 0; u < n_units; ++u)
    if (local[u] > worst) worst = local[u];
  if (!statuses) free(local);
  return worst;
}

typedef struct {
  const void* q;
  int in_dtype;
  const void* keys;
  const void* values;
  int kv_dtype;
  float* output;
  int status;
} prefill_ctx;

/* Decode of position p against cache rows 0..p (qx-runtime lib.rs:472-550,
 * plain variant). */
static void prefill_body(void* vctx, int p) {
  prefill_ctx* c = (prefill_ctx*)vctx;
  float query[G_HIDDEN];
  for (int i = 0; i < G_HIDDEN; ++i)
    query[i] = load_elem(c->q, (size_t)p * G_HIDDEN + i, c->in_dtype);
  if (qxo_rotate_heads(query, G_HEADS, (uint32_t)p) != QXO_OK) {
    c->status = QXO_ERR_NONFINITE;
    return;
  }
  const int len = p + 1;
  float* scores = (float*)malloc(sizeof(float) * (size_t)len);
  float* ex = (float*)malloc(sizeof(float) * (size_t)len);
  for (int qh = 0; qh < G_HEADS; ++qh) {
    const int kvh = qh / (G_HEADS / G_KV_HEADS);
    const float* qv = query + qh * G_HEAD_DIM;
    for (int j = 0; j < len; ++j) {
      float score = 0.0f;
      size_t base = ((size_t)j * G_KV_HEADS + kvh) * G_HEAD_DIM;
      for (int d = 0; d < G_HEAD_DIM; ++d)
        score = fmaf(qv[d], load_elem(c->keys, base + d, c->kv_dtype), score);
      scores[j] = score * G_ATTENTION_MULTIPLIER;
    }
    float m = -INFINITY;
    for (int j = 0; j < len; ++j) m = rust_max(m, scores[j]);
    float sum = 0.0f;
    for (int j = 0; j < len; ++j) {
      if (!qxo_exp_f32(scores[j] - m, &ex[j])) c->status = QXO_ERR_NONFINITE;
      sum += ex[j];
    }
    for (int j = 0; j < len; ++j) scores[j] = ex[j] / sum;
    float* out = c->output + (size_t)p * G_HIDDEN + qh * G_HEAD_DIM;
    for (int d = 0; d < G_HEAD_DIM; ++d) out[d] = 0.0f;
    for (int j = 0; j < len; ++j) {
      float w = scores[j];
      size_t base = ((size_t)j * G_KV_HEADS + kvh) * G_HEAD_DIM;
      for (int d = 0; d < G_HEAD_DIM; ++d)
        out[d] = fmaf(w, load_elem(c->values, base + d, c->kv_dtype), out[d]);
    }
  }
  free(scores);
  free(ex);
}

/* Prefill = decode iterated over positions 0..L-1 (the reference prefills a
 * prompt by sequential one-token decode, qx-runtime-v2 lib.rs:4152-4187).
 * All rows are rotated and stored first; the decode at position p then sees
 * exactly rows 0..p, so positions are evaluated in parallel with results
 * identical to the sequential loop. */
int qxo_granite_prefill(const void* q, const void* k, const void* v,
                        int in_dtype, int length, void* keys, void* values,
                        int kv_dtype, float* output, int threads) {
  if (length <= 0 || length > G_MAX_CONTEXT) return QXO_ERR_INVALID_ARG;
  const size_t kw = G_KV_HEADS * G_HEAD_DIM;
  for (int p = 0; p < length; ++p) {
    float key[G_KV_HEADS * G_HEAD_DIM];
    for (size_t i = 0; i < kw; ++i) key[i] = load_elem(k, (size_t)p * kw + i, in_dtype);
    if (qxo_rotate_heads(key, G_KV_HEADS, (uint32_t)p) != QXO_OK) return QXO_ERR_NONFINITE;
    for (size_t i = 0; i < kw; ++i) {
      store_elem(keys, (size_t)p * kw + i, kv_dtype, key[i]);
      store_elem(values, (size_t)p * kw + i, kv_dtype,
                 load_elem(v, (size_t)p * kw + i, in_dtype));
    }
  }
  prefill_ctx c = {q, in_dtype, keys, values, kv_dtype, output, QXO_OK};
  qxo_parallel_for(length, threads, prefill_body, &c);
  return c.status;
}

/* ---- Qwen3, tools/qx-qwen-parity/src/main.rs ---- */
static inline float h2f(uint16_t bits, int dtype) {
  return dtype == QXO_F16 ? qxo_f16_to_f32(bits) : qxo_bf16_to_f32(bits);
}
static inline uint16_t f2h(float f, int dtype) {
  return dtype == QXO_F16 ? qxo_f32_to_f16(f) : qxo_f32_to_bf16(f);
}

/* angle = position * 1e6^(-i/64); (sin, cos) = angle.sin_cos() (:1193-1195). */
void qxo_qwen_rope_table(uint32_t position, float* cosine, float* sine) {
  for (int i = 0; i < 64; ++i) {
    float inv = powf(1000000.0f, -(float)i / 64.0f);
    float angle = (float)position * inv;
    sine[i] = sinf(angle);
    cosine[i] = cosf(angle);
  }
}

/* cpu_qk_norm_rope :1170-1210 (transform :1177-1204). */
static void qwen_transform(const uint16_t* values, int heads, const float* norm,
                           uint32_t position, int dtype, uint16_t* output) {
  float cosine[64], sine[64];
  qxo_qwen_rope_table(position, cosine, sine);
  memcpy(output, values, sizeof(uint16_t) * (size_t)heads * Q_HEAD_DIM);
  for (int head = 0; head < heads; ++head) {
    const int offset = head * Q_HEAD_DIM;
    float sum = 0.0f;
    for (int i = 0; i < Q_HEAD_DIM; ++i) {
      float value = h2f(values[offset + i], dtype);
      float sq = value * value;
      sum = sum + sq;
    }
    float inverse_rms = 1.0f / sqrtf(sum / 128.0f + 1.0e-6f);
    for (int index = 0; index < 64; ++index) {
      float left = h2f(values[offset + index], dtype) * inverse_rms;
      left = left * norm[index];
      float right = h2f(values[offset + 64 + index], dtype) * inverse_rms;
      right = right * norm[64 + index];
      float a = left * cosine[index];
      float b = right * sine[index];
      float c = right * cosine[index];
      float d = left * sine[index];
      output[offset + index] = f2h(a - b, dtype);
      output[offset + 64 + index] = f2h(c + d, dtype);
    }
  }
}

void qxo_qwen_qk_norm_rope(const uint16_t* query, const uint16_t* key,
                           const float* query_norm, const float* key_norm,
                           uint32_t position, int dtype, uint16_t* query_out,
                           uint16_t* key_out) {
  qwen_transform(query, Q_HEADS, query_norm, position, dtype, query_out);
  qwen_transform(key, Q_KV_HEADS, key_norm, position, dtype, key_out);
}

typedef struct {
  const uint16_t* query;
  const uint16_t* key_cache;
  const uint16_t* value_cache;
  int context, dtype;
  float* out_f32;
  uint16_t* out_bits;
} qwen_ctx;

static void qwen_head_body(void* vctx, int qh) {
  qwen_ctx* c = (qwen_ctx*)vctx;
  const float root = sqrtf((float)Q_HEAD_DIM);
  const int context = c->context, dtype = c->dtype;
  const int kh = qh / 8;
  const int qo = qh * Q_HEAD_DIM;
  float* scores = (float*)malloc(sizeof(float) * (size_t)context);
  for (int t = 0; t < context; ++t) {
    size_t ko = ((size_t)t * Q_KV_HEADS + kh) * Q_HEAD_DIM;
    float s = 0.0f;
    for (int k = 0; k < Q_HEAD_DIM; ++k) {
      float prod = h2f(c->query[qo + k], dtype) * h2f(c->key_cache[ko + k], dtype);
      s = s + prod;
    }
    scores[t] = s / root;
  }
  float maximum = -INFINITY;
  for (int t = 0; t < context; ++t) maximum = rust_max(maximum, scores[t]);
  float denominator = 0.0f;
  for (int t = 0; t < context; ++t) {
    scores[t] = expf(scores[t] - maximum); /* now the weights */
    denominator = denominator + scores[t];
  }
  for (int d = 0; d < Q_HEAD_DIM; ++d) {
    float acc = 0.0f;
    for (int t = 0; t < context; ++t) {
      size_t off = ((size_t)t * Q_KV_HEADS + kh) * Q_HEAD_DIM + d;
      float prod = scores[t] * h2f(c->value_cache[off], dtype);
      acc = acc + prod;
    }
    float val = acc / denominator;
    c->out_f32[qo + d] = val;
    if (c->out_bits) c->out_bits[qo + d] = f2h(val, dtype);
  }
  free(scores);
}

/* cpu_gqa_attention :1218-1258. */
void qxo_qwen_gqa_attention(const uint16_t* query, const uint16_t* key_cache,
                            const uint16_t* value_cache, int context, int dtype,
                            float* out_f32, uint16_t* out_bits, int threads) {
  qwen_ctx c = {query, key_cache, value_cache, context, dtype, out_f32, out_bits};
  qxo_parallel_for(Q_HEADS, threads, qwen_head_body, &c);
}

/* ===================================================================== */
/* Attention sub-layer with Q4 projections                               */
/* (qx-runtime-v2 CpuQ4Reference::step, lib.rs:4680-4706)                */
/* ===================================================================== */

/* cpu_rms_norm_simd, qx-runtime-v2 lib.rs:4924-4946. */
int qxo_rms_norm_simd(const float* input, const float* weight, float* out) {
  float threads[256];
  for (int tid = 0; tid < 256; ++tid) {
    float sum = 0.0f;
    for (int index = tid; index < G_HIDDEN; index += 256) sum = fmaf(input[index], input[index], sum);
    threads[tid] = sum;
  }
  float groups[32] = {0};
  for (int group = 0; group < 8; ++group) groups[group] = qxo_reduce_simd32(threads + group * 32);
  const float mean_square = qxo_reduce_simd32(groups) / (float)G_HIDDEN;
  float scale;
  if (!qxo_rsqrt_f32(mean_square + 1e-6f, &scale)) return 0; /* RMS_EPSILON, qx-model lib.rs:24 */
  for (int i = 0; i < G_HIDDEN; ++i) out[i] = input[i] * scale * weight[i];
  return 1;
}

/* QuantizedTensor::quantize (qx-quant lib.rs:313-360) for Q4, group 32:
 * scale = max|x| / 7 rounded to FP16 (1.0 for an all-zero group), code =
 * clamp(round(x / scale), -7, 7) + 7 packed low nibble first (pack_scaled,
 * :1383-1404). */
void qxo_q4_quantize(const float* src, int rows, int cols, uint8_t* codes, uint16_t* scales) {
  const int groups = cols / 32;
  for (int r = 0; r < rows; ++r)
    for (int g = 0; g < groups; ++g) {
      const float* x = src + (size_t)r * cols + g * 32;
      float max_abs = 0.0f;
      for (int i = 0; i < 32; ++i) max_abs = fmaxf(max_abs, fabsf(x[i]));
      const float scale = max_abs == 0.0f ? 1.0f : max_abs / 7.0f;
      const uint16_t bits = qxo_f32_to_f16(scale);
      const float stored = qxo_f16_to_f32(bits);
      scales[(size_t)r * groups + g] = bits;
      uint8_t* dst = codes + ((size_t)r * groups + g) * 16;
      memset(dst, 0, 16);
      for (int i = 0; i < 32; ++i) {
        float q = roundf(x[i] / stored); /* Rust round: half away from zero */
        q = q < -7.0f ? -7.0f : (q > 7.0f ? 7.0f : q);
        const uint8_t code = (uint8_t)((int)q + 7);
        dst[i / 2] |= (uint8_t)((code & 0xF) << ((i & 1) * 4));
      }
    }
}

/* QuantizedTensor::mat_vec_simd32 (qx-quant lib.rs:892-933) with
 * decode_scaled (:1472-1485): value = (code - 7) * scale. */
void qxo_q4_mat_vec_simd32(const uint8_t* codes, const uint16_t* scales, int rows, int cols,
                           const float* input, float* out) {
  const int groups = cols / 32;
  for (int r = 0; r < rows; ++r) {
    float lanes[32] = {0};
    for (int g = 0; g < groups; ++g) {
      const float scale = qxo_f16_to_f32(scales[(size_t)r * groups + g]);
      const uint8_t* packed = codes + ((size_t)r * groups + g) * 16;
      for (int i = 0; i < 32; ++i) {
        const int column = g * 32 + i;
        const uint8_t code = (packed[i / 2] >> ((i & 1) * 4)) & 0xF;
        const float value = (float)((int)code - 7) * scale;
        lanes[column % 32] = fmaf(value, input[column], lanes[column % 32]);
      }
    }
    out[r] = qxo_reduce_simd32(lanes);
  }
}

/* The attention sub-layer of a Granite layer with Q4 weights.
 * cpu_twin = 0: the arithmetic of the V2 GPU stage encode_attention_layer
 *   (crates/qx-runtime-v2/src/lib.rs:6916-6994): rms_norm, the Q4 q/k/v
 *   mat-vecs, RoPE with the fma pair of the Metal kernel qx_v2_rope_kv
 *   (kernels/v2_decode.metal:244-289, the same operations as V1's
 *   rotate_heads), attention as V1's plain granite_attention_decode (valid
 *   to 4096 positions), the Q4 o-projection and the fma residual. This is
 *   what libqxcuda's qxc_attention_layer computes.
 * cpu_twin = 1: CpuQ4Reference::step's attention part (lib.rs:4686-4706)
 *   exactly: cpu_rotate_heads (no fma) and CpuQ4Cache::attend (hierarchical
 *   sums, at most 512 positions; QXO_ERR_INVALID_ARG beyond, where the
 *   reference's partials slice panics). */
int qxo_granite_attention_layer(const float* hidden, const float* input_norm,
                                const uint8_t* q_codes, const uint16_t* q_scales,
                                const uint8_t* k_codes, const uint16_t* k_scales,
                                const uint8_t* v_codes, const uint16_t* v_scales,
                                const uint8_t* o_codes, const uint16_t* o_scales,
                                int position, float* keys, float* values, int* length,
                                int capacity, int cpu_twin, float* out, float* attention_out) {
  float normalized[G_HIDDEN], q[G_HIDDEN], k[G_KV_HEADS * G_HEAD_DIM], v[G_KV_HEADS * G_HEAD_DIM];
  float attention[G_HIDDEN], projection[G_HIDDEN];
  if (!qxo_rms_norm_simd(hidden, input_norm, normalized)) return QXO_ERR_NONFINITE;
  qxo_q4_mat_vec_simd32(q_codes, q_scales, G_HIDDEN, G_HIDDEN, normalized, q);
  qxo_q4_mat_vec_simd32(k_codes, k_scales, G_KV_HEADS * G_HEAD_DIM, G_HIDDEN, normalized, k);
  qxo_q4_mat_vec_simd32(v_codes, v_scales, G_KV_HEADS * G_HEAD_DIM, G_HIDDEN, normalized, v);
  const int st = granite_decode_impl(q, k, v, position, keys, values, QXO_F32, QXO_F32, length, capacity,
                                     cpu_twin ? 1 : 0, cpu_twin ? 1 : 0, attention);
  if (st != QXO_OK) return st;
  if (attention_out) memcpy(attention_out, attention, sizeof(attention));
  qxo_q4_mat_vec_simd32(o_codes, o_scales, G_HIDDEN, G_HIDDEN, attention, projection);
  for (int i = 0; i < G_HIDDEN; ++i) out[i] = fmaf(0.22f, projection[i], hidden[i]); /* RESIDUAL_MULTIPLIER */
  return QXO_OK;
}

/* ===================================================================== */
/* KV-slot commitments: BLAKE3 and qx-commit's chunk trees               */
/* ===================================================================== */

/* BLAKE3 as published (the reference links the blake3 crate 1.8.7). Only
 * single-chunk inputs (<= 1024 bytes) occur on this path. */
static const uint32_t B3_IV[8] = {0x6A09E667u, 0xBB67AE85u, 0x3C6EF372u, 0xA54FF53Au,
                                  0x510E527Fu, 0x9B05688Cu, 0x1F83D9ABu, 0x5BE0CD19u};
static const uint8_t B3_PERM[16] = {2, 6, 3, 10, 7, 0, 4, 13, 1, 11, 12, 5, 9, 14, 15, 8};

static uint32_t b3_rotr(uint32_t v, int n) { return (v >> n) | (v << (32 - n)); }

static void b3_g(uint32_t* s, int a, int b, int c, int d, uint32_t x, uint32_t y) {
  s[a] = s[a] + s[b] + x;
  s[d] = b3_rotr(s[d] ^ s[a], 16);
  s[c] = s[c] + s[d];
  s[b] = b3_rotr(s[b] ^ s[c], 12);
  s[a] = s[a] + s[b] + y;
  s[d] = b3_rotr(s[d] ^ s[a], 8);
  s[c] = s[c] + s[d];
  s[b] = b3_rotr(s[b] ^ s[c], 7);
}

static void b3_compress(const uint32_t cv[8], const uint8_t block[64], uint32_t block_len, uint32_t flags,
                        uint32_t out[8]) {
  uint32_t m[16], s[16], t[16];
  for (int i = 0; i < 16; ++i)
    m[i] = (uint32_t)block[4 * i] | ((uint32_t)block[4 * i + 1] << 8) | ((uint32_t)block[4 * i + 2] << 16) |
           ((uint32_t)block[4 * i + 3] << 24);
  for (int i = 0; i < 8; ++i) s[i] = cv[i];
  for (int i = 0; i < 4; ++i) s[8 + i] = B3_IV[i];
  s[12] = 0; /* chunk counter: one chunk */
  s[13] = 0;
  s[14] = block_len;
  s[15] = flags;
  for (int round = 0; round < 7; ++round) {
    b3_g(s, 0, 4, 8, 12, m[0], m[1]);
    b3_g(s, 1, 5, 9, 13, m[2], m[3]);
    b3_g(s, 2, 6, 10, 14, m[4], m[5]);
    b3_g(s, 3, 7, 11, 15, m[6], m[7]);
    b3_g(s, 0, 5, 10, 15, m[8], m[9]);
    b3_g(s, 1, 6, 11, 12, m[10], m[11]);
    b3_g(s, 2, 7, 8, 13, m[12], m[13]);
    b3_g(s, 3, 4, 9, 14, m[14], m[15]);
    for (int i = 0; i < 16; ++i) t[i] = m[B3_PERM[i]];
    memcpy(m, t, sizeof(m));
  }
  for (int i = 0; i < 8; ++i) out[i] = s[i] ^ s[i + 8];
}

int qxo_blake3_single_chunk(const uint8_t* input, size_t len, uint8_t out[32]) {
  if (len > 1024) return 0;
  uint32_t cv[8];
  memcpy(cv, B3_IV, sizeof(cv));
  const size_t blocks = len == 0 ? 1 : (len + 63) / 64;
  for (size_t b = 0; b < blocks; ++b) {
    uint8_t block[64] = {0};
    const size_t n = b + 1 < blocks ? 64 : len - b * 64;
    memcpy(block, input + b * 64, n);
    uint32_t flags = (b == 0 ? 1u : 0u) | (b + 1 == blocks ? 2u | 8u : 0u); /* CHUNK_START, CHUNK_END|ROOT */
    uint32_t next[8];
    b3_compress(cv, block, (uint32_t)n, flags, next);
    memcpy(cv, next, sizeof(cv));
  }
  for (int i = 0; i < 8; ++i) {
    out[4 * i] = (uint8_t)cv[i];
    out[4 * i + 1] = (uint8_t)(cv[i] >> 8);
    out[4 * i + 2] = (uint8_t)(cv[i] >> 16);
    out[4 * i + 3] = (uint8_t)(cv[i] >> 24);
  }
  return 1;
}

/* hash_domain (qx-commit hash.rs): domain, then per field u64 LE length and
 * the field's bytes. */
static int b3_domain(const char* domain, const uint8_t* const* fields, const size_t* lens, int n, uint8_t out[32]) {
  uint8_t buf[1024];
  size_t at = strlen(domain);
  memcpy(buf, domain, at);
  for (int f = 0; f < n; ++f) {
    if (at + 8 + lens[f] > sizeof(buf)) return 0;
    for (int i = 0; i < 8; ++i) buf[at + i] = (uint8_t)((uint64_t)lens[f] >> (8 * i));
    at += 8;
    memcpy(buf + at, fields[f], lens[f]);
    at += lens[f];
  }
  return qxo_blake3_single_chunk(buf, at, out);
}

int qxo_chunk_tree_hash(const uint8_t* bytes, size_t len, const char* leaf_domain, const char* tree_domain,
                        uint8_t out[32]) {
  if (len == 0) return 0;
  const size_t leaves = (len + 255) / 256;
  size_t cap = 1;
  while (cap < leaves) cap <<= 1;
  uint8_t (*nodes)[32] = malloc(cap * 32);
  if (!nodes) return 0;
  for (size_t i = 0; i < leaves; ++i) {
    const uint8_t index[4] = {(uint8_t)i, (uint8_t)(i >> 8), (uint8_t)(i >> 16), (uint8_t)(i >> 24)};
    const size_t n = i + 1 < leaves ? 256 : len - i * 256;
    const uint8_t* fields[2] = {index, bytes + i * 256};
    const size_t lens[2] = {4, n};
    b3_domain(leaf_domain, fields, lens, 2, nodes[i]);
  }
  if (cap > leaves) {
    uint8_t empty[32];
    const uint8_t* fields[1] = {(const uint8_t*)tree_domain};
    const size_t lens[1] = {strlen(tree_domain)};
    b3_domain("QX:MERKLE:EMPTY:V1", fields, lens, 1, empty);
    for (size_t i = leaves; i < cap; ++i) memcpy(nodes[i], empty, 32);
  }
  for (size_t width = cap; width > 1; width /= 2)
    for (size_t i = 0; i < width / 2; ++i) {
      uint8_t pair[64];
      memcpy(pair, nodes[2 * i], 32);
      memcpy(pair + 32, nodes[2 * i + 1], 32);
      qxo_blake3_single_chunk(pair, 64, nodes[i]);
    }
  memcpy(out, nodes[0], 32);
  free(nodes);
  return 1;
}

int qxo_kv_leaf_hash(uint16_t layer, uint32_t token, const uint8_t* key_bytes, size_t key_len,
                     const uint8_t* value_bytes, size_t value_len, uint8_t out[32]) {
  uint8_t key_root[32], value_root[32];
  if (!qxo_chunk_tree_hash(key_bytes, key_len, "QX:KV:KEY:CHUNK:V1", "QX:KV:KEY:TREE:V1", key_root)) return 0;
  if (!qxo_chunk_tree_hash(value_bytes, value_len, "QX:KV:VALUE:CHUNK:V1", "QX:KV:VALUE:TREE:V1", value_root))
    return 0;
  const uint8_t l[2] = {(uint8_t)layer, (uint8_t)(layer >> 8)};
  const uint8_t t[4] = {(uint8_t)token, (uint8_t)(token >> 8), (uint8_t)(token >> 16), (uint8_t)(token >> 24)};
  const uint8_t* fields[4] = {l, t, key_root, value_root};
  const size_t lens[4] = {2, 4, 32, 32};
  return b3_domain("QX:KV:V1", fields, lens, 4, out);
}
