/*
 * mrml_oracle.c — CPU restatement of the MRML MoE FFN path (test
 * infrastructure; see mrml_oracle.h).  Build: oracle/Makefile.
 *
 * Reference files cited below are paths inside mitchellrenouf/QT_llama.cpp,
 * crate crates/mrml-tensor unless stated otherwise.
 */
#include "mrml_oracle.h"

#include <math.h>
#include <pthread.h>
#include <stdlib.h>
#include <string.h>

#if defined(__FAST_MATH__)
#error "the oracle must be built without fast-math"
#endif

/* ---------------------------------------------------------------- f16 --- */

float oracle_f16_to_f32(uint16_t h) { /* quant.rs:47-77 */
  uint32_t sign = (h >> 15) & 1u, exp = (h >> 10) & 0x1fu, mant = h & 0x3ffu;
  uint32_t bits;
  if (exp == 0) {
    if (mant == 0) {
      bits = sign << 31;
    } else {
      uint32_t m = mant, e = 0;
      while ((m & 0x400u) == 0) {
        m <<= 1;
        e += 1;
      }
      m &= 0x3ffu;
      bits = (sign << 31) | ((127u - 15u + 1u - e) << 23) | (m << 13);
    }
  } else if (exp == 31) {
    bits = (sign << 31) | (0xffu << 23) | (mant << 13);
  } else {
    bits = (sign << 31) | ((exp + 112u) << 23) | (mant << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

uint16_t oracle_f32_to_f16(float f) { /* quant.rs:81-104 */
  uint32_t bits;
  memcpy(&bits, &f, 4);
  uint16_t sign = (uint16_t)((bits >> 31) & 1u);
  int32_t exp = (int32_t)((bits >> 23) & 0xffu);
  uint32_t mant = bits & 0x7fffffu;
  if (exp == 255) return (uint16_t)((sign << 15) | (mant == 0 ? 0x7c00u : 0x7e00u));
  int32_t exp16 = exp - 127 + 15;
  if (exp16 >= 31) return (uint16_t)((sign << 15) | 0x7c00u);
  if (exp16 <= 0) return 0; /* flushed to +0, sign dropped, as in the reference */
  return (uint16_t)((sign << 15) | ((uint32_t)exp16 << 10) | (mant >> 13));
}

static inline uint16_t rd16(const uint8_t *p) { return (uint16_t)(p[0] | (p[1] << 8)); }

/* -------------------------------------------------------- quantisers --- */

/* Rust's saturating float-to-int `as i32`: NaN -> 0, clamped to the range. */
static inline int sat_i32(float v) {
  if (v != v) return 0;
  if (v >= 2147483647.0f) return 2147483647;
  if (v <= -2147483648.0f) return (-2147483647 - 1);
  return (int)v;
}

void oracle_quantize_q8_0(const float *src, size_t n, uint8_t *dst) { /* quant.rs:193-228 */
  for (size_t b = 0; b < n / 32; b++) {
    const float *s = src + b * 32;
    uint8_t *o = dst + b * 34;
    float max_val = 0.0f;
    for (int i = 0; i < 32; i++) {
      float a = fabsf(s[i]);
      if (a > max_val) max_val = a;
    }
    float scale = max_val / 127.0f;
    uint16_t d = oracle_f32_to_f16(scale);
    float id = scale != 0.0f ? 1.0f / scale : 0.0f;
    o[0] = (uint8_t)(d & 0xff);
    o[1] = (uint8_t)(d >> 8);
    for (int i = 0; i < 32; i++) {
      float v = roundf(s[i] * id);
      if (v != v) v = 0.0f; /* Rust `as i8` maps NaN to 0 */
      if (v < -128.0f) v = -128.0f;
      if (v > 127.0f) v = 127.0f;
      o[2 + i] = (uint8_t)(int8_t)v;
    }
  }
}

void oracle_quantize_q4_0(const float *src, size_t n, uint8_t *dst) { /* quant.rs:372-389 */
  for (size_t b = 0; b < n / 32; b++) {
    const float *v = src + b * 32;
    uint8_t *o = dst + b * 18;
    float max_abs = 0.0f;
    for (int i = 0; i < 32; i++) max_abs = fmaxf(max_abs, fabsf(v[i])); /* f32::max */
    float scale = max_abs > 0.0f ? max_abs / 8.0f : 0.0f;
    uint16_t d = oracle_f32_to_f16(scale);
    o[0] = (uint8_t)(d & 0xff);
    o[1] = (uint8_t)(d >> 8);
    float inverse = scale > 0.0f ? 1.0f / scale : 0.0f;
    for (int i = 0; i < 16; i++) {
      /* `round(x) as i32` saturates in Rust; values here are bounded by 8. */
      int lo = sat_i32(roundf(v[i] * inverse));
      int hi = sat_i32(roundf(v[i + 16] * inverse));
      lo = (lo < -8 ? -8 : lo > 7 ? 7 : lo) + 8;
      hi = (hi < -8 ? -8 : hi > 7 ? 7 : hi) + 8;
      o[2 + i] = (uint8_t)(lo | (hi << 4));
    }
  }
}

void oracle_dequantize_q4_0(const uint8_t *src, size_t n_blocks, float *out) { /* quant.rs:135-163 */
  for (size_t b = 0; b < n_blocks; b++) {
    const uint8_t *blk = src + b * 18;
    float d = oracle_f16_to_f32(rd16(blk));
    for (int i = 0; i < 16; i++) {
      uint8_t byte = blk[2 + i];
      out[b * 32 + i] = (float)((int)(byte & 0x0f) - 8) * d;
      out[b * 32 + i + 16] = (float)((int)(byte >> 4) - 8) * d;
    }
  }
}

void oracle_dequantize_q8_0(const uint8_t *src, size_t n_blocks, float *out) { /* quant.rs:166-190 */
  for (size_t b = 0; b < n_blocks; b++) {
    const uint8_t *blk = src + b * 34;
    float d = oracle_f16_to_f32(rd16(blk));
    for (int i = 0; i < 32; i++) out[b * 32 + i] = (float)(int8_t)blk[2 + i] * d;
  }
}

/* -------------------------------------------------------- block dots --- */

float oracle_vec_dot_q4_0_q8_0(const uint8_t *w, const uint8_t *a, int n) { /* quant.rs:335-369 */
  float sum = 0.0f;
  for (int b = 0; b < n / 32; b++) {
    const uint8_t *wb = w + (size_t)b * 18;
    const uint8_t *ab = a + (size_t)b * 34;
    float d_w = oracle_f16_to_f32(rd16(wb));
    float d_a = oracle_f16_to_f32(rd16(ab));
    int32_t block_sum = 0;
    for (int i = 0; i < 16; i++) {
      int32_t q0 = (int32_t)(wb[2 + i] & 0x0f) - 8;
      int32_t q1 = (int32_t)(wb[2 + i] >> 4) - 8;
      block_sum += q0 * (int32_t)(int8_t)ab[2 + i] + q1 * (int32_t)(int8_t)ab[2 + i + 16];
    }
    float s = d_w * d_a;
    sum += (float)block_sum * s;
  }
  return sum;
}

float oracle_vec_dot_q8_0_q8_0(const uint8_t *w, const uint8_t *a, int n) { /* quant.rs:564-577 */
  float sum = 0.0f;
  for (int b = 0; b < n / 32; b++) {
    const uint8_t *wb = w + (size_t)b * 34;
    const uint8_t *ab = a + (size_t)b * 34;
    float dx = oracle_f16_to_f32(rd16(wb));
    float dy = oracle_f16_to_f32(rd16(ab));
    int32_t block_sum = 0;
    for (int i = 0; i < 32; i++) block_sum += (int32_t)(int8_t)wb[2 + i] * (int32_t)(int8_t)ab[2 + i];
    float s = dx * dy;
    sum += (float)block_sum * s;
  }
  return sum;
}

/* ------------------------------------------------------- worker pool --- */
/* A persistent pool, like parallel.rs:42-71: workers wait for a range job;
 * the caller splits [0, len) into min(workers, ceil(len/64)) equal chunks
 * (parallel.rs:73-116) and waits for all of them. */

typedef void (*range_fn)(void *ctx, int start, int end);

typedef struct {
  pthread_mutex_t mu;
  pthread_cond_t cv_work, cv_done;
  int workers;
  pthread_t *threads;
  /* current job */
  range_fn fn;
  void *ctx;
  int len, chunk, next, pending;
  unsigned long generation;
} pool_t;

static pool_t g_pool;
static int g_pool_ready = 0;
static pthread_mutex_t g_pool_init = PTHREAD_MUTEX_INITIALIZER;

static void *pool_worker(void *arg) {
  (void)arg;
  pthread_mutex_lock(&g_pool.mu);
  for (;;) {
    while (g_pool.fn == NULL || g_pool.next >= g_pool.len) pthread_cond_wait(&g_pool.cv_work, &g_pool.mu);
    int start = g_pool.next;
    int end = start + g_pool.chunk < g_pool.len ? start + g_pool.chunk : g_pool.len;
    g_pool.next = end;
    range_fn fn = g_pool.fn;
    void *ctx = g_pool.ctx;
    pthread_mutex_unlock(&g_pool.mu);
    fn(ctx, start, end);
    pthread_mutex_lock(&g_pool.mu);
    if (--g_pool.pending == 0) {
      g_pool.fn = NULL;
      pthread_cond_signal(&g_pool.cv_done);
    }
  }
  return NULL;
}

static void pool_ensure(int workers) {
  pthread_mutex_lock(&g_pool_init);
  if (!g_pool_ready || g_pool.workers < workers) {
    if (!g_pool_ready) {
      pthread_mutex_init(&g_pool.mu, NULL);
      pthread_cond_init(&g_pool.cv_work, NULL);
      pthread_cond_init(&g_pool.cv_done, NULL);
      g_pool.workers = 0;
      g_pool.threads = NULL;
      g_pool_ready = 1;
    }
    g_pool.threads = (pthread_t *)realloc(g_pool.threads, sizeof(pthread_t) * (size_t)workers);
    for (int i = g_pool.workers; i < workers; i++) pthread_create(&g_pool.threads[i], NULL, pool_worker, NULL);
    g_pool.workers = workers;
  }
  pthread_mutex_unlock(&g_pool_init);
}

static void for_each_range(int n_threads, int len, int minimum_chunk, range_fn fn, void *ctx) {
  if (n_threads <= 1 || len <= minimum_chunk) {
    fn(ctx, 0, len);
    return;
  }
  pool_ensure(n_threads);
  int jobs = (len + minimum_chunk - 1) / minimum_chunk;
  if (jobs > n_threads) jobs = n_threads;
  int chunk = (len + jobs - 1) / jobs;
  pthread_mutex_lock(&g_pool.mu);
  g_pool.ctx = ctx;
  g_pool.len = len;
  g_pool.chunk = chunk;
  g_pool.next = 0;
  g_pool.pending = (len + chunk - 1) / chunk;
  g_pool.fn = fn;
  pthread_cond_broadcast(&g_pool.cv_work);
  while (g_pool.fn != NULL) pthread_cond_wait(&g_pool.cv_done, &g_pool.mu);
  pthread_mutex_unlock(&g_pool.mu);
}

/* ------------------------------------------------------------ GEMV ---- */

typedef struct {
  int wtype;
  const uint8_t *w, *x_q8;
  float *y;
  int n_cols;
  size_t row_bytes;
} gemv_ctx;

static void gemv_rows(void *p, int start, int end) {
  gemv_ctx *c = (gemv_ctx *)p;
  for (int r = start; r < end; r++) {
    const uint8_t *row = c->w + (size_t)r * c->row_bytes;
    c->y[r] = c->wtype == ORACLE_Q4_0 ? oracle_vec_dot_q4_0_q8_0(row, c->x_q8, c->n_cols)
                                      : oracle_vec_dot_q8_0_q8_0(row, c->x_q8, c->n_cols);
  }
}

static size_t block_bytes(int wtype) { return wtype == ORACLE_Q4_0 ? 18 : 34; }

static void mat_vec_q8_threads(int wtype, const uint8_t *w, const uint8_t *x_q8, float *y, int n_rows,
                               int n_cols, int n_threads) { /* ops.rs:221-260 */
  gemv_ctx c = {wtype, w, x_q8, y, n_cols, (size_t)(n_cols / 32) * block_bytes(wtype)};
  if (n_rows <= 64)
    gemv_rows(&c, 0, n_rows);
  else
    for_each_range(n_threads, n_rows, 64, gemv_rows, &c);
}

void oracle_mat_vec_q8(int wtype, const uint8_t *w, const uint8_t *x_q8, float *y, int n_rows, int n_cols) {
  mat_vec_q8_threads(wtype, w, x_q8, y, n_rows, n_cols, 1);
}

void oracle_mat_vec_f32(int wtype, const uint8_t *w, const float *x, float *y, int n_rows, int n_cols) {
  uint8_t *xq = (uint8_t *)malloc((size_t)(n_cols / 32) * 34); /* ops.rs:175-177 */
  oracle_quantize_q8_0(x, (size_t)n_cols, xq);
  oracle_mat_vec_q8(wtype, w, xq, y, n_rows, n_cols);
  free(xq);
}

/* ------------------------------------------------------ elementwise --- */

float oracle_gelu_approx(float x) { /* ops.rs:101-104, left-to-right evaluation */
  const float sqrt_2_over_pi = 0.7978845608f;
  float cube = 0.044715f * x * x * x;
  float inner = sqrt_2_over_pi * (x + cube);
  return 0.5f * x * (1.0f + tanhf(inner));
}

void oracle_geglu(const float *gate, const float *up, float *out, int n) { /* ops.rs:107-114 */
  for (int i = 0; i < n; i++) out[i] = oracle_gelu_approx(gate[i]) * up[i];
}

void oracle_rms_norm(const float *x, const float *weight, float eps, float *out, int n) { /* ops.rs:24-49 */
  float sum_sq = 0.0f;
  for (int i = 0; i < n; i++) sum_sq += x[i] * x[i];
  float mean_sq = sum_sq / (float)n;
  float scale = 1.0f / sqrtf(mean_sq + eps);
  for (int i = 0; i < n; i++) out[i] = weight ? x[i] * scale * weight[i] : x[i] * scale;
}

/* ------------------------------------------------------ FFN prologue --- */

void oracle_ffn_prologue(const float *hidden, const float *attn, const float *post_attn_norm,
                         const float *ffn_norm, const float *pre_ffw_norm_2, const float *router_scale,
                         float *attn_res, float *x_shared, float *x_moe, float *router_x, int H, int T, float eps) {
  float *tmp = (float *)malloc(sizeof(float) * (size_t)H);
  float *res = (float *)malloc(sizeof(float) * (size_t)H);
  float inv_sqrt_dim = 1.0f / sqrtf((float)H); /* model.rs:1776 */
  for (int t = 0; t < T; t++) {
    size_t o = (size_t)t * H;
    if (attn) { /* model.rs:1730-1739 */
      oracle_rms_norm(attn + o, post_attn_norm, eps, tmp, H);
      for (int i = 0; i < H; i++) res[i] = hidden[o + i] + tmp[i];
    } else {
      for (int i = 0; i < H; i++) res[i] = hidden[o + i];
    }
    if (attn_res)
      for (int i = 0; i < H; i++) attn_res[o + i] = res[i];
    if (x_shared) oracle_rms_norm(res, ffn_norm, eps, x_shared + o, H); /* model.rs:1751-1753 */
    if (x_moe) oracle_rms_norm(res, pre_ffw_norm_2, eps, x_moe + o, H); /* model.rs:1760-1767 */
    if (router_x) {                                                     /* model.rs:1774-1784 */
      oracle_rms_norm(res, NULL, eps, tmp, H);
      for (int i = 0; i < H; i++) {
        float scale = router_scale ? router_scale[i] : 1.0f;
        router_x[o + i] = tmp[i] * inv_sqrt_dim * scale;
      }
    }
  }
  free(tmp);
  free(res);
}

void oracle_ffn_epilogue(const float *attn_res, const float *mlp_raw, const float *moe_raw,
                         const float *post_ffw_norm_1, const float *post_ffw_norm_2, const float *post_ffw_norm,
                         float out_scale, float *hidden, int H, int T, float eps) {
  float *zeros = (float *)calloc((size_t)H, sizeof(float));
  float *mlp_out = (float *)malloc(sizeof(float) * (size_t)H);
  float *moe_out = (float *)malloc(sizeof(float) * (size_t)H);
  float *comb = (float *)malloc(sizeof(float) * (size_t)H);
  float *normed = (float *)malloc(sizeof(float) * (size_t)H);
  for (int t = 0; t < T; t++) {
    size_t o = (size_t)t * H;
    oracle_rms_norm(mlp_raw ? mlp_raw + o : zeros, post_ffw_norm_1, eps, mlp_out, H); /* model.rs:2176-2177 */
    oracle_rms_norm(moe_raw + o, post_ffw_norm_2, eps, moe_out, H);                  /* model.rs:2179-2180 */
    for (int i = 0; i < H; i++) comb[i] = mlp_out[i] + moe_out[i];                   /* model.rs:2182-2185 */
    oracle_rms_norm(comb, post_ffw_norm, eps, normed, H);                           /* model.rs:2187-2193 */
    for (int i = 0; i < H; i++) hidden[o + i] = (attn_res[o + i] + normed[i]) * out_scale; /* model.rs:2194-2196 */
  }
  free(zeros);
  free(mlp_out);
  free(moe_out);
  free(comb);
  free(normed);
}

/* ----------------------------------------------------------- router --- */

typedef struct {
  float v;
  int id;
} scored;

static int scored_desc(const void *pa, const void *pb) {
  const scored *a = (const scored *)pa, *b = (const scored *)pb;
  if (a->v > b->v) return -1;
  if (a->v < b->v) return 1;
  return a->id - b->id; /* exact ties: lower expert id first */
}

static void topk_softmax(const float *logits, int32_t *ids, float *probs, int E, int K, scored *tmp) {
  for (int e = 0; e < E; e++) {
    tmp[e].v = logits[e];
    tmp[e].id = e;
  }
  qsort(tmp, (size_t)E, sizeof(scored), scored_desc); /* model.rs:1816-1818 */
  float max_l = tmp[0].v;
  float sum_exp = 0.0f;
  for (int k = 0; k < K; k++) { /* model.rs:1819-1826 */
    ids[k] = tmp[k].id;
    float p = expf(tmp[k].v - max_l);
    probs[k] = p;
    sum_exp += p;
  }
  float denom = sum_exp > 1e-6f ? sum_exp : 1e-6f; /* f32::max(sum, 1e-6) */
  for (int k = 0; k < K; k++) probs[k] /= denom; /* model.rs:1827-1829 */
}

void oracle_moe_router(const float *W, const float *x, float *logits, int32_t *ids, float *probs, int H, int E,
                       int K, int T) {
  scored *tmp = (scored *)malloc(sizeof(scored) * (size_t)E);
  for (int t = 0; t < T; t++) {
    const float *xt = x + (size_t)t * H;
    float *lt = logits + (size_t)t * E;
    for (int e = 0; e < E; e++) { /* model.rs:1804-1814 */
      const float *we = W + (size_t)e * H;
      float dot = 0.0f;
      for (int i = 0; i < H; i++) dot += xt[i] * we[i];
      lt[e] = dot;
    }
    topk_softmax(lt, ids + (size_t)t * K, probs + (size_t)t * K, E, K, tmp);
  }
  free(tmp);
}

void oracle_moe_route_from_logits(const float *logits, int32_t *ids, float *probs, int E, int K, int T) {
  scored *tmp = (scored *)malloc(sizeof(scored) * (size_t)E);
  for (int t = 0; t < T; t++)
    topk_softmax(logits + (size_t)t * E, ids + (size_t)t * K, probs + (size_t)t * K, E, K, tmp);
  free(tmp);
}

/* ---------------------------------------------------------- experts --- */

static void expert_forward(int wtype, const uint8_t *gate_up, const uint8_t *down, int e, const uint8_t *x_q8,
                           int H, int I, float *gate, float *up, float *act, uint8_t *act_q8, float *down_out,
                           int n_threads) {
  size_t bb = block_bytes(wtype);
  size_t gu_row = (size_t)(H / 32) * bb, dn_row = (size_t)(I / 32) * bb;
  const uint8_t *g = gate_up + (size_t)e * 2 * I * gu_row; /* model.rs:2123-2136 */
  const uint8_t *u = g + (size_t)I * gu_row;
  const uint8_t *d = down + (size_t)e * H * dn_row;
  mat_vec_q8_threads(wtype, g, x_q8, gate, I, H, n_threads); /* model.rs:2142-2148 */
  mat_vec_q8_threads(wtype, u, x_q8, up, I, H, n_threads);   /* model.rs:2149 */
  oracle_geglu(gate, up, act, I);                             /* model.rs:2151-2152 */
  oracle_quantize_q8_0(act, (size_t)I, act_q8);               /* ops.rs:175-177 via model.rs:2155 */
  mat_vec_q8_threads(wtype, d, act_q8, down_out, H, I, n_threads);
}

void oracle_moe_expert_trace(int wtype, const uint8_t *gate_up, const uint8_t *down, int expert, const float *x,
                             int H, int I, float *gate, float *up, float *act, float *down_out) {
  uint8_t *xq = (uint8_t *)malloc((size_t)(H / 32) * 34);
  uint8_t *aq = (uint8_t *)malloc((size_t)(I / 32) * 34);
  oracle_quantize_q8_0(x, (size_t)H, xq);
  expert_forward(wtype, gate_up, down, expert, xq, H, I, gate, up, act, aq, down_out, 1);
  free(xq);
  free(aq);
}

void oracle_moe_experts(int wtype, const uint8_t *gate_up, const uint8_t *down, const int32_t *ids,
                        const float *probs, const float *down_scale, const float *x, float *out, int H, int I,
                        int E, int K, int T, int n_threads) {
  (void)E;
  uint8_t *xq = (uint8_t *)malloc((size_t)(H / 32) * 34);
  uint8_t *aq = (uint8_t *)malloc((size_t)(I / 32) * 34);
  float *gate = (float *)malloc(sizeof(float) * (size_t)I);
  float *up = (float *)malloc(sizeof(float) * (size_t)I);
  float *act = (float *)malloc(sizeof(float) * (size_t)I);
  float *dn = (float *)malloc(sizeof(float) * (size_t)H);
  for (int t = 0; t < T; t++) {
    float *o = out + (size_t)t * H;
    for (int i = 0; i < H; i++) o[i] = 0.0f; /* moe_raw starts at zero, model.rs:1839-1845 */
    oracle_quantize_q8_0(x + (size_t)t * H, (size_t)H, xq); /* model.rs:2114-2115 */
    for (int k = 0; k < K; k++) {
      float alpha = probs[(size_t)t * K + k];
      if (alpha <= 0.0001f) continue; /* model.rs:2118-2121 */
      int e = ids[(size_t)t * K + k];
      expert_forward(wtype, gate_up, down, e, xq, H, I, gate, up, act, aq, dn, n_threads);
      float scale = down_scale ? down_scale[e] : 1.0f; /* model.rs:2157-2161 */
      for (int i = 0; i < H; i++) o[i] += alpha * dn[i] * scale; /* model.rs:2163-2165 */
    }
  }
  free(xq);
  free(aq);
  free(gate);
  free(up);
  free(act);
  free(dn);
}
