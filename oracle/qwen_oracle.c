/*
 * qwen_oracle.c -- CPU restatement of the reference's quantized Qwen2.5-1.5B decoder-layer host path.
 *
 * TEST INFRASTRUCTURE ONLY. This file is the checker for the CUDA product path: only tests/,
 * __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference legs load it. No product
 * code links, loads or calls it, and the product never falls back to it.
 *
 * Parity pin: with wbits == 4 every entry point below is checked bit-for-bit against the reference's
 * own host libraries (libqwen_decode_stub.so / libqwen_prefill_stub.so built from the reference
 * sources by oracle/Makefile into oracle/_ref/) on seeded dense inputs and on the reference's sparse
 * known-answer cases; tests/golden/ holds the digests that pin it (tests/golden/make_golden.py).
 *
 * What it restates (reference paths are relative to the reference project root):
 *   - int4 nibble decode / per-channel dequant:  hls/decode_only/qwen_decode_attention_kernel.cpp:44-60
 *   - serial projection (`project_tiled`):        hls/decode_only/qwen_decode_attention_kernel.cpp:62-98,
 *                                                 hls/decode_only/qwen_decode_mlp_kernel.cpp:44-77,
 *                                                 hls/prefill_only/qwen_prefill_attention_kernel.cpp:163-202,
 *                                                 hls/prefill_only/qwen_prefill_mlp_kernel.cpp:217-254
 *   - decode RMSNorm (double):                    hls/decode_only/qwen_decode_attention_kernel.cpp:13-27
 *   - decode RoPE (double pow/cos/sin):           hls/decode_only/qwen_decode_attention_kernel.cpp:29-42
 *   - decode KV append + 2-pass softmax context:  hls/decode_only/qwen_decode_attention_kernel.cpp:100-162
 *   - decode attention orchestration:             hls/decode_only/qwen_decode_attention_kernel.cpp:168-218
 *   - decode MLP (expf SiLU, `+a`):               hls/decode_only/qwen_decode_mlp_kernel.cpp:79-122
 *   - prefill approx_sqrt/wrap/sincos/exp:        hls/prefill_only/qwen_prefill_attention_kernel.cpp:47-110
 *   - prefill RMSNorm (fp32 + approx_sqrt):       hls/prefill_only/qwen_prefill_attention_kernel.cpp:112-126
 *   - prefill RoPE (serial inv_freq product):     hls/prefill_only/qwen_prefill_attention_kernel.cpp:128-143
 *   - prefill causal 2-pass context:              hls/prefill_only/qwen_prefill_attention_kernel.cpp:204-289
 *   - prefill attention orchestration:            hls/prefill_only/qwen_prefill_attention_kernel.cpp:2232-2367
 *   - prefill MLP (approx_exp SiLU, `+a`):        hls/prefill_only/qwen_prefill_mlp_kernel.cpp:256-337
 *   - caller-side bf16 RNE rounding:              verification/reference_wrapper_backend.py:40-46
 *   - caller-side int4 per-channel quantizer:     verification/real_host_top_backend.py:31-41
 *
 * Extensions beyond the reference (same arithmetic, labelled):
 *   - wbits == 8: int8 codes (one byte per weight, row-major) in place of packed nibbles; every other
 *     operation is unchanged. This is the W8 track's oracle; the reference has no int8 path.
 *   - a deterministic synthetic-parameter generator and the caller-side final RMSNorm / fp16 LM head /
 *     argmax, which the reference takes from a Hugging Face checkpoint that is not available here.
 *
 * Build: oracle/Makefile, `gcc -O2 -ffp-contract=off -fopenmp`. No FMA contraction, so every float
 * operation rounds exactly as the reference's x86-64 `-O2` build does. Work is split across threads
 * only over independent outputs (rows, tokens, heads); each output's own sum stays serial in the
 * reference's order, so the thread count never changes a result bit.
 */
#include <math.h>
#include <stddef.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#define QO_HIDDEN 1536
#define QO_INTER 8960
#define QO_HEADS 12
#define QO_KV_HEADS 2
#define QO_HEAD_DIM 128
#define QO_KV_WIDTH (QO_KV_HEADS * QO_HEAD_DIM)
#define QO_GROUPS (QO_HEADS / QO_KV_HEADS)
#define QO_VOCAB 151936
#define QO_EPS 1.0e-6f
#define QO_THETA 1000000.0f

/* prefill constants, hls/prefill_only/qwen_prefill_attention_kernel.cpp:25-29 */
static const float kPi = 3.14159265358979323846f;
static const float kTwoPi = 6.28318530717958647692f;
static const float kHalfPi = 1.57079632679489661923f;
static const float kAttentionScaling = 0.08838834764831845f;
static const float kRopeFreqStep = 0.8058421877614801f;

/* ------------------------------------------------------------------------------------------------ */
/* weight decode                                                                                     */
/* ------------------------------------------------------------------------------------------------ */

/* Signed weight code at flat index `flat` (= out * in_dim + in).
 * wbits 4: low nibble at even flat index, `nibble >= 8 ? nibble - 16 : nibble`
 *          (qwen_decode_attention_kernel.cpp:44-60).
 * wbits 8: one int8 per weight (W8 track). */
static inline int weight_code(const uint8_t* w, int wbits, size_t flat) {
  if (wbits == 8) {
    return (int)(int8_t)w[flat];
  }
  const uint8_t packed = w[flat >> 1];
  const int nibble = (flat & 1u) ? ((packed >> 4) & 0xF) : (packed & 0xF);
  return nibble >= 8 ? nibble - 16 : nibble;
}

int oracle_weight_code(const uint8_t* w, int wbits, uint64_t flat) { return weight_code(w, wbits, (size_t)flat); }

/* y[o] = (bias ? bias[o] : 0) then acc += x[i] * (float(code) * scale[o]) serially over i.
 * The reference's tiling (128 or runtime tiles) carries the partial sum across input tiles, so the
 * per-output order is exactly i = 0..in_dim-1 (qwen_decode_attention_kernel.cpp:62-98). */
static void project_rows(const float* x, const uint8_t* w, int wbits, const float* bias, const float* scales,
                         int out_dim, int in_dim, float* y) {
  int o;
#pragma omp parallel for schedule(static)
  for (o = 0; o < out_dim; ++o) {
    const float s = scales[o];
    float acc = bias ? bias[o] : 0.0f;
    const size_t base = (size_t)o * (size_t)in_dim;
    for (int i = 0; i < in_dim; ++i) {
      const float wv = (float)weight_code(w, wbits, base + (size_t)i) * s;
      const float p = x[i] * wv;
      acc = acc + p;
    }
    y[o] = acc;
  }
}

/* Same as project_rows but without the OpenMP split (used inside token-parallel loops). */
static void project_rows_serial(const float* x, const uint8_t* w, int wbits, const float* bias, const float* scales,
                                int out_dim, int in_dim, float* y) {
  for (int o = 0; o < out_dim; ++o) {
    const float s = scales[o];
    float acc = bias ? bias[o] : 0.0f;
    const size_t base = (size_t)o * (size_t)in_dim;
    for (int i = 0; i < in_dim; ++i) {
      const float wv = (float)weight_code(w, wbits, base + (size_t)i) * s;
      const float p = x[i] * wv;
      acc = acc + p;
    }
    y[o] = acc;
  }
}

void oracle_project(const float* x, const uint8_t* w, int wbits, const float* bias, const float* scales, int out_dim,
                    int in_dim, float* y) {
  project_rows(x, w, wbits, bias, scales, out_dim, in_dim, y);
}

/* ------------------------------------------------------------------------------------------------ */
/* decode-path elementwise math (exact libm)                                                          */
/* ------------------------------------------------------------------------------------------------ */

/* qwen_decode_attention_kernel.cpp:13-27 (duplicate at qwen_decode_mlp_kernel.cpp:28-42) */
void oracle_decode_rmsnorm(const float* x, const float* weight, float eps, float* out) {
  double ms = 0.0;
  for (int d = 0; d < QO_HIDDEN; ++d) {
    ms += (double)x[d] * (double)x[d];
  }
  ms /= (double)QO_HIDDEN;
  const double inv = 1.0 / sqrt(ms + (double)eps);
  for (int d = 0; d < QO_HIDDEN; ++d) {
    out[d] = (float)((double)x[d] * inv * (double)weight[d]);
  }
}

/* cos/sin of the decode RoPE angle for 64 pairs at `pos` (qwen_decode_attention_kernel.cpp:29-34). */
void oracle_decode_rope_cos_sin(int pos, float* cosv, float* sinv) {
  for (int pair = 0; pair < QO_HEAD_DIM / 2; ++pair) {
    const double angle =
        (double)pos * pow((double)QO_THETA, -2.0 * (double)pair / (double)QO_HEAD_DIM);
    cosv[pair] = (float)cos(angle);
    sinv[pair] = (float)sin(angle);
  }
}

/* rotate-half pairs (i, i+64) (qwen_decode_attention_kernel.cpp:35-41 and prefill :135-140) */
static void rope_apply(float* head, const float* cosv, const float* sinv) {
  for (int pair = 0; pair < QO_HEAD_DIM / 2; ++pair) {
    const float even = head[pair];
    const float odd = head[pair + QO_HEAD_DIM / 2];
    const float a = even * cosv[pair];
    const float b = odd * sinv[pair];
    const float c = odd * cosv[pair];
    const float e = even * sinv[pair];
    head[pair] = a - b;
    head[pair + QO_HEAD_DIM / 2] = c + e;
  }
}

/* qwen_decode_attention_kernel.cpp:113-162: per head, pass 1 = max of (q.k)*scaling over tokens,
 * pass 2 = expf(s*scaling - max), denom and accum, out = accum * (1/denom). */
static void decode_context(const float* q, const float* kc, const float* vc, int total, float* ctx) {
  const float scaling = (float)(1.0 / sqrt((double)QO_HEAD_DIM));
  int head;
#pragma omp parallel for schedule(static)
  for (head = 0; head < QO_HEADS; ++head) {
    const int kvh = head / QO_GROUPS;
    const float* qh = q + head * QO_HEAD_DIM;
    float max_score = -1.0e30f;
    for (int t = 0; t < total; ++t) {
      const float* kh = kc + (size_t)t * QO_KV_WIDTH + kvh * QO_HEAD_DIM;
      float s = 0.0f;
      for (int d = 0; d < QO_HEAD_DIM; ++d) {
        const float p = qh[d] * kh[d];
        s = s + p;
      }
      const float ss = s * scaling;
      max_score = (max_score < ss) ? ss : max_score; /* std::max(a,b) returns a unless a < b */
    }
    float denom = 0.0f;
    float acc[QO_HEAD_DIM];
    for (int d = 0; d < QO_HEAD_DIM; ++d) acc[d] = 0.0f;
    for (int t = 0; t < total; ++t) {
      const float* kh = kc + (size_t)t * QO_KV_WIDTH + kvh * QO_HEAD_DIM;
      const float* vh = vc + (size_t)t * QO_KV_WIDTH + kvh * QO_HEAD_DIM;
      float s = 0.0f;
      for (int d = 0; d < QO_HEAD_DIM; ++d) {
        const float p = qh[d] * kh[d];
        s = s + p;
      }
      const float arg = s * scaling - max_score;
      const float e = expf(arg);
      denom = denom + e;
      for (int d = 0; d < QO_HEAD_DIM; ++d) {
        const float p = e * vh[d];
        acc[d] = acc[d] + p;
      }
    }
    const float inv = denom > 0.0f ? 1.0f / denom : 0.0f;
    for (int d = 0; d < QO_HEAD_DIM; ++d) ctx[head * QO_HEAD_DIM + d] = acc[d] * inv;
  }
}

/* qwen_decode_attention_kernel.cpp:168-218 (status 1 on null / negative history, else 0). The output
 * is o_proj(context) only: the reference's quantized layer does not add the attention residual. */
int oracle_decode_attention(int wbits, const float* x, int past, const float* ln_w, const uint8_t* qw,
                            const uint8_t* kw, const uint8_t* vw, const uint8_t* ow, const float* qb,
                            const float* kb, const float* vb, const float* qs, const float* ks, const float* vs,
                            const float* os, float* kc, float* vc, float* out) {
  if (!x || !out || past < 0 || !ln_w || !qw || !kw || !vw || !ow || !qb || !kb || !vb || !qs || !ks || !vs ||
      !os || !kc || !vc) {
    return 1;
  }
  float xn[QO_HIDDEN], q[QO_HIDDEN], k[QO_KV_WIDTH], v[QO_KV_WIDTH], ctx[QO_HIDDEN];
  float cosv[QO_HEAD_DIM / 2], sinv[QO_HEAD_DIM / 2];
  oracle_decode_rmsnorm(x, ln_w, QO_EPS, xn);
  project_rows(xn, qw, wbits, qb, qs, QO_HIDDEN, QO_HIDDEN, q);
  project_rows(xn, kw, wbits, kb, ks, QO_KV_WIDTH, QO_HIDDEN, k);
  project_rows(xn, vw, wbits, vb, vs, QO_KV_WIDTH, QO_HIDDEN, v);
  oracle_decode_rope_cos_sin(past, cosv, sinv);
  for (int h = 0; h < QO_HEADS; ++h) rope_apply(q + h * QO_HEAD_DIM, cosv, sinv);
  for (int h = 0; h < QO_KV_HEADS; ++h) rope_apply(k + h * QO_HEAD_DIM, cosv, sinv);
  memcpy(kc + (size_t)past * QO_KV_WIDTH, k, sizeof(k));
  memcpy(vc + (size_t)past * QO_KV_WIDTH, v, sizeof(v));
  decode_context(q, kc, vc, past + 1, ctx);
  project_rows(ctx, ow, wbits, NULL, os, QO_HIDDEN, QO_HIDDEN, out);
  return 0;
}

/* qwen_decode_mlp_kernel.cpp:79-122: silu(v) = v / (1 + expf(-v)); out = a + down(silu(g) * u). */
int oracle_decode_mlp(int wbits, const float* a, const float* ln_w, const uint8_t* gw, const uint8_t* uw,
                      const uint8_t* dw, const float* gs, const float* us, const float* ds, float* out) {
  if (!a || !out || !ln_w || !gw || !uw || !dw || !gs || !us || !ds) return 1;
  float xn[QO_HIDDEN], down[QO_HIDDEN];
  float* g = (float*)malloc(sizeof(float) * QO_INTER);
  float* u = (float*)malloc(sizeof(float) * QO_INTER);
  float* h = (float*)malloc(sizeof(float) * QO_INTER);
  oracle_decode_rmsnorm(a, ln_w, QO_EPS, xn);
  project_rows(xn, gw, wbits, NULL, gs, QO_INTER, QO_HIDDEN, g);
  project_rows(xn, uw, wbits, NULL, us, QO_INTER, QO_HIDDEN, u);
  for (int i = 0; i < QO_INTER; ++i) {
    const float e = expf(-g[i]);
    const float silu = g[i] / (1.0f + e);
    h[i] = silu * u[i];
  }
  project_rows(h, dw, wbits, NULL, ds, QO_HIDDEN, QO_INTER, down);
  for (int i = 0; i < QO_HIDDEN; ++i) out[i] = a[i] + down[i];
  free(g);
  free(u);
  free(h);
  return 0;
}

/* ------------------------------------------------------------------------------------------------ */
/* prefill-path approximations (hls/prefill_only/qwen_prefill_attention_kernel.cpp:47-143)          */
/* ------------------------------------------------------------------------------------------------ */

float oracle_approx_sqrt(float value) { /* :47-57 */
  if (value <= 0.0f) return 0.0f;
  float guess = value > 1.0f ? value : 1.0f;
  for (int iter = 0; iter < 6; ++iter) {
    const float q = value / guess;
    const float s = guess + q;
    guess = 0.5f * s;
  }
  return guess;
}

float oracle_wrap_angle(float angle) { /* :59-67 */
  while (angle > kPi) angle -= kTwoPi;
  while (angle < -kPi) angle += kTwoPi;
  return angle;
}

void oracle_approx_sincos(float angle, float* sin_value, float* cos_value) { /* :69-85 */
  float reduced = oracle_wrap_angle(angle);
  float cos_sign = 1.0f;
  if (reduced > kHalfPi) {
    reduced = kPi - reduced;
    cos_sign = -1.0f;
  } else if (reduced < -kHalfPi) {
    reduced = -kPi - reduced;
    cos_sign = -1.0f;
  }
  const float c6 = -1.0f / 5040.0f, c4 = 1.0f / 120.0f, c2 = -1.0f / 6.0f;
  const float d6 = -1.0f / 720.0f, d4 = 1.0f / 24.0f;
  const float x2 = reduced * reduced;
  /* sin: reduced * (1 + x2 * (-1/6 + x2 * (1/120 + x2 * (-1/5040)))) */
  float t = x2 * c6;
  t = c4 + t;
  t = x2 * t;
  t = c2 + t;
  t = x2 * t;
  t = 1.0f + t;
  const float sin_poly = reduced * t;
  /* cos: 1 + x2 * (-0.5 + x2 * (1/24 + x2 * (-1/720))) */
  float c = x2 * d6;
  c = d4 + c;
  c = x2 * c;
  c = -0.5f + c;
  c = x2 * c;
  const float cos_poly = 1.0f + c;
  *sin_value = sin_poly;
  *cos_value = cos_sign * cos_poly;
}

float oracle_approx_exp(float value) { /* :87-110 */
  if (value <= -16.0f) return 0.0f;
  int half_steps = 0;
  float scaled = value;
  while (scaled < -1.0f) {
    scaled *= 0.5f;
    ++half_steps;
  }
  float term = 1.0f;
  float series = 1.0f;
  for (int degree = 1; degree <= 6; ++degree) {
    const float q = scaled / (float)degree;
    term = term * q;
    series = series + term;
  }
  for (int step = 0; step < half_steps; ++step) series = series * series;
  return series > 0.0f ? series : 0.0f;
}

/* :112-126 */
void oracle_prefill_rmsnorm(const float* x, const float* weight, float eps, float* out) {
  float ms = 0.0f;
  for (int d = 0; d < QO_HIDDEN; ++d) {
    const float p = x[d] * x[d];
    ms = ms + p;
  }
  ms = ms / (float)QO_HIDDEN;
  const float inv = 1.0f / oracle_approx_sqrt(ms + eps);
  for (int d = 0; d < QO_HIDDEN; ++d) {
    const float a = x[d] * inv;
    out[d] = a * weight[d];
  }
}

/* cos/sin table of the prefill RoPE at `pos`: inv_freq starts at 1 and is multiplied by
 * kRopeFreqStep after every pair; angle = (float)pos * inv_freq (:128-143). */
void oracle_prefill_rope_cos_sin(int pos, float* cosv, float* sinv) {
  float inv_freq = 1.0f;
  for (int pair = 0; pair < QO_HEAD_DIM / 2; ++pair) {
    const float angle = (float)pos * inv_freq;
    oracle_approx_sincos(angle, &sinv[pair], &cosv[pair]);
    inv_freq *= kRopeFreqStep;
  }
}

/* Causal 2-pass context for one query (:204-289). Pass 1 takes the max of score*scaling over keys
 * 0..query; pass 2 accumulates approx_exp(score*scaling - max). The reference's key and head tiling
 * does not change the per-head order. */
static void prefill_context_query(const float* q, const float* kc, const float* vc, int query, float* ctx) {
  for (int head = 0; head < QO_HEADS; ++head) {
    const int kvh = head / QO_GROUPS;
    const float* qh = q + head * QO_HEAD_DIM;
    float max_score = -1.0e30f;
    for (int key = 0; key <= query; ++key) {
      const float* kh = kc + (size_t)key * QO_KV_WIDTH + kvh * QO_HEAD_DIM;
      float s = 0.0f;
      for (int d = 0; d < QO_HEAD_DIM; ++d) {
        const float p = qh[d] * kh[d];
        s = s + p;
      }
      const float ss = s * kAttentionScaling;
      max_score = ss > max_score ? ss : max_score;
    }
    float denom = 0.0f;
    float acc[QO_HEAD_DIM];
    for (int d = 0; d < QO_HEAD_DIM; ++d) acc[d] = 0.0f;
    for (int key = 0; key <= query; ++key) {
      const float* kh = kc + (size_t)key * QO_KV_WIDTH + kvh * QO_HEAD_DIM;
      const float* vh = vc + (size_t)key * QO_KV_WIDTH + kvh * QO_HEAD_DIM;
      float s = 0.0f;
      for (int d = 0; d < QO_HEAD_DIM; ++d) {
        const float p = qh[d] * kh[d];
        s = s + p;
      }
      const float ss = s * kAttentionScaling;
      const float e = oracle_approx_exp(ss - max_score);
      denom = denom + e;
      for (int d = 0; d < QO_HEAD_DIM; ++d) {
        const float p = e * vh[d];
        acc[d] = acc[d] + p;
      }
    }
    const float inv = denom > 0.0f ? 1.0f / denom : 0.0f;
    for (int d = 0; d < QO_HEAD_DIM; ++d) ctx[head * QO_HEAD_DIM + d] = acc[d] * inv;
  }
}

/* Prefill attention over tokens [0, seq_len): phase 1 writes post-RoPE K and biased V into the
 * token-major caches, phase 2 computes Q, context and o_proj per query (:2232-2367). Tile arguments
 * of the reference do not change numerics; the validation that depends on them lives in the
 * product's C-ABI and is compared directly against the reference library in tests. */
int oracle_prefill_attention(int wbits, const float* x, int seq_len, const float* ln_w, const uint8_t* qw,
                             const uint8_t* kw, const uint8_t* vw, const uint8_t* ow, const float* qb,
                             const float* kb, const float* vb, const float* qs, const float* ks, const float* vs,
                             const float* os, float* kc, float* vc, float* out) {
  if (!x || !out || seq_len <= 0 || !ln_w || !qw || !kw || !vw || !ow || !qb || !kb || !vb || !qs || !ks ||
      !vs || !os || !kc || !vc) {
    return 1;
  }
  int t;
#pragma omp parallel for schedule(dynamic, 1)
  for (t = 0; t < seq_len; ++t) {
    float xn[QO_HIDDEN], cosv[QO_HEAD_DIM / 2], sinv[QO_HEAD_DIM / 2];
    float* k = kc + (size_t)t * QO_KV_WIDTH;
    float* v = vc + (size_t)t * QO_KV_WIDTH;
    oracle_prefill_rmsnorm(x + (size_t)t * QO_HIDDEN, ln_w, QO_EPS, xn);
    project_rows_serial(xn, kw, wbits, kb, ks, QO_KV_WIDTH, QO_HIDDEN, k);
    project_rows_serial(xn, vw, wbits, vb, vs, QO_KV_WIDTH, QO_HIDDEN, v);
    oracle_prefill_rope_cos_sin(t, cosv, sinv);
    for (int h = 0; h < QO_KV_HEADS; ++h) rope_apply(k + h * QO_HEAD_DIM, cosv, sinv);
  }
#pragma omp parallel for schedule(dynamic, 1)
  for (t = 0; t < seq_len; ++t) {
    float xn[QO_HIDDEN], q[QO_HIDDEN], ctx[QO_HIDDEN], cosv[QO_HEAD_DIM / 2], sinv[QO_HEAD_DIM / 2];
    oracle_prefill_rmsnorm(x + (size_t)t * QO_HIDDEN, ln_w, QO_EPS, xn);
    project_rows_serial(xn, qw, wbits, qb, qs, QO_HIDDEN, QO_HIDDEN, q);
    oracle_prefill_rope_cos_sin(t, cosv, sinv);
    for (int h = 0; h < QO_HEADS; ++h) rope_apply(q + h * QO_HEAD_DIM, cosv, sinv);
    prefill_context_query(q, kc, vc, t, ctx);
    project_rows_serial(ctx, ow, wbits, NULL, os, QO_HIDDEN, QO_HIDDEN, out + (size_t)t * QO_HIDDEN);
  }
  return 0;
}

/* hls/prefill_only/qwen_prefill_mlp_kernel.cpp:256-337 (tile validation lives in the C-ABI). */
int oracle_prefill_mlp(int wbits, const float* a, int seq_len, const float* ln_w, const uint8_t* gw,
                       const uint8_t* uw, const uint8_t* dw, const float* gs, const float* us, const float* ds,
                       float* out) {
  if (!a || !out || seq_len <= 0 || !ln_w || !gw || !uw || !dw || !gs || !us || !ds) return 1;
  int t;
#pragma omp parallel for schedule(dynamic, 1)
  for (t = 0; t < seq_len; ++t) {
    float xn[QO_HIDDEN], down[QO_HIDDEN];
    float* g = (float*)malloc(sizeof(float) * QO_INTER * 3);
    float* u = g + QO_INTER;
    float* h = u + QO_INTER;
    const float* at = a + (size_t)t * QO_HIDDEN;
    oracle_prefill_rmsnorm(at, ln_w, QO_EPS, xn);
    project_rows_serial(xn, gw, wbits, NULL, gs, QO_INTER, QO_HIDDEN, g);
    project_rows_serial(xn, uw, wbits, NULL, us, QO_INTER, QO_HIDDEN, u);
    for (int i = 0; i < QO_INTER; ++i) {
      const float e = oracle_approx_exp(-g[i]);
      const float silu = g[i] / (1.0f + e);
      h[i] = silu * u[i];
    }
    project_rows_serial(h, dw, wbits, NULL, ds, QO_HIDDEN, QO_INTER, down);
    for (int i = 0; i < QO_HIDDEN; ++i) out[(size_t)t * QO_HIDDEN + i] = at[i] + down[i];
    free(g);
  }
  return 0;
}

/* ------------------------------------------------------------------------------------------------ */
/* caller-side helpers                                                                               */
/* ------------------------------------------------------------------------------------------------ */

/* The host C library's expf over an array: the function the reference host library calls for
 * std::exp on floats (qwen_decode_attention_kernel.cpp:149, qwen_decode_mlp_kernel.cpp:80), so that
 * tests can compare a GPU restatement with it on the same machine. */
void oracle_expf_array(const float* x, float* y, uint64_t n) {
  int64_t i;
#pragma omp parallel for schedule(static)
  for (i = 0; i < (int64_t)n; ++i) y[i] = expf(x[i]);
}

/* Round-to-nearest-even to bf16, kept in fp32 (reference_wrapper_backend.py:40-46). */
void oracle_round_bf16(float* x, uint64_t n) {
  for (uint64_t i = 0; i < n; ++i) {
    uint32_t bits;
    memcpy(&bits, &x[i], 4);
    const uint32_t lsb = (bits >> 16) & 1u;
    bits += 0x7FFFu + lsb;
    bits &= 0xFFFF0000u;
    memcpy(&x[i], &bits, 4);
  }
}

/* Per-output-channel symmetric quantizer (real_host_top_backend.py:31-41): scale = max|w| / qmax
 * (1 when the row is all zero), code = clip(rint(w / scale), -qmax-1, qmax). qmax = 7 packs two
 * codes per byte with the even flat index in the low nibble; qmax = 127 stores one int8 per byte. */
void oracle_quantize_rows(const float* w, int out_dim, int in_dim, int wbits, uint8_t* codes, float* scales) {
  const float qmax = wbits == 8 ? 127.0f : 7.0f;
  const int lo = wbits == 8 ? -128 : -8, hi = wbits == 8 ? 127 : 7;
  if (wbits == 4) memset(codes, 0, ((size_t)out_dim * in_dim + 1) / 2);
  for (int o = 0; o < out_dim; ++o) {
    const float* row = w + (size_t)o * in_dim;
    float m = 0.0f;
    for (int i = 0; i < in_dim; ++i) {
      const float a = fabsf(row[i]);
      m = a > m ? a : m;
    }
    const float s = m > 0.0f ? m / qmax : 1.0f;
    scales[o] = s;
    for (int i = 0; i < in_dim; ++i) {
      int q = (int)rintf(row[i] / s);
      q = q < lo ? lo : (q > hi ? hi : q);
      const size_t flat = (size_t)o * in_dim + i;
      if (wbits == 8) {
        codes[flat] = (uint8_t)(int8_t)q;
      } else {
        const uint8_t nib = (uint8_t)(q & 0xF);
        if (flat & 1u)
          codes[flat >> 1] |= (uint8_t)(nib << 4);
        else
          codes[flat >> 1] |= nib;
      }
    }
  }
}

/* ------------------------------------------------------------------------------------------------ */
/* deterministic synthetic parameters (shared bit-for-bit with the device generator)                  */
/* ------------------------------------------------------------------------------------------------ */

/* SplitMix64 finalizer (Steele, Lea, Flood 2014). */
static inline uint64_t mix64(uint64_t x) {
  x ^= x >> 30;
  x *= 0xBF58476D1CE4E5B9ull;
  x ^= x >> 27;
  x *= 0x94D049BB133111EBull;
  x ^= x >> 31;
  return x;
}

/* Approximately N(0,1): a 12-term Irwin-Hall sum of 16-bit uniforms from a counter-based hash of
 * (seed, stream, index). Integer arithmetic plus one exact int->float conversion and one power-of-2
 * scale, so host and device produce identical values; the sample is then scaled by `sigma` and
 * shifted by `mean` with two rounded fp32 operations. */
float oracle_synth_normal(uint64_t seed, uint64_t stream, uint64_t index, float mean, float sigma) {
  const uint64_t key = mix64(seed ^ mix64(stream + 0x9E3779B97F4A7C15ull));
  int64_t sum = 0;
  for (uint64_t j = 0; j < 3; ++j) {
    const uint64_t h = mix64(key + index * 3ull + j);
    sum += (int64_t)(h & 0xFFFF) + (int64_t)((h >> 16) & 0xFFFF) + (int64_t)((h >> 32) & 0xFFFF) +
           (int64_t)((h >> 48) & 0xFFFF);
  }
  const float z = (float)(2 * sum - 12 * 65535) * (1.0f / 131072.0f);
  const float scaled = z * sigma;
  return scaled + mean;
}

void oracle_synth_fill(uint64_t seed, uint64_t stream, uint64_t count, float mean, float sigma, float* out) {
  int64_t i;
#pragma omp parallel for schedule(static)
  for (i = 0; i < (int64_t)count; ++i) out[i] = oracle_synth_normal(seed, stream, (uint64_t)i, mean, sigma);
}

/* fp32 -> fp16 bits, round to nearest even (finite inputs of moderate range; used for the
 * synthetic embedding table). */
uint16_t oracle_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  const uint32_t sign = (x >> 16) & 0x8000u;
  const int32_t exp = (int32_t)((x >> 23) & 0xFF) - 127 + 15;
  uint32_t mant = x & 0x7FFFFFu;
  if (((x >> 23) & 0xFF) == 0xFF) return (uint16_t)(sign | 0x7C00u | (mant ? 0x200u : 0));
  if (exp >= 31) return (uint16_t)(sign | 0x7C00u);
  if (exp <= 0) {
    if (exp < -10) return (uint16_t)sign;
    mant |= 0x800000u;
    const int shift = 14 - exp;
    uint32_t h = mant >> shift;
    const uint32_t rem = mant & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1);
    if (rem > half || (rem == half && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
  }
  uint32_t h = ((uint32_t)exp << 10) | (mant >> 13);
  const uint32_t rem = mant & 0x1FFFu;
  if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h;
  return (uint16_t)(sign | h);
}

float oracle_f16_to_f32(uint16_t h) {
  const uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t exp = (h >> 10) & 0x1F;
  uint32_t mant = h & 0x3FFu;
  uint32_t bits;
  if (exp == 0) {
    if (mant == 0) {
      bits = sign;
    } else {
      int e = -1;
      do {
        ++e;
        mant <<= 1;
      } while (!(mant & 0x400u));
      bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((mant & 0x3FFu) << 13);
    }
  } else if (exp == 31) {
    bits = sign | 0x7F800000u | (mant << 13);
  } else {
    bits = sign | ((exp + 127 - 15) << 23) | (mant << 13);
  }
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

/* Caller-side final step (harness-defined; the reference uses the Hugging Face final norm and LM
 * head, real_host_top_backend.py:138-146): decode-style double RMSNorm with weight `norm_w`, then
 * logits[v] = sum_d float(E[v][d]) * y[d] in fp32 (serial over d), greedy argmax (lowest index on
 * ties). Returns the argmax; writes logits when `logits` is non-null. */
int oracle_lm_head_argmax(const float* hidden, const float* norm_w, const uint16_t* embed_f16, int vocab,
                          float* logits) {
  float y[QO_HIDDEN];
  oracle_decode_rmsnorm(hidden, norm_w, QO_EPS, y);
  float* lg = logits ? logits : (float*)malloc(sizeof(float) * (size_t)vocab);
  int v;
#pragma omp parallel for schedule(static)
  for (v = 0; v < vocab; ++v) {
    const uint16_t* row = embed_f16 + (size_t)v * QO_HIDDEN;
    float acc = 0.0f;
    for (int d = 0; d < QO_HIDDEN; ++d) {
      const float p = oracle_f16_to_f32(row[d]) * y[d];
      acc = acc + p;
    }
    lg[v] = acc;
  }
  int best = 0;
  for (v = 1; v < vocab; ++v)
    if (lg[v] > lg[best]) best = v;
  if (!logits) free(lg);
  return best;
}
