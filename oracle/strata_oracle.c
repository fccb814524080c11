/*
 * strata_oracle.c — CPU oracle for the decoder-block hot path.
 *
 * TEST INFRASTRUCTURE ONLY: the checker, never the product.  Built with
 * -ffp-contract=off so that `acc += a * b` is a separate multiply and add, as
 * it is in the reference's Rust (which never contracts to FMA).
 *
 * Reference citations are paths inside the ferrite-strata project.
 */
#include "strata_oracle.h"

#include <math.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

/* ------------------------------------------------------------------------ */
/* bf16                                                                     */
/* ------------------------------------------------------------------------ */

uint16_t ora_f32_to_bf16(float x) {
  uint32_t bits;
  memcpy(&bits, &x, 4);
  if ((bits & 0x7f800000u) == 0x7f800000u && (bits & 0x007fffffu) != 0) {
    return (uint16_t)((bits >> 16) | 0x0040u); /* quiet NaN, sign kept */
  }
  uint32_t lsb = (bits >> 16) & 1u;
  bits += 0x7fffu + lsb; /* round to nearest, ties to even */
  return (uint16_t)(bits >> 16);
}

float ora_bf16_to_f32(uint16_t x) {
  uint32_t bits = (uint32_t)x << 16;
  float f;
  memcpy(&f, &bits, 4);
  return f;
}

void ora_round_bf16(const float *x, int64_t n, uint16_t *out) {
  for (int64_t i = 0; i < n; ++i) out[i] = ora_f32_to_bf16(x[i]);
}

void ora_widen_bf16(const uint16_t *x, int64_t n, float *out) {
  for (int64_t i = 0; i < n; ++i) out[i] = ora_bf16_to_f32(x[i]);
}

/* ------------------------------------------------------------------------ */
/* Reference kernels: crates/ferrite-strata-cpu/src/backend.rs              */
/* ------------------------------------------------------------------------ */

/* Abramowitz & Stegun 7.1.26, as backend.rs:467-478 evaluates it. */
float ora_erf(float x) {
  float sign = x < 0.0f ? -1.0f : 1.0f;
  float ax = fabsf(x);
  float t = 1.0f / (1.0f + 0.3275911f * ax);
  float poly = ((((1.0614054f * t - 1.4531521f) * t) + 1.4214138f) * t -
                0.28449672f) * t + 0.2548296f;
  float y = 1.0f - poly * t * expf(-ax * ax);
  return sign * y;
}

/* Exact GELU, x * Phi(x) (backend.rs:459-461). */
float ora_gelu(float x) {
  return 0.5f * x * (1.0f + ora_erf(x / 1.41421356237309504880f));
}

void ora_map_gelu(const float *x, int64_t n, float *out) {
  for (int64_t i = 0; i < n; ++i) out[i] = ora_gelu(x[i]);
}
void ora_map_exp(const float *x, int64_t n, float *out) {
  for (int64_t i = 0; i < n; ++i) out[i] = expf(x[i]);
}
void ora_map_log(const float *x, int64_t n, float *out) {
  for (int64_t i = 0; i < n; ++i) out[i] = logf(x[i]);
}

/* NumPy broadcasting: right-align, a missing or unit source axis repeats
 * index 0 (backend.rs:665-706 for the rank <= 2 cases it handles). */
int ora_broadcast_to(const float *a, const int64_t *a_dims, int a_rank,
                     float *out, const int64_t *out_dims, int out_rank) {
  if (a_rank > out_rank || out_rank > 8) return -1;
  int64_t src_stride[8] = {0};
  int off = out_rank - a_rank;
  int64_t stride = 1;
  for (int ax = out_rank - 1; ax >= 0; --ax) {
    int sa = ax - off;
    if (sa < 0) {
      src_stride[ax] = 0;
      continue;
    }
    int64_t sd = a_dims[sa];
    if (sd != 1 && sd != out_dims[ax]) return -1;
    src_stride[ax] = sd == 1 ? 0 : stride;
    stride *= sd;
  }
  int64_t total = 1;
  for (int ax = 0; ax < out_rank; ++ax) total *= out_dims[ax];
  int64_t idx[8] = {0};
  for (int64_t i = 0; i < total; ++i) {
    int64_t src = 0;
    for (int ax = 0; ax < out_rank; ++ax) src += idx[ax] * src_stride[ax];
    out[i] = a[src];
    for (int ax = out_rank - 1; ax >= 0; --ax) {
      if (++idx[ax] < out_dims[ax]) break;
      idx[ax] = 0;
    }
  }
  return 0;
}

int ora_elementwise(int op, const float *a, const int64_t *a_dims, int a_rank,
                    const float *b, const int64_t *b_dims, int b_rank,
                    float *out, const int64_t *out_dims, int out_rank) {
  int64_t total = 1;
  for (int ax = 0; ax < out_rank; ++ax) total *= out_dims[ax];
  float *ea = (float *)malloc(sizeof(float) * (size_t)(total ? total : 1));
  float *eb = (float *)malloc(sizeof(float) * (size_t)(total ? total : 1));
  int rc = -1;
  if (ea && eb &&
      ora_broadcast_to(a, a_dims, a_rank, ea, out_dims, out_rank) == 0 &&
      ora_broadcast_to(b, b_dims, b_rank, eb, out_dims, out_rank) == 0) {
    for (int64_t i = 0; i < total; ++i)
      out[i] = op == 0 ? ea[i] + eb[i] : ea[i] * eb[i];
    rc = 0;
  }
  free(ea);
  free(eb);
  return rc;
}

/* Naive m x k @ k x n, f32, inner index ascending (backend.rs:508-531). */
void ora_matmul(const float *a, const float *b, int64_t m, int64_t k,
                int64_t n, float *out) {
  for (int64_t r = 0; r < m; ++r)
    for (int64_t c = 0; c < n; ++c) {
      float acc = 0.0f;
      for (int64_t i = 0; i < k; ++i) acc += a[r * k + i] * b[i * n + c];
      out[r * n + c] = acc;
    }
}

/* x @ w^T + bias with w as [out, in] (backend.rs:607-637). */
void ora_linear(const float *x, const float *w, const float *bias, int64_t m,
                int64_t k, int64_t n, float *out) {
  for (int64_t r = 0; r < m; ++r)
    for (int64_t c = 0; c < n; ++c) {
      float acc = 0.0f;
      for (int64_t i = 0; i < k; ++i) acc += x[r * k + i] * w[c * k + i];
      if (bias) acc += bias[c];
      out[r * n + c] = acc;
    }
}

/* Row softmax with the row max subtracted (backend.rs:538-555). */
void ora_softmax(const float *x, int64_t rows, int64_t cols, float *out) {
  for (int64_t r = 0; r < rows; ++r) {
    const float *row = x + r * cols;
    float mx = -INFINITY;
    for (int64_t c = 0; c < cols; ++c) mx = fmaxf(mx, row[c]);
    float sum = 0.0f;
    for (int64_t c = 0; c < cols; ++c) sum += expf(row[c] - mx);
    for (int64_t c = 0; c < cols; ++c) out[r * cols + c] = expf(row[c] - mx) / sum;
  }
}

/* Biased-variance LayerNorm over the trailing axis (backend.rs:562-600). */
void ora_layer_norm(const float *x, const float *gamma, const float *beta,
                    int64_t rows, int64_t cols, float eps, float *out) {
  float cols_f = (float)cols;
  for (int64_t r = 0; r < rows; ++r) {
    const float *row = x + r * cols;
    float sum = 0.0f;
    for (int64_t c = 0; c < cols; ++c) sum += row[c];
    float mean = sum / cols_f;
    float var = 0.0f;
    for (int64_t c = 0; c < cols; ++c) {
      float d = row[c] - mean;
      var += d * d;
    }
    var /= cols_f;
    float den = sqrtf(var + eps);
    for (int64_t c = 0; c < cols; ++c)
      out[r * cols + c] = ((row[c] - mean) / den) * gamma[c] + beta[c];
  }
}

void ora_transpose2(const float *x, int64_t rows, int64_t cols, float *out) {
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t c = 0; c < cols; ++c) out[c * rows + r] = x[r * cols + c];
}

/* Columns start, start+stride, ... below end, dropping any >= cols
 * (backend.rs:708-742). */
int64_t ora_slice_cols(const float *x, int64_t rows, int64_t cols,
                       int64_t start, int64_t end, int64_t stride, float *out) {
  if (stride <= 0) return -1;
  int64_t n = 0;
  for (int64_t i = start; i < end; i += stride)
    if (i >= 0 && i < cols) ++n;
  for (int64_t r = 0; r < rows; ++r) {
    int64_t j = 0;
    for (int64_t i = start; i < end; i += stride)
      if (i >= 0 && i < cols) out[r * n + j++] = x[r * cols + i];
  }
  return n;
}

/* ------------------------------------------------------------------------ */
/* Quantisation conventions (defined by this backend; the reference has none) */
/* ------------------------------------------------------------------------ */

static float clampf(float v, float lo, float hi) {
  return v < lo ? lo : (v > hi ? hi : v);
}

void ora_quant_w8pc(const float *w, int64_t n, int64_t k, int8_t *q,
                    float *s) {
  for (int64_t r = 0; r < n; ++r) {
    float amax = 0.0f;
    for (int64_t c = 0; c < k; ++c) amax = fmaxf(amax, fabsf(w[r * k + c]));
    float sc = amax / 127.0f;
    s[r] = sc;
    for (int64_t c = 0; c < k; ++c) {
      float v = sc == 0.0f ? 0.0f : clampf(rintf(w[r * k + c] / sc), -127.0f, 127.0f);
      q[r * k + c] = (int8_t)v;
    }
  }
}

void ora_quant_w4g32(const float *w, int64_t n, int64_t k, uint8_t *packed,
                     uint16_t *s_bf16) {
  int64_t groups = k / 32;
  for (int64_t r = 0; r < n; ++r)
    for (int64_t g = 0; g < groups; ++g) {
      const float *src = w + r * k + g * 32;
      float amax = 0.0f;
      for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(src[i]));
      uint16_t sb = ora_f32_to_bf16(amax / 7.0f);
      float sc = ora_bf16_to_f32(sb);
      s_bf16[r * groups + g] = sb;
      for (int i = 0; i < 32; i += 2) {
        int lo = sc == 0.0f ? 0 : (int)clampf(rintf(src[i] / sc), -8.0f, 7.0f);
        int hi = sc == 0.0f ? 0 : (int)clampf(rintf(src[i + 1] / sc), -8.0f, 7.0f);
        packed[r * (k / 2) + g * 16 + i / 2] =
            (uint8_t)((lo & 0xf) | ((hi & 0xf) << 4));
      }
    }
}

void ora_dequant_w8pc(const int8_t *q, const float *s, int64_t n, int64_t k,
                      float *w) {
  for (int64_t r = 0; r < n; ++r)
    for (int64_t c = 0; c < k; ++c) w[r * k + c] = (float)q[r * k + c] * s[r];
}

static inline int nibble(const uint8_t *packed, int64_t row_bytes, int64_t r,
                         int64_t c) {
  uint8_t b = packed[r * row_bytes + c / 2];
  int v = (c & 1) ? (b >> 4) : (b & 0xf);
  return v >= 8 ? v - 16 : v;
}

void ora_dequant_w4g32(const uint8_t *packed, const uint16_t *s_bf16,
                       int64_t n, int64_t k, float *w) {
  int64_t groups = k / 32;
  for (int64_t r = 0; r < n; ++r)
    for (int64_t c = 0; c < k; ++c)
      w[r * k + c] = (float)nibble(packed, k / 2, r, c) *
                     ora_bf16_to_f32(s_bf16[r * groups + c / 32]);
}

/* ------------------------------------------------------------------------ */
/* Decoder ops (new; parity unpinned by the reference)                      */
/* ------------------------------------------------------------------------ */

void ora_rms_norm(const float *x, const float *g, int64_t rows, int64_t cols,
                  float eps, float *out) {
  for (int64_t r = 0; r < rows; ++r) {
    const float *row = x + r * cols;
    float ss = 0.0f;
    for (int64_t c = 0; c < cols; ++c) ss += row[c] * row[c];
    float inv = 1.0f / sqrtf(ss / (float)cols + eps);
    for (int64_t c = 0; c < cols; ++c) out[r * cols + c] = (row[c] * inv) * g[c];
  }
}

void ora_rope(const float *x, const int32_t *pos, int64_t rows, int64_t heads,
              int64_t head_dim, double theta, float *out) {
  int64_t half = head_dim / 2;
  int64_t width = heads * head_dim;
  for (int64_t r = 0; r < rows; ++r)
    for (int64_t h = 0; h < heads; ++h) {
      const float *src = x + r * width + h * head_dim;
      float *dst = out + r * width + h * head_dim;
      for (int64_t i = 0; i < half; ++i) {
        double inv = pow(theta, -2.0 * (double)i / (double)head_dim);
        double ang = (double)pos[r] * inv;
        double c = cos(ang), s = sin(ang);
        double x1 = src[i], x2 = src[i + half];
        dst[i] = (float)(x1 * c - x2 * s);
        dst[i + half] = (float)(x2 * c + x1 * s);
      }
    }
}

float ora_silu(float x) { return x / (1.0f + expf(-x)); }

void ora_swiglu(const float *gate, const float *up, int64_t n, float *out) {
  for (int64_t i = 0; i < n; ++i) out[i] = ora_silu(gate[i]) * up[i];
}

static void attention_row(const float *q, const float *k_cache,
                          const float *v_cache, int32_t seq, int32_t pos,
                          int64_t heads, int64_t kv_heads, int64_t head_dim,
                          int64_t max_len, float *out, float *scores) {
  int64_t group = heads / kv_heads;
  float scale = 1.0f / sqrtf((float)head_dim);
  int64_t len = (int64_t)pos + 1;
  for (int64_t h = 0; h < heads; ++h) {
    int64_t kvh = h / group;
    const float *qh = q + h * head_dim;
    const float *kb = k_cache + (((int64_t)seq * kv_heads + kvh) * max_len) * head_dim;
    const float *vb = v_cache + (((int64_t)seq * kv_heads + kvh) * max_len) * head_dim;
    for (int64_t t = 0; t < len; ++t) {
      float acc = 0.0f;
      for (int64_t d = 0; d < head_dim; ++d) acc += qh[d] * kb[t * head_dim + d];
      scores[t] = acc * scale;
    }
    ora_softmax(scores, 1, len, scores);
    for (int64_t d = 0; d < head_dim; ++d) {
      float acc = 0.0f;
      for (int64_t t = 0; t < len; ++t) acc += scores[t] * vb[t * head_dim + d];
      out[h * head_dim + d] = acc;
    }
  }
}

void ora_attention(const float *q, const float *k_cache, const float *v_cache,
                   const int32_t *seq, const int32_t *pos, int64_t rows,
                   int64_t heads, int64_t kv_heads, int64_t head_dim,
                   int64_t max_len, float *out) {
  float *scores = (float *)malloc(sizeof(float) * (size_t)max_len);
  for (int64_t r = 0; r < rows; ++r)
    attention_row(q + r * heads * head_dim, k_cache, v_cache, seq[r], pos[r],
                  heads, kv_heads, head_dim, max_len, out + r * heads * head_dim,
                  scores);
  free(scores);
}

void ora_attention_mt(const float *q, const float *k_cache,
                      const float *v_cache, const int32_t *seq,
                      const int32_t *pos, int64_t rows, int64_t heads,
                      int64_t kv_heads, int64_t head_dim, int64_t max_len,
                      float *out, int threads) {
#pragma omp parallel num_threads(threads)
  {
    float *scores = (float *)malloc(sizeof(float) * (size_t)max_len);
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; ++r)
      attention_row(q + r * heads * head_dim, k_cache, v_cache, seq[r], pos[r],
                    heads, kv_heads, head_dim, max_len,
                    out + r * heads * head_dim, scores);
    free(scores);
  }
}

static void linear_w4g32_row(const float *xr, const uint8_t *packed,
                             const uint16_t *s_bf16, int64_t k, int64_t c,
                             float *out) {
  int64_t groups = k / 32, row_bytes = k / 2;
  float acc = 0.0f;
  for (int64_t i = 0; i < k; ++i) {
    float wv = (float)nibble(packed, row_bytes, c, i) *
               ora_bf16_to_f32(s_bf16[c * groups + i / 32]);
    acc += xr[i] * wv;
  }
  *out = acc;
}

void ora_linear_w4g32(const float *x, const uint8_t *packed,
                      const uint16_t *s_bf16, int64_t m, int64_t k, int64_t n,
                      float *out) {
  for (int64_t r = 0; r < m; ++r)
    for (int64_t c = 0; c < n; ++c)
      linear_w4g32_row(x + r * k, packed, s_bf16, k, c, out + r * n + c);
}

void ora_linear_w4g32_mt(const float *x, const uint8_t *packed,
                         const uint16_t *s_bf16, int64_t m, int64_t k,
                         int64_t n, float *out, int threads) {
#pragma omp parallel for collapse(2) schedule(static) num_threads(threads)
  for (int64_t r = 0; r < m; ++r)
    for (int64_t c = 0; c < n; ++c)
      linear_w4g32_row(x + r * k, packed, s_bf16, k, c, out + r * n + c);
}

static void linear_w8pc_row(const float *xr, const int8_t *q, const float *s,
                            int64_t k, int64_t c, float *out) {
  float acc = 0.0f;
  for (int64_t i = 0; i < k; ++i) acc += xr[i] * ((float)q[c * k + i] * s[c]);
  *out = acc;
}

void ora_linear_w8pc(const float *x, const int8_t *q, const float *s,
                     int64_t m, int64_t k, int64_t n, float *out) {
  for (int64_t r = 0; r < m; ++r)
    for (int64_t c = 0; c < n; ++c)
      linear_w8pc_row(x + r * k, q, s, k, c, out + r * n + c);
}

void ora_linear_w8pc_mt(const float *x, const int8_t *q, const float *s,
                        int64_t m, int64_t k, int64_t n, float *out,
                        int threads) {
#pragma omp parallel for collapse(2) schedule(static) num_threads(threads)
  for (int64_t r = 0; r < m; ++r)
    for (int64_t c = 0; c < n; ++c)
      linear_w8pc_row(x + r * k, q, s, k, c, out + r * n + c);
}

int ora_embed(const int32_t *ids, int64_t rows, const float *table,
              int64_t vocab, int64_t dim, float *out) {
  int rc = 0;
  for (int64_t r = 0; r < rows; ++r) {
    if (ids[r] < 0 || ids[r] >= vocab) {
      rc = -1;
      continue;
    }
    memcpy(out + r * dim, table + (int64_t)ids[r] * dim, sizeof(float) * (size_t)dim);
  }
  return rc;
}

void ora_argmax(const float *x, int64_t rows, int64_t cols, int32_t *out) {
  for (int64_t r = 0; r < rows; ++r) {
    int32_t best = 0;
    float bv = -INFINITY;
    int found = 0;
    for (int64_t c = 0; c < cols; ++c) {
      float v = x[r * cols + c];
      if (isnan(v)) continue;
      if (!found || v > bv) {
        bv = v;
        best = (int32_t)c;
        found = 1;
      }
    }
    out[r] = best;
  }
}

/* ------------------------------------------------------------------------ */
/* Deterministic inputs: splitmix64 + Box-Muller                            */
/* ------------------------------------------------------------------------ */

static uint64_t splitmix64(uint64_t *state) {
  uint64_t z = (*state += 0x9e3779b97f4a7c15ull);
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

void ora_normal_f32(uint64_t seed, int64_t n, double mean, double std,
                    float *out) {
  uint64_t st = seed;
  const double two_pi = 6.283185307179586476925286766559;
  for (int64_t i = 0; i < n; i += 2) {
    double u1 = ((double)(splitmix64(&st) >> 11) + 0.5) * (1.0 / 9007199254740992.0);
    double u2 = (double)(splitmix64(&st) >> 11) * (1.0 / 9007199254740992.0);
    double r = sqrt(-2.0 * log(u1));
    out[i] = (float)(mean + std * r * cos(two_pi * u2));
    if (i + 1 < n) out[i + 1] = (float)(mean + std * r * sin(two_pi * u2));
  }
}

void ora_uniform_i32(uint64_t seed, int64_t n, int32_t lo, int32_t hi,
                     int32_t *out) {
  uint64_t st = seed;
  uint64_t span = (uint64_t)((int64_t)hi - (int64_t)lo);
  for (int64_t i = 0; i < n; ++i)
    out[i] = (int32_t)((int64_t)lo + (int64_t)(splitmix64(&st) % span));
}

int ora_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
