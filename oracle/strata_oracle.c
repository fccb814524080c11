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
/* MX weights (OCP Microscaling Formats v1.0, restated; the reference names  */
/* the element types in dtype.rs:41-85 but computes none of them).           */
/* A block of 32 codes along k shares one E8M0 scale 2^(e - 127) (code 255  */
/* is NaN).  FP8 E4M3: sign, 4-bit exponent (bias 7), 3-bit mantissa,       */
/* largest 448, 0x7f / 0xff NaN.  FP4 E2M1: sign, 2-bit exponent (bias 1),  */
/* 1-bit mantissa: 0, 0.5, 1, 1.5, 2, 3, 4, 6; packed two per byte with the */
/* even k in the low nibble.  The block scale is 2^(floor(log2(amax)) -     */
/* emax), emax = 8 (E4M3) or 2 (E2M1), an all-zero block taking code 0;    */
/* each value divided by it rounds to nearest even, saturating at the       */
/* format's largest magnitude.  Dequantisation, code * 2^(e - 127), is      */
/* exact in f32 and in bf16.                                                */
/* ------------------------------------------------------------------------ */

float ora_e4m3_to_f32(uint8_t c) {
  const int e = (c >> 3) & 15, m = c & 7;
  float v;
  if ((c & 0x7f) == 0x7f) return NAN;
  if (e == 0)
    v = ldexpf((float)m, -9);
  else
    v = ldexpf(1.0f + (float)m / 8.0f, e - 7);
  return (c & 0x80) ? -v : v;
}

float ora_e2m1_to_f32(uint8_t c) {
  static const float mag[8] = {0.0f, 0.5f, 1.0f, 1.5f, 2.0f, 3.0f, 4.0f, 6.0f};
  const float v = mag[c & 7];
  return (c & 8) ? -v : v;
}

uint8_t ora_f32_to_e4m3(float x) {
  if (isnan(x)) return 0x7f;
  const uint8_t sign = signbit(x) ? 0x80 : 0;
  const float a = fabsf(x);
  if (a >= 448.0f) return sign | 0x7e;
  if (a < ldexpf(1.0f, -6)) {  /* subnormal range: steps of 2^-9 */
    const int m = (int)rintf(ldexpf(a, 9));
    return sign | (uint8_t)m;  /* m == 8 is the smallest normal, code 0x08 */
  }
  int e;
  frexpf(a, &e); /* a = f * 2^e, f in [0.5, 1) */
  e -= 1;        /* a in [2^e, 2^(e+1)) */
  int m = (int)rintf((ldexpf(a, -e) - 1.0f) * 8.0f);
  if (m == 8) {
    m = 0;
    e += 1;
  }
  if (e + 7 > 15 || (e + 7 == 15 && m == 7)) return sign | 0x7e;
  return sign | (uint8_t)(((e + 7) << 3) | m);
}

uint8_t ora_f32_to_e2m1(float x) {
  const uint8_t sign = signbit(x) ? 8 : 0;
  const float a = fabsf(x);
  uint8_t idx;
  /* nearest of 0, .5, 1, 1.5, 2, 3, 4, 6; a tie goes to the even mantissa */
  if (isnan(x)) idx = 0;
  else if (a <= 0.25f) idx = 0;
  else if (a < 0.75f) idx = 1;
  else if (a <= 1.25f) idx = 2;
  else if (a < 1.75f) idx = 3;
  else if (a <= 2.5f) idx = 4;
  else if (a < 3.5f) idx = 5;
  else if (a <= 5.0f) idx = 6;
  else idx = 7;
  return sign | idx;
}

/* The E8M0 scale code of a block whose largest magnitude is amax. */
static uint8_t mx_scale_code(float amax, int emax) {
  if (!(amax > 0.0f)) return 0;
  int e;
  frexpf(amax, &e);
  int x = (e - 1) - emax + 127;
  if (x < 0) x = 0;
  if (x > 254) x = 254;
  return (uint8_t)x;
}

static float e8m0_to_f32(uint8_t s) { return s == 255 ? NAN : ldexpf(1.0f, (int)s - 127); }

/* fmt 0: E4M3 codes [n, k]; fmt 1: E2M1 codes packed [n, k/2].  Scales
   [n, k/32]. */
void ora_quant_mx(const float *w, int64_t n, int64_t k, int fmt, uint8_t *codes, uint8_t *scales) {
  const int64_t blocks = k / 32;
  for (int64_t r = 0; r < n; ++r)
    for (int64_t b = 0; b < blocks; ++b) {
      const float *src = w + r * k + b * 32;
      float amax = 0.0f;
      for (int i = 0; i < 32; ++i) amax = fmaxf(amax, fabsf(src[i]));
      const uint8_t sc = mx_scale_code(amax, fmt == 0 ? 8 : 2);
      scales[r * blocks + b] = sc;
      const int shift = 127 - (int)sc; /* divide by 2^(sc - 127) exactly */
      for (int i = 0; i < 32; ++i) {
        const float q = ldexpf(src[i], shift);
        if (fmt == 0) {
          codes[r * k + b * 32 + i] = ora_f32_to_e4m3(q);
        } else {
          const uint8_t c = ora_f32_to_e2m1(q);
          uint8_t *dst = codes + r * (k / 2) + b * 16 + i / 2;
          *dst = (i & 1) ? (uint8_t)((*dst & 0x0f) | (c << 4)) : (uint8_t)((*dst & 0xf0) | c);
        }
      }
    }
}

static inline float mx_code(const uint8_t *codes, int64_t k, int fmt, int64_t r, int64_t c) {
  if (fmt == 0) return ora_e4m3_to_f32(codes[r * k + c]);
  const uint8_t b = codes[r * (k / 2) + c / 2];
  return ora_e2m1_to_f32((c & 1) ? (b >> 4) : (b & 15));
}

void ora_dequant_mx(const uint8_t *codes, const uint8_t *scales, int64_t n, int64_t k, int fmt, float *w) {
  for (int64_t r = 0; r < n; ++r)
    for (int64_t c = 0; c < k; ++c)
      w[r * k + c] = mx_code(codes, k, fmt, r, c) * e8m0_to_f32(scales[r * (k / 32) + c / 32]);
}

/* y = x . dequant(W)^T, each weight dequantised exactly and accumulated in
   k order in f32, as the int4 linear above. */
static void linear_mx_row(const float *xr, const uint8_t *codes, const uint8_t *scales, int64_t k, int fmt,
                          int64_t c, float *out) {
  float acc = 0.0f;
  for (int64_t i = 0; i < k; ++i)
    acc += xr[i] * (mx_code(codes, k, fmt, c, i) * e8m0_to_f32(scales[c * (k / 32) + i / 32]));
  *out = acc;
}

void ora_linear_mx_mt(const float *x, const uint8_t *codes, const uint8_t *scales, int fmt, int64_t m, int64_t k,
                      int64_t n, float *out, int threads) {
#pragma omp parallel for collapse(2) schedule(static) num_threads(threads)
  for (int64_t r = 0; r < m; ++r)
    for (int64_t c = 0; c < n; ++c) linear_mx_row(x + r * k, codes, scales, k, fmt, c, out + r * n + c);
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
