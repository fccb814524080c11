/*
 * strata_oracle.h — CPU oracle for the decoder-block hot path.
 *
 * TEST INFRASTRUCTURE ONLY.  This library is the checker the B200 backend is
 * compared against; it is called from tests/, from __graft_entry__.smoke() and
 * from bench.py's CPU-baseline leg, and never from the product path.
 *
 * Two kinds of function live here:
 *
 *  1. Restatements of the reference CPU backend's kernels
 *     (crates/ferrite-strata-cpu/src/backend.rs:448-742): strict k-order f32
 *     accumulation, max-subtracted softmax, biased-variance LayerNorm,
 *     Abramowitz & Stegun 7.1.26 erf for exact GELU, NumPy broadcasting.
 *     These are pinned by the reference's own known-answer tests
 *     (crates/ferrite-strata-cpu/tests/kernels.rs).
 *
 *  2. The decoder ops the reference does not have (RMSNorm, RoPE, SiLU/SwiGLU,
 *     causal/GQA attention over a KV cache, int8/int4 quantisation, bf16
 *     rounding, embedding gather, argmax).  They are written from the
 *     mathematics in the same naive style.  No reference code or test pins
 *     them: their parity is unpinned and rests on this file's own
 *     known-answer tests.
 *
 * All functions are single-threaded unless the name ends in `_mt`, which
 * splits the outermost loop across `threads` OpenMP threads without changing
 * any per-element accumulation order (results are bit-identical to the
 * single-threaded form).
 */
#ifndef STRATA_ORACLE_H
#define STRATA_ORACLE_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---- bf16 ---------------------------------------------------------------- */
uint16_t ora_f32_to_bf16(float x); /* round to nearest even; NaN stays NaN */
float ora_bf16_to_f32(uint16_t x);
void ora_round_bf16(const float *x, int64_t n, uint16_t *out);
void ora_widen_bf16(const uint16_t *x, int64_t n, float *out);

/* ---- reference kernels (cpu/backend.rs) ---------------------------------- */
float ora_erf(float x);  /* backend.rs:467-478 */
float ora_gelu(float x); /* backend.rs:459-461 */
void ora_map_gelu(const float *x, int64_t n, float *out);
void ora_map_exp(const float *x, int64_t n, float *out);
void ora_map_log(const float *x, int64_t n, float *out);
/* NumPy-broadcast elementwise add (op=0) or mul (op=1), rank <= 8
 * (backend.rs:480-500, 665-706).  Returns 0, or -1 if not broadcastable. */
int ora_elementwise(int op, const float *a, const int64_t *a_dims, int a_rank,
                    const float *b, const int64_t *b_dims, int b_rank,
                    float *out, const int64_t *out_dims, int out_rank);
int ora_broadcast_to(const float *a, const int64_t *a_dims, int a_rank,
                     float *out, const int64_t *out_dims, int out_rank);
void ora_matmul(const float *a, const float *b, int64_t m, int64_t k,
                int64_t n, float *out); /* backend.rs:508-531 */
void ora_linear(const float *x, const float *w, const float *bias, int64_t m,
                int64_t k, int64_t n, float *out); /* backend.rs:607-637 */
void ora_softmax(const float *x, int64_t rows, int64_t cols,
                 float *out); /* backend.rs:538-555 */
void ora_layer_norm(const float *x, const float *gamma, const float *beta,
                    int64_t rows, int64_t cols, float eps,
                    float *out); /* backend.rs:562-600 */
void ora_transpose2(const float *x, int64_t rows, int64_t cols,
                    float *out); /* backend.rs:639-657 */
/* Slice along axis 1 of a rank-2 tensor (backend.rs:708-742).  Returns the
 * number of output columns. */
int64_t ora_slice_cols(const float *x, int64_t rows, int64_t cols,
                       int64_t start, int64_t end, int64_t stride, float *out);

/* ---- quantisation (the build's conventions; bit-exact contract) ---------- */
/* int8 symmetric per output channel: s[n] = max|w[n,:]| / 127 (f32),
 * q = clamp(rne(w / s), -127, 127); an all-zero row has s = 0 and q = 0. */
void ora_quant_w8pc(const float *w, int64_t n, int64_t k, int8_t *q,
                    float *s);
/* int4 symmetric, group 32 along k: s = bf16(max|w_g| / 7), then
 * q = clamp(rne(w / f32(s)), -8, 7), two per byte, low nibble = even k. */
void ora_quant_w4g32(const float *w, int64_t n, int64_t k, uint8_t *packed,
                     uint16_t *s_bf16);
void ora_dequant_w8pc(const int8_t *q, const float *s, int64_t n, int64_t k,
                      float *w);
void ora_dequant_w4g32(const uint8_t *packed, const uint16_t *s_bf16,
                       int64_t n, int64_t k, float *w);

/* ---- decoder ops --------------------------------------------------------- */
/* y = x * rsqrt(mean(x^2) + eps) * g, f32 statistics in column order. */
void ora_rms_norm(const float *x, const float *g, int64_t rows, int64_t cols,
                  float eps, float *out);
/* Rotate-half RoPE on `heads` heads of `head_dim` per row; row r has position
 * pos[r].  inv_freq_i = theta^(-2i/head_dim), angles in double. */
void ora_rope(const float *x, const int32_t *pos, int64_t rows, int64_t heads,
              int64_t head_dim, double theta, float *out);
float ora_silu(float x);
void ora_swiglu(const float *gate, const float *up, int64_t n, float *out);
/* Causal/GQA attention for a set of query rows against a KV cache laid out
 * [batch, kv_heads, max_len, head_dim].  Query row r belongs to sequence
 * seq[r] and sits at position pos[r]; it attends to cache positions
 * 0..pos[r] inclusive.  q: [rows, heads*head_dim]; out same shape.  Scores are
 * k-order f32 dot products times 1/sqrt(head_dim), then the reference softmax. */
void ora_attention(const float *q, const float *k_cache, const float *v_cache,
                   const int32_t *seq, const int32_t *pos, int64_t rows,
                   int64_t heads, int64_t kv_heads, int64_t head_dim,
                   int64_t max_len, float *out);
/* Linear with dequantised weights, k-order f32 accumulation:
 * out[m, n] = sum_k x[m, k] * deq(w)[n, k]  (+ residual[m, n] if non-null). */
void ora_linear_w4g32(const float *x, const uint8_t *packed,
                      const uint16_t *s_bf16, int64_t m, int64_t k, int64_t n,
                      float *out);
void ora_linear_w8pc(const float *x, const int8_t *q, const float *s,
                     int64_t m, int64_t k, int64_t n, float *out);
void ora_linear_w4g32_mt(const float *x, const uint8_t *packed,
                         const uint16_t *s_bf16, int64_t m, int64_t k,
                         int64_t n, float *out, int threads);
void ora_linear_w8pc_mt(const float *x, const int8_t *q, const float *s,
                        int64_t m, int64_t k, int64_t n, float *out,
                        int threads);
void ora_attention_mt(const float *q, const float *k_cache,
                      const float *v_cache, const int32_t *seq,
                      const int32_t *pos, int64_t rows, int64_t heads,
                      int64_t kv_heads, int64_t head_dim, int64_t max_len,
                      float *out, int threads);
/* Row gather: out[r, :] = table[ids[r], :].  Returns -1 on an id out of
 * range (nothing written for that row), else 0. */
int ora_embed(const int32_t *ids, int64_t rows, const float *table,
              int64_t vocab, int64_t dim, float *out);
/* Argmax per row; the lowest index wins ties; NaN never wins. */
void ora_argmax(const float *x, int64_t rows, int64_t cols, int32_t *out);

/* ---- MX weights (OCP Microscaling v1.0; block 32 along k, E8M0 scales) -- */
float ora_e4m3_to_f32(uint8_t c);
float ora_e2m1_to_f32(uint8_t c);
uint8_t ora_f32_to_e4m3(float x); /* nearest even, saturating at 448 */
uint8_t ora_f32_to_e2m1(float x); /* nearest even, saturating at 6 */
/* fmt 0: E4M3 codes [n, k]; fmt 1: E2M1 codes packed [n, k/2] (even k low) */
void ora_quant_mx(const float *w, int64_t n, int64_t k, int fmt, uint8_t *codes, uint8_t *scales);
void ora_dequant_mx(const uint8_t *codes, const uint8_t *scales, int64_t n, int64_t k, int fmt, float *w);
void ora_linear_mx_mt(const float *x, const uint8_t *codes, const uint8_t *scales, int fmt, int64_t m, int64_t k,
                      int64_t n, float *out, int threads);

/* ---- deterministic inputs ------------------------------------------------ */
/* splitmix64 stream feeding Box-Muller in double; returns N(mean, std) as f32
 * (rounded from double).  Shared by tests and bench so GPU and CPU inputs are
 * byte-identical. */
void ora_normal_f32(uint64_t seed, int64_t n, double mean, double std,
                    float *out);
void ora_uniform_i32(uint64_t seed, int64_t n, int32_t lo, int32_t hi,
                     int32_t *out); /* [lo, hi) */

int ora_max_threads(void);

#ifdef __cplusplus
}
#endif
#endif
