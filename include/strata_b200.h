/*
 * strata_b200.h — what libstrata_b200.so adds on top of strata_plugin.h.
 *
 * 1. A vendor extension on the plugin's extension chain
 *    (StrataPluginV1::extension_start, raw.rs:51-85).  The reference's ABI 0.1
 *    allocates a buffer per value per run and copies host bytes in and out
 *    (crates/ferrite-strata-plugin-api/src/host/plugin.rs:382-534); that path
 *    is kept unchanged.  The extension lets a host keep buffers resident on
 *    the device across runs (weights, KV caches), wrap device memory it
 *    already owns, enqueue a run without blocking, and join a tensor-parallel
 *    group.  A host that does not know the extension type skips it
 *    (loader.rs:279-316), so ABI 0.1 hosts are unaffected.
 *
 * 2. Kernel-level entry points with plain device pointers, used by the
 *    plugin's own executor and callable directly (for example from ctypes)
 *    to check one kernel in isolation.  Pointers are device pointers; `stream`
 *    is a cudaStream_t passed as void* (null = the legacy default stream).
 *    Every entry point returns 0 on success and a negative STRATA_* status on
 *    a rejected argument or a launch failure; kernels are asynchronous.
 *
 * bf16 tensors are passed as uint16_t bit patterns.
 */
#ifndef STRATA_B200_H
#define STRATA_B200_H

#include "strata_plugin.h"

#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------ */
/* Extension on the plugin's chain                                          */
/* ------------------------------------------------------------------------ */

/* Vendor-chosen tag ("B2DV"), outside the ABI's own 0..2 range. */
#define STRATA_B200_EXT_DEVICE 0x56443242u
#define STRATA_B200_EXT_DEVICE_VERSION 1u

typedef struct StrataB200DeviceExt {
  StrataExtBase base; /* ty == STRATA_B200_EXT_DEVICE */
  uint32_t version;   /* STRATA_B200_EXT_DEVICE_VERSION */
  uint32_t reserved;

  /* Wrap `bytes` of device memory the caller owns as a buffer.  The plugin
   * never frees it; buffer_release only drops the handle. */
  int32_t (*buffer_wrap)(void *ctx, void *device_ptr, uint64_t bytes,
                         StrataBuffer **out_buffer);
  /* The device address and byte size behind a buffer. */
  int32_t (*buffer_device_ptr)(void *ctx, const StrataBuffer *buffer,
                               void **out_ptr, uint64_t *out_bytes);
  /* Enqueue a run on the plugin's stream and return without waiting.
   * Device-side failures surface at the next synchronize or buffer_read. */
  int32_t (*run_async)(void *ctx, const StrataRunArgs *args,
                       StrataError **out_error);
  /* Wait for everything enqueued, then report any device-side failure. */
  int32_t (*synchronize)(void *ctx, StrataError **out_error);
  /* The cudaStream_t the plugin launches on. */
  void *(*stream)(void *ctx);
  /* Number of kernel launches the plugin has enqueued since load (CUDA-graph
   * replays count every kernel inside the graph). */
  uint64_t (*launch_count)(void *ctx);
  /* Tensor parallelism: rank 0 creates an id (128 bytes), every rank passes
   * it to tp_init with its own rank.  Collective; call before compile. */
  int32_t (*tp_unique_id)(void *ctx, uint8_t out_id[128]);
  int32_t (*tp_init)(void *ctx, int32_t rank, int32_t world_size,
                     const uint8_t id[128], StrataError **out_error);
  /* Select the CUDA device for this context (before any other call). */
  int32_t (*set_device)(void *ctx, int32_t device);
} StrataB200DeviceExt;

/* ------------------------------------------------------------------------ */
/* Step profile                                                             */
/* ------------------------------------------------------------------------ */

/* With STRATA_B200_STEP_TIMES=1 in the environment when the library loads,
 * every run is eager (no CUDA graph) and each of its steps is bracketed by
 * CUDA events on the plugin's stream; the device time accumulates per step
 * class ("gemv:swiglu", "attention", "all_reduce_add_norm", ...).  This
 * writes {"class": [steps, milliseconds], ...} into buf (NUL-terminated when
 * it fits), clears the totals when reset is non-zero, and returns the bytes
 * the JSON needs.  No counterpart in the reference. */
uint64_t strata_b200_step_times(char *buf, uint64_t cap, int32_t reset);

/* ------------------------------------------------------------------------ */
/* Kernel-level entry points                                                */
/* ------------------------------------------------------------------------ */

/* Quantisation, bit-exact with the CPU oracle.  w is f32 [n, k]. */
int32_t strata_b200_quant_w4g32(const float *w, int64_t n, int64_t k,
                                uint8_t *packed, uint16_t *scale_bf16,
                                void *stream);
int32_t strata_b200_quant_w8pc(const float *w, int64_t n, int64_t k,
                               int8_t *q, float *scale, void *stream);
int32_t strata_b200_dequant_w4g32(const uint8_t *packed,
                                  const uint16_t *scale_bf16, int64_t n,
                                  int64_t k, float *w, void *stream);
int32_t strata_b200_dequant_w8pc(const int8_t *q, const float *scale,
                                 int64_t n, int64_t k, float *w, void *stream);

/* y[m, n] = sum_k x[m, k] * deq(W)[n, k]  (+ residual[m, n] when non-null);
 * bf16 in and out, f32 accumulation.  k must be a multiple of 32 (w4g32) or
 * 16 (w8pc). */
int32_t strata_b200_linear_w4g32(const uint16_t *x, int64_t m, int64_t k,
                                 const uint8_t *packed,
                                 const uint16_t *scale_bf16, int64_t n,
                                 const uint16_t *residual, uint16_t *y,
                                 void *stream);
int32_t strata_b200_linear_w8pc(const uint16_t *x, int64_t m, int64_t k,
                                const int8_t *q, const float *scale,
                                int64_t n, const uint16_t *residual,
                                uint16_t *y, void *stream);

/* The same with MX weights (OCP Microscaling; the element types of
 * crates/ferrite-strata/src/dtype.rs:41-85, DType::microscaled): codes E4M3
 * [n, k] one byte each (mxfp8) or E2M1 [n, k] packed two per byte, even k in
 * the low nibble (mxfp4); scales E8M0 [n, k/32], one byte each.  Weights are
 * dequantised exactly (code * 2^(e - 127)).  k % 128 == 0 and n % 16 == 0 for
 * m <= 64 (the tensor-core GEMV). */
int32_t strata_b200_linear_mxfp8(const uint16_t *x, int64_t m, int64_t k,
                                 const uint8_t *codes,
                                 const uint8_t *scale_e8m0, int64_t n,
                                 const uint16_t *residual, uint16_t *y,
                                 void *stream);
int32_t strata_b200_linear_mxfp4(const uint16_t *x, int64_t m, int64_t k,
                                 const uint8_t *codes,
                                 const uint8_t *scale_e8m0, int64_t n,
                                 const uint16_t *residual, uint16_t *y,
                                 void *stream);

/* y[m, n] = sum_k x[m, k] * w[n, k]  (+ residual[m, n] when non-null) with
 * bf16 weights [n, k]: the reference's f32 `linear` (crates/ferrite-strata-cpu/
 * src/backend.rs:607-637) in bf16 storage with f32 accumulation.  k must be a
 * multiple of 8.  Batches of more than 64 rows run on the tcgen05 tensor cores
 * (so do the int4, int8 and MX entry points, after expanding the weights into
 * a bf16 scratch buffer the library keeps per device and stream; a call that
 * needs a larger one than it has allocates it with cudaMalloc, also while the
 * stream is being captured, and the smaller one stays allocated for graphs
 * that name it). */
int32_t strata_b200_linear_bf16(const uint16_t *x, int64_t m, int64_t k,
                                const uint16_t *w, int64_t n,
                                const uint16_t *residual, uint16_t *y,
                                void *stream);

int32_t strata_b200_rms_norm_bf16(const uint16_t *x, const uint16_t *gamma,
                                  int64_t rows, int64_t cols, float eps,
                                  uint16_t *y, void *stream);
int32_t strata_b200_rope_bf16(const uint16_t *x, const int32_t *pos,
                              int64_t rows, int64_t heads, int64_t head_dim,
                              float theta, uint16_t *y, void *stream);
int32_t strata_b200_swiglu_bf16(const uint16_t *gate, const uint16_t *up,
                                int64_t n, uint16_t *y, void *stream);

/* Decode attention.  q [batch, heads*head_dim]; k_new/v_new
 * [batch, kv_heads*head_dim] are written into the caches
 * [batch, kv_heads, max_len, head_dim] at position pos[b], then row b attends
 * to positions 0..pos[b].  `scratch` must hold
 * strata_b200_attention_decode_scratch_bytes(...) bytes. */
uint64_t strata_b200_attention_decode_scratch_bytes(int64_t batch,
                                                    int64_t heads,
                                                    int64_t head_dim,
                                                    int64_t max_len);
int32_t strata_b200_attention_decode_bf16(
    const uint16_t *q, const uint16_t *k_new, const uint16_t *v_new,
    uint16_t *k_cache, uint16_t *v_cache, const int32_t *pos, int64_t batch,
    int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t max_len,
    void *scratch, uint16_t *out, void *stream);

/* Decode attention that allocates nothing.  No counterpart in the reference:
 * it exists for callers that cannot call cudaMalloc -- for example code running
 * while a stream is captured in a mode that refuses allocation, or a runtime
 * whose device memory is all owned by its own pool.  The split-KV partials go
 * to a scratch area inside the library (a __device__ array of
 * strata_b200_noalloc_scratch_capacity() bytes, 32 MiB, reserved on every GPU
 * that loads the library until the process exits) instead of a caller buffer.
 * Same arguments and results as strata_b200_attention_decode_bf16 otherwise.
 * Returns STRATA_RESOURCE_EXHAUSTED if the shape needs more scratch than the
 * capacity.  The first call on a device looks up the scratch address there;
 * make that first call before any stream capture.  Calls that overlap on the
 * GPU share the scratch and race: serialise them (one stream, or events). */
uint64_t strata_b200_noalloc_scratch_capacity(void);
int32_t strata_b200_attention_decode_bf16_noalloc(
    const uint16_t *q, const uint16_t *k_new, const uint16_t *v_new,
    uint16_t *k_cache, uint16_t *v_cache, const int32_t *pos, int64_t batch,
    int64_t heads, int64_t kv_heads, int64_t head_dim, int64_t max_len,
    uint16_t *out, void *stream);

int32_t strata_b200_embed_bf16(const int32_t *ids, int64_t rows,
                               const uint16_t *table, int64_t vocab,
                               int64_t dim, uint16_t *out, void *stream);
int32_t strata_b200_argmax_bf16(const uint16_t *x, int64_t rows, int64_t cols,
                                int32_t *out, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* STRATA_B200_H */
