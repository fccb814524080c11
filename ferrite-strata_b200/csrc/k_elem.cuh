// Launcher declarations for every kernel family, used by the executor and the
// kernel-level C entry points.
#pragma once

#include "common.cuh"
#include "k_linear.cuh"

namespace sb {

// Output shape plus per-axis element strides of the operands (0 where an
// operand is broadcast along that axis).
struct BcastShape {
  int rank;
  int64_t total;
  int64_t dims[8];
  int64_t sa[8];
  int64_t sb[8];
};

template <typename T>
// g_ready: gamma is written by none of the kernels this launch depends on
// (it is read before the programmatic-launch wait).
int launch_rms_norm(const T* x, const T* g, int64_t rows, int64_t cols, float eps, T* y,
                    cudaStream_t st, bool g_ready = false);
template <typename T>
int launch_rope(const T* x, const int32_t* pos, int64_t rows, int64_t heads, int64_t head_dim,
                double theta, T* y, cudaStream_t st, const double* inv_freq = nullptr);
template <typename T>
int launch_swiglu(const T* gate, const T* up, int64_t n, T* y, cudaStream_t st);
// op: 0 = add, 1 = mul
template <typename T>
int launch_binary(int op, const T* a, const T* b, T* out, const BcastShape& sh, cudaStream_t st);
// op: 0 = gelu (exact), 1 = exp, 2 = log
template <typename T>
int launch_unary(int op, const T* x, int64_t n, T* y, cudaStream_t st);
template <typename T>
int launch_softmax(const T* x, int64_t rows, int64_t cols, T* y, cudaStream_t st);
template <typename T>
int launch_layer_norm(const T* x, const T* gamma, const T* beta, int64_t rows, int64_t cols,
                      float eps, T* y, cudaStream_t st);
template <typename T>
int launch_transpose2(const T* x, int64_t rows, int64_t cols, T* y, cudaStream_t st);
template <typename T>
int launch_slice_cols(const T* x, int64_t rows, int64_t cols, int64_t start, int64_t stride,
                      int64_t out_cols, T* y, cudaStream_t st);
template <typename T>
int launch_broadcast(const T* a, T* out, const BcastShape& sh, cudaStream_t st);
template <typename T>
int launch_embed(const int32_t* ids, int64_t rows, const T* table, int64_t vocab, int64_t dim,
                 T* out, int* err, cudaStream_t st);
template <typename T>
int launch_argmax(const T* x, int64_t rows, int64_t cols, int32_t* out, cudaStream_t st);
// out[b] = x[b * tokens_per_seq + tokens_per_seq - 1]: each sequence's last row.
template <typename T>
int launch_last_rows(const T* x, int64_t batch, int64_t tokens_per_seq, int64_t cols, T* out, cudaStream_t st);
int launch_gemm_f32(const float* a, const float* b, const float* bias, int64_t m, int64_t k,
                    int64_t n, bool b_is_nk, float* c, cudaStream_t st);
// dir 0: f32 -> bf16, dir 1: bf16 -> f32
int launch_convert(int dir, const void* x, int64_t n, void* y, cudaStream_t st);

// Attention (k_attention.cu).
int attention_splits(int64_t rows, int64_t kv_heads, int64_t max_len);
uint64_t attention_scratch_bytes(int64_t rows, int64_t heads, int64_t kv_heads, int64_t head_dim,
                                 int64_t max_len);
template <typename T>
int launch_kv_append(const T* k_new, const T* v_new, T* k_cache, T* v_cache, const int32_t* pos,
                     int64_t rows, int64_t tokens_per_seq, int64_t kv_heads, int64_t head_dim,
                     int64_t max_len, int* err, cudaStream_t st, const KvPages& kp = KvPages{});
template <typename T>
int launch_attention(const T* q, const T* k_cache, const T* v_cache, const int32_t* pos,
                     int64_t rows, int64_t tokens_per_seq, int64_t heads, int64_t kv_heads,
                     int64_t head_dim, int64_t max_len, float* scratch, T* out, int* err,
                     cudaStream_t st);

// bf16 decode/prefill attention with cache prefetch under programmatic launch.
int attention_chunk(int64_t rows, int64_t kv_heads);
int attention_v2_splits(int64_t rows, int64_t kv_heads, int64_t max_len);
uint64_t attention_v2_scratch_bytes(int64_t rows, int64_t heads, int64_t kv_heads, int64_t head_dim,
                                    int64_t max_len);
// A paged cache (kp.paged()) runs only on the tensor-core kernels: prefill
// when attention_prefill_supported, else decode when attention_tc_supported.
int launch_attention_v2(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                        const int32_t* pos, int64_t rows, int64_t tokens_per_seq, int64_t heads,
                        int64_t kv_heads, int64_t head_dim, int64_t max_len, bool pos_external,
                        float* scratch, uint16_t* out, int* err, cudaStream_t st,
                        const KvPages& kp = KvPages{});

// Tensor-core bf16 decode attention (k_attn_tc.cu); launch_attention_v2 uses
// it when supported.  Positions per split and the split-KV merge.
int attention_tc_span(int64_t rows, int64_t kv_heads, int64_t max_len);
bool attention_tc_supported(int64_t heads, int64_t kv_heads, int64_t head_dim);
int launch_attention_tc(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* pos,
                        int64_t rows, int64_t tokens_per_seq, int64_t heads, int64_t kv_heads, int64_t head_dim,
                        int64_t max_len, bool pos_external, float* scratch, uint16_t* out, int* err,
                        cudaStream_t st, const KvPages& kp = KvPages{});
// Prefill attention (k_attn_prefill.cu): 64-row query tiles of one sequence;
// launch_attention_v2 uses it for 16 or more tokens per sequence.
bool attention_prefill_supported(int64_t rows, int64_t tokens_per_seq, int64_t heads, int64_t kv_heads,
                                 int64_t head_dim);
int launch_attention_prefill(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* pos,
                             int64_t rows, int64_t tokens_per_seq, int64_t heads, int64_t kv_heads, int64_t head_dim,
                             int64_t max_len, uint16_t* out, int* err, cudaStream_t st,
                             const KvPages& kp = KvPages{});
int launch_attention_merge_bf16(const float* scratch, int64_t rows, int64_t heads, int64_t head_dim, int splits,
                                uint16_t* out, cudaStream_t st);

// tcgen05 bf16 GEMM for prefill-sized batches (k_gemm_tc.cu).  Linear layers
// with more than kGemvMaxRows rows of x use it; fewer rows stay on the GEMV.
constexpr int64_t kGemvMaxRows = 64;
bool gemm_tc_supported(int64_t m, int64_t n, int64_t k, const void* x, const void* w);
int launch_gemm_tc_bf16(const uint16_t* x, int64_t m, int64_t k, const uint16_t* w, int64_t n, const float* scale,
                        const uint16_t* residual, int64_t ldr, uint16_t* y, int64_t ldy, int* err, cudaStream_t st);
// y[m, n] = silu(x w_gate^T * s_gate) * (x w_up^T * s_up): gate and up of the
// same output features in one tcgen05 GEMM (bf16 weights, optional f32 scales).
int launch_gemm_tc_swiglu(const uint16_t* x, int64_t m, int64_t k, const uint16_t* w_gate, const uint16_t* w_up,
                          int64_t n, const float* s_gate, const float* s_up, uint16_t* y, int64_t ldy, int* err,
                          cudaStream_t st);
// Weights as bf16 [n, k]: fmt 1 = int8 codes (exact), fmt 0 = int4 code * bf16 group scale,
// fmt 2 / 3 = MXFP8 / MXFP4 code * E8M0 scale (exact).
int launch_codes_to_bf16(const void* w, const void* scale, int fmt, int64_t n, int64_t k, uint16_t* out,
                         cudaStream_t st);

// One-shot NVLink all-reduce (k_allreduce.cu).  Each rank's exchange region
// (allreduce_region_bytes(), CUDA IPC memory) holds per-block flags and four
// message slots; `peers.base[r]` is rank r's region as mapped in this process.
struct ArPeers {
  void* base[8];
};
constexpr size_t kArFlagBytes = 4096;              // flags of up to 128 blocks x 8 ranks
constexpr size_t kArSlotBytes = size_t(1) << 20;  // largest message
constexpr int kArMaxRows = 64;                    // rows of the fused all-reduce + add + RMSNorm
size_t allreduce_region_bytes();
size_t allreduce_counter_bytes();
bool allreduce_bf16_supported(int64_t n, const void* x, const void* y, int world);
int launch_allreduce_bf16(const uint16_t* x, uint16_t* y, int64_t n, int rank, int world, const ArPeers& peers,
                          uint32_t* counters, int* err, cudaStream_t st);
// h = bf16(all-reduce(x) + r), n = rms_norm(h) * gamma, one row per block.
bool allreduce_add_norm_supported(int64_t rows, int64_t cols, const void* x, const void* r, const void* gamma,
                                  const void* h, const void* n, int world);
int launch_allreduce_add_norm_bf16(const uint16_t* x, const uint16_t* r, const uint16_t* gamma, uint16_t* h,
                                   uint16_t* n, int64_t rows, int64_t cols, float eps, int rank, int world,
                                   const ArPeers& peers, uint32_t* counters, int* err, cudaStream_t st);

// Distributed argmax over a vocabulary split by rows between the tensor-
// parallel ranks (k_allreduce.cu).  x is this rank's logits [rows, cols];
// column c is vocabulary id offset + c.  Every rank gets, per row, the argmax
// over all ranks' columns with the replicated argmax's rules (NaN skipped,
// lowest id on ties, 0 for a row of NaNs).  world == 1 needs no peers.  With
// keys set, the rank's 64-bit keys go there instead (for a u64 max all-reduce
// by NCCL, then launch_vocab_argmax_decode).  The peer exchange (world > 1,
// no keys) takes at most kAmMaxRows rows; the other two forms take any.
constexpr int kAmMaxRows = 4096;  // rows of one exchange
template <typename T>
int launch_vocab_argmax(const T* x, int64_t rows, int64_t cols, int64_t offset, int rank, int world,
                        const ArPeers* peers, uint32_t* counters, uint64_t* keys, int32_t* out, int* err,
                        cudaStream_t st);
int launch_vocab_argmax_decode(const uint64_t* keys, int64_t rows, int32_t* out, cudaStream_t st);

// Quantisation (k_quant.cu).
int launch_quant_w4g32(const float* w, int64_t n, int64_t k, uint8_t* packed, uint16_t* scale,
                       cudaStream_t st);
int launch_quant_w8pc(const float* w, int64_t n, int64_t k, int8_t* q, float* scale,
                      cudaStream_t st);
int launch_dequant_w4g32(const uint8_t* packed, const uint16_t* scale, int64_t n, int64_t k,
                         float* w, cudaStream_t st);
int launch_dequant_w8pc(const int8_t* q, const float* scale, int64_t n, int64_t k, float* w,
                        cudaStream_t st);

}  // namespace sb
