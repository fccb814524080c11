// Kernel-level C entry points declared in include/strata_b200.h.
#include "../../include/strata_b200.h"
#include "k_elem.cuh"
#include "k_gemv_mma.cuh"

#include <algorithm>
#include <cstdlib>
#include <map>
#include <mutex>
#include <utility>
#include <vector>

namespace sb {
std::atomic<uint64_t> g_launches{0};

bool pdl_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("STRATA_B200_PDL");
    return !(v && *v == '0');
  }();
  return on;
}
}

using namespace sb;

static inline cudaStream_t S(void* s) { return reinterpret_cast<cudaStream_t>(s); }

// Weight-expansion scratch of the linear entry points: one grow-only device
// buffer per (device, stream).  Work on one stream runs in order, so a buffer
// is never used by two launches at once.  A buffer that must grow is
// replaced by one of at least twice its size and the old one is kept, never
// freed: a CUDA graph captured from an earlier call may still name it (the
// kept buffers add up to less than the live one).  Allocation is a plain
// cudaMalloc in the relaxed capture mode, so a call made while its stream is
// being captured gets ordinary device memory, valid outside the graph too,
// rather than a graph-owned allocation.  The buffers live until the process
// exits.
static void* linear_scratch(cudaStream_t st, size_t bytes) {
  static std::mutex mu;
  static std::map<std::pair<int, cudaStream_t>, std::pair<void*, size_t>> bufs;
  static std::vector<void*> kept;
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return nullptr;
  std::lock_guard<std::mutex> lk(mu);
  auto& e = bufs[{dev, st}];
  if (e.first && e.second >= bytes) return e.first;
  const size_t want = std::max(bytes, 2 * e.second);
  cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
  cudaThreadExchangeStreamCaptureMode(&mode);
  void* p = nullptr;
  const cudaError_t rc = cudaMalloc(&p, want);
  cudaThreadExchangeStreamCaptureMode(&mode);
  if (rc != cudaSuccess) {
    cudaGetLastError();  // leave no sticky error for the caller's next check
    return nullptr;
  }
  if (e.first) kept.push_back(e.first);
  e = {p, want};
  return p;
}

extern "C" {

int32_t strata_b200_quant_w4g32(const float* w, int64_t n, int64_t k, uint8_t* packed,
                                uint16_t* scale_bf16, void* stream) {
  return launch_quant_w4g32(w, n, k, packed, scale_bf16, S(stream));
}

int32_t strata_b200_quant_w8pc(const float* w, int64_t n, int64_t k, int8_t* q, float* scale,
                               void* stream) {
  return launch_quant_w8pc(w, n, k, q, scale, S(stream));
}

int32_t strata_b200_dequant_w4g32(const uint8_t* packed, const uint16_t* scale_bf16, int64_t n,
                                  int64_t k, float* w, void* stream) {
  return launch_dequant_w4g32(packed, scale_bf16, n, k, w, S(stream));
}

int32_t strata_b200_dequant_w8pc(const int8_t* q, const float* scale, int64_t n, int64_t k,
                                 float* w, void* stream) {
  return launch_dequant_w8pc(q, scale, n, k, w, S(stream));
}

static int32_t linear_common(WFormat fmt, const uint16_t* x, int64_t m, int64_t k, const void* w,
                             const void* s, int64_t n, const uint16_t* residual, uint16_t* y,
                             void* stream) {
  if (m < 0 || k <= 0 || n < 0 || m > INT32_MAX || k > INT32_MAX || n > INT32_MAX)
    return SB_INVALID_ARGUMENT;
  LinearBatch b{};
  b.x = x;
  b.m = int(m);
  b.k = int(k);
  b.fmt = fmt;
  b.epi = residual ? Epilogue::Residual : Epilogue::None;
  b.njobs = 1;
  b.jobs[0] = LinearJob{w, s, int(n), y, int(n), residual, int(n)};
  if (m > kGemvMaxRows && gemm_tc_supported(m, n, k, x, w)) {
    // Prefill-sized batches: tcgen05 GEMM over bf16 weights.  Quantized
    // weights are first expanded into the stream's cached scratch (int8: the
    // exact codes, scaled per channel in the GEMM epilogue; int4: code * group
    // scale rounded to bf16; MX: code * 2^(e - 127), exact).
    const cudaStream_t st = S(stream);
    if (fmt == WFormat::BF16)
      return launch_gemm_tc_bf16(x, m, k, static_cast<const uint16_t*>(w), n, nullptr, residual, n, y, n, nullptr,
                                 st);
    void* tmp = linear_scratch(st, size_t(n) * size_t(k) * 2);
    if (!tmp) return SB_RESOURCE_EXHAUSTED;
    const int cf = fmt == WFormat::W8PC ? 1 : fmt == WFormat::MXFP8 ? 2 : fmt == WFormat::MXFP4 ? 3 : 0;
    int rc = launch_codes_to_bf16(w, s, cf, n, k, static_cast<uint16_t*>(tmp), st);
    if (rc == SB_OK)
      rc = launch_gemm_tc_bf16(x, m, k, static_cast<const uint16_t*>(tmp), n,
                               fmt == WFormat::W8PC ? static_cast<const float*>(s) : nullptr, residual, n, y, n,
                               nullptr, st);
    return rc;
  }
  GemvMmaArgs ga{};
  ga.lb = b;
  ga.mode = GemvMode::Plain;
  ga.pdl = pdl_enabled();
  if (gemv_mma_supported(ga)) return launch_gemv_mma(ga, S(stream));
  return launch_linear(b, S(stream));
}

int32_t strata_b200_linear_bf16(const uint16_t* x, int64_t m, int64_t k, const uint16_t* w, int64_t n,
                                const uint16_t* residual, uint16_t* y, void* stream) {
  return linear_common(WFormat::BF16, x, m, k, w, nullptr, n, residual, y, stream);
}

int32_t strata_b200_linear_w4g32(const uint16_t* x, int64_t m, int64_t k, const uint8_t* packed,
                                 const uint16_t* scale_bf16, int64_t n, const uint16_t* residual,
                                 uint16_t* y, void* stream) {
  return linear_common(WFormat::W4G32, x, m, k, packed, scale_bf16, n, residual, y, stream);
}

int32_t strata_b200_linear_w8pc(const uint16_t* x, int64_t m, int64_t k, const int8_t* q,
                                const float* scale, int64_t n, const uint16_t* residual,
                                uint16_t* y, void* stream) {
  return linear_common(WFormat::W8PC, x, m, k, q, scale, n, residual, y, stream);
}

int32_t strata_b200_linear_mxfp8(const uint16_t* x, int64_t m, int64_t k, const uint8_t* codes,
                                 const uint8_t* scale_e8m0, int64_t n, const uint16_t* residual, uint16_t* y,
                                 void* stream) {
  return linear_common(WFormat::MXFP8, x, m, k, codes, scale_e8m0, n, residual, y, stream);
}

int32_t strata_b200_linear_mxfp4(const uint16_t* x, int64_t m, int64_t k, const uint8_t* codes,
                                 const uint8_t* scale_e8m0, int64_t n, const uint16_t* residual, uint16_t* y,
                                 void* stream) {
  return linear_common(WFormat::MXFP4, x, m, k, codes, scale_e8m0, n, residual, y, stream);
}

int32_t strata_b200_rms_norm_bf16(const uint16_t* x, const uint16_t* gamma, int64_t rows,
                                  int64_t cols, float eps, uint16_t* y, void* stream) {
  return launch_rms_norm<uint16_t>(x, gamma, rows, cols, eps, y, S(stream));
}

int32_t strata_b200_rope_bf16(const uint16_t* x, const int32_t* pos, int64_t rows, int64_t heads,
                              int64_t head_dim, float theta, uint16_t* y, void* stream) {
  return launch_rope<uint16_t>(x, pos, rows, heads, head_dim, double(theta), y, S(stream));
}

int32_t strata_b200_swiglu_bf16(const uint16_t* gate, const uint16_t* up, int64_t n, uint16_t* y,
                                void* stream) {
  return launch_swiglu<uint16_t>(gate, up, n, y, S(stream));
}

uint64_t strata_b200_attention_decode_scratch_bytes(int64_t batch, int64_t heads,
                                                    int64_t head_dim, int64_t max_len) {
  // The split count depends on the kv-head count only through the grid size;
  // size for the worst case (one kv head per query head).
  const uint64_t splits64 = uint64_t((max_len + 63) / 64);  // the most splits any kv-head count uses
  return uint64_t(batch) * heads * splits64 * (head_dim + 2) * sizeof(float);
}

int32_t strata_b200_attention_decode_bf16(const uint16_t* q, const uint16_t* k_new,
                                          const uint16_t* v_new, uint16_t* k_cache,
                                          uint16_t* v_cache, const int32_t* pos, int64_t batch,
                                          int64_t heads, int64_t kv_heads, int64_t head_dim,
                                          int64_t max_len, void* scratch, uint16_t* out,
                                          void* stream) {
  int rc = launch_kv_append<uint16_t>(k_new, v_new, k_cache, v_cache, pos, batch, 1, kv_heads,
                                      head_dim, max_len, nullptr, S(stream));
  if (rc) return rc;
  return launch_attention_v2(q, k_cache, v_cache, pos, batch, 1, heads, kv_heads, head_dim, max_len,
                             true, static_cast<float*>(scratch), out, nullptr, S(stream));
}

int32_t strata_b200_embed_bf16(const int32_t* ids, int64_t rows, const uint16_t* table,
                               int64_t vocab, int64_t dim, uint16_t* out, void* stream) {
  return launch_embed<uint16_t>(ids, rows, table, vocab, dim, out, nullptr, S(stream));
}

int32_t strata_b200_argmax_bf16(const uint16_t* x, int64_t rows, int64_t cols, int32_t* out,
                                void* stream) {
  return launch_argmax<uint16_t>(x, rows, cols, out, S(stream));
}

}  // extern "C"
