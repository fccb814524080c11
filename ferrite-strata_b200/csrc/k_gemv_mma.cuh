// Tensor-core GEMV for decode-sized batches.
#pragma once

#include "k_linear.cuh"

namespace sb {

enum class GemvMode : int {
  Plain = 0,       // jobs stacked along output rows; optional residual per job
  SwiGLU = 1,      // jobs[0] = gate, jobs[1] = up; y = silu(gate) * up
  QkvRope = 2,     // jobs q, k, v: rope on q and k, k/v appended into the caches
};

struct QkvExtra {
  const int32_t* pos;      // [M]
  uint16_t* q_out;         // [M, Hq * hd] (roped q)
  uint16_t* k_out;         // optional [M, Hkv * hd] (roped k), may be null
  uint16_t* v_out;         // optional [M, Hkv * hd], may be null
  uint16_t* k_cache;       // [B, Hkv, L, hd], or page pools [pages, Hkv, page_size, hd] with kp's table
  uint16_t* v_cache;
  int hq, hkv, head_dim, max_len, tokens_per_seq;
  double theta;
  int* err;
  KvPages kp;
  const double* inv_freq;  // [head_dim / 2] theta^(-2j/d), or null: computed with pow
};

struct GemvMmaArgs {
  LinearBatch lb;  // x, m, k, fmt, jobs (w, s, n, y, residual)
  GemvMode mode;
  QkvExtra qkv;
  bool pdl;        // launch with programmatic dependent launch
};

// Whether the tensor-core path takes this batch (else the CUDA-core GEMV).
bool gemv_mma_supported(const GemvMmaArgs& a);
int launch_gemv_mma(const GemvMmaArgs& a, cudaStream_t st);


}  // namespace sb
