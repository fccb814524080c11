// Quantised Linear: job descriptors shared by the launchers and the executor.
#pragma once

#include "common.cuh"

namespace sb {

// MXFP8: E4M3 codes [N, K]; MXFP4: E2M1 codes packed two per byte [N, K/2];
// both with one E8M0 scale byte per row and group of 32 along K.
enum class WFormat : int { W4G32 = 0, W8PC = 1, BF16 = 2, MXFP8 = 3, MXFP4 = 4 };
enum class Epilogue : int { None = 0, Residual = 1, SwiGLU = 2 };

// One weight matrix applied to the shared activation x[M, K].
struct LinearJob {
  const void* w;        // int4 packed [N, K/2] u8, int8 [N, K], or bf16 [N, K]
  const void* s;        // bf16 [N, K/32] (w4g32), f32 [N] (w8pc), unused (bf16)
  int n;                // output features
  uint16_t* y;          // bf16 [M, ldy]
  int ldy;
  const uint16_t* residual;  // bf16 [M, ldr] added in the epilogue, or null
  int ldr;
};

constexpr int kMaxJobs = 3;

struct LinearBatch {
  const uint16_t* x;  // bf16 [M, K], row stride k
  int m, k;
  WFormat fmt;
  Epilogue epi;       // SwiGLU: jobs[0] = gate, jobs[1] = up, output in jobs[0].y
  int njobs;
  LinearJob jobs[kMaxJobs];
};

int launch_linear(const LinearBatch& b, cudaStream_t st);

}  // namespace sb
