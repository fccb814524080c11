// Register-level helpers shared by the tensor-core GEMV kernels: the
// mma.sync m16n8k16 bf16 contraction and the int4 / int8 code-to-bf16
// conversions that feed its A fragments.
#pragma once

#include "common.cuh"

namespace sb {

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// a * 1 - 136 on both bf16 halves (exact: a is 136 + code).
__device__ __forceinline__ uint32_t bf16x2_minus136(uint32_t a) {
  uint32_t r;
  asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(0x3F803F80u), "r"(0xC308C308u));
  return r;
}

// Nibbles j and j + 4 of the raw code word u as the bf16 pair (code_j,
// code_j+4).  One lop3 computes (a & 0x000F000F) ^ 0x43084308: it keeps the
// two nibbles, flips their sign bits (two's-complement c becomes c + 8) and
// sets the exponent of bf16 128, giving 136 + c; the fma removes the 136.
// The right shift is a high multiply so that it issues on the FMA pipe, which
// leaves the ALU pipe (the busiest in this loop) to the lop3 and permutes.
__device__ __forceinline__ uint32_t int4_pair(uint32_t u, int j) {
  uint32_t a = u, v;
  if (j) asm("mul.hi.u32 %0, %1, %2;" : "=r"(a) : "r"(u), "r"(1u << (32 - 4 * j)));
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(v) : "r"(a), "r"(0x000F000Fu), "r"(0x43084308u));
  return bf16x2_minus136(v);
}

__device__ __forceinline__ float int8_code(uint32_t u, int j) {
  return __uint_as_float(((u >> (8 * j)) & 0xFFu) | 0x4B000000u) - 8388736.0f;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

}  // namespace sb
