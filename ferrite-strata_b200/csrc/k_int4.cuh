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

// ---- MX weights (E8M0 block scales; FP8 E4M3 and FP4 E2M1 codes) ---------

// The E4M3 codes in bytes (0, 2) / (1, 3) of u as bf16 pairs holding each
// code's value times 2^-120: the bf16 exponent and mantissa fields take the
// code's bits unchanged (bias 127 against 7), so the map is exact for every
// finite code, subnormal codes included (they become bf16 subnormals).
__device__ __forceinline__ uint32_t e4m3_pair02(uint32_t u) {
  return ((u << 4) & 0x07F007F0u) | ((u << 8) & 0x80008000u);
}
__device__ __forceinline__ uint32_t e4m3_pair13(uint32_t u) {
  return ((u >> 4) & 0x07F007F0u) | (u & 0x80008000u);
}

// The eight E2M1 codes of u (code i in bits 4i..4i+3) as four bf16 pairs
// (codes 2j, 2j + 1), each holding twice the code's value: 2|v| is one of
// 0, 1, 2, 3, 4, 6, 8, 12, all normal bf16 integers, looked up by permute
// from the low (L) and high (H) bytes of their bf16 patterns; the sign bits
// are moved onto the pairs' sign positions by one more permute each.
__device__ __forceinline__ void e2m1_pairs(uint32_t u, uint32_t (&pr)[4]) {
  constexpr uint32_t kL0 = 0x40008000u, kL1 = 0x4000C080u;  // low bytes of bf16(0, 1, 2, 3 | 4, 6, 8, 12)
  constexpr uint32_t kH0 = 0x40403F00u, kH1 = 0x41414040u;  // high bytes
  const uint32_t m = u & 0x77777777u, m2 = m >> 16;
  const uint32_t l0 = prmt(kL0, kL1, m), h0 = prmt(kH0, kH1, m);
  const uint32_t l1 = prmt(kL0, kL1, m2), h1 = prmt(kH0, kH1, m2);
  const uint32_t u4 = u << 4;  // byte b, bit 7: the sign of code 2b (u itself: of code 2b + 1)
  pr[0] = prmt(l0, h0, 0x5140) ^ (prmt(u4, u, 0x4000) & 0x80008000u);
  pr[1] = prmt(l0, h0, 0x7362) ^ (prmt(u4, u, 0x5010) & 0x80008000u);
  pr[2] = prmt(l1, h1, 0x5140) ^ (prmt(u4, u, 0x6020) & 0x80008000u);
  pr[3] = prmt(l1, h1, 0x7362) ^ (prmt(u4, u, 0x7030) & 0x80008000u);
}

// 2^(e - 127 - adj) for an E8M0 code e, or 0 where that is below f32's
// normal range (a block scale of 2^-126 or less: its codes contribute less
// than 6 * 2^-126 each).
__device__ __forceinline__ float e8m0_scale(uint32_t e, int adj) {
  const int x = int(e) - adj;
  return x >= 1 ? __uint_as_float(uint32_t(x) << 23) : 0.0f;
}

// Exact f32 values of MX codes and scales (for the bf16 weight expansion).
__device__ __forceinline__ float e4m3_f32(uint32_t c) {
  const uint32_t e = (c >> 3) & 15u, m = c & 7u;
  float v = e ? __uint_as_float(((e + 120u) << 23) | (m << 20)) : float(m) * 0x1p-9f;
  if ((c & 0x7Fu) == 0x7Fu) v = __int_as_float(0x7FC00000);
  return (c & 0x80u) ? -v : v;
}
__device__ __forceinline__ float e2m1_f32(uint32_t c) {
  const uint32_t e = (c >> 1) & 3u, m = c & 1u;
  const float v = e ? __uint_as_float(((e + 126u) << 23) | (m << 22)) : float(m) * 0.5f;
  return (c & 8u) ? -v : v;
}
__device__ __forceinline__ float e8m0_f32(uint32_t s) {
  if (s == 255u) return __int_as_float(0x7FC00000);
  return s ? __uint_as_float(s << 23) : 0x1p-127f;
}

__device__ __forceinline__ float int8_code(uint32_t u, int j) {
  return __uint_as_float(((u >> (8 * j)) & 0xFFu) | 0x4B000000u) - 8388736.0f;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

}  // namespace sb
