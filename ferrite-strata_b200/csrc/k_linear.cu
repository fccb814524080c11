// Weight-quantised Linear for decode-sized batches (HBM-bound GEMV).
//
// y[m, n] = sum_k x[m, k] * deq(W)[n, k], f32 accumulation, bf16 out.
//
// Design: each warp owns two output rows and streams them along k in 16-byte
// chunks (one chunk = one int4 group of 32 codes, or 16 int8 codes), using
// 128-bit non-allocating loads so the weights stream past L1.  Codes are
// dequantised in registers with the exponent trick (code + 2^23 as an f32 bit
// pattern, minus the bias), multiplied against the activations (small, L1/L2
// resident), scaled once per group, and reduced across the warp with
// shuffles.  Several matrices that share x run in one launch (q/k/v, or
// gate/up), and the epilogue can add a residual or apply SwiGLU to a
// gate/up pair without writing the intermediate to HBM.
#include "k_linear.cuh"

namespace sb {

namespace {

template <WFormat F>
struct Fmt;

template <>
struct Fmt<WFormat::W4G32> {
  static constexpr int kPerChunk = 32;  // codes per 16-byte chunk
  static __device__ __forceinline__ int64_t row_bytes(int k) { return k / 2; }
};
template <>
struct Fmt<WFormat::W8PC> {
  static constexpr int kPerChunk = 16;
  static __device__ __forceinline__ int64_t row_bytes(int k) { return k; }
};
template <>
struct Fmt<WFormat::BF16> {
  static constexpr int kPerChunk = 8;
  static __device__ __forceinline__ int64_t row_bytes(int k) { return int64_t(k) * 2; }
};

// 8 int4 codes of one 32-bit word -> f32, in k order (nibble i = k offset i).
__device__ __forceinline__ void dq_int4_word(uint32_t w, float (&q)[8]) {
  const uint32_t u = w ^ 0x88888888u;  // each nibble becomes code + 8
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const uint32_t bits = ((u >> (4 * i)) & 0xfu) | 0x4b000000u;  // 2^23 + code + 8
    q[i] = __uint_as_float(bits) - 8388616.0f;
  }
}

// 4 int8 codes of one 32-bit word -> f32, byte j = k offset j.
__device__ __forceinline__ void dq_int8_word(uint32_t w, float (&q)[4]) {
  const uint32_t u = w ^ 0x80808080u;  // each byte becomes code + 128
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const uint32_t bits = ((u >> (8 * j)) & 0xffu) | 0x4b000000u;
    q[j] = __uint_as_float(bits) - 8388736.0f;
  }
}

// All codes of one 16-byte weight chunk as f32, in k order.
template <WFormat F>
__device__ __forceinline__ void dequant_chunk(const uint4& w, float (&q)[Fmt<F>::kPerChunk]) {
  const uint32_t ws[4] = {w.x, w.y, w.z, w.w};
  if constexpr (F == WFormat::W4G32) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float t[8];
      dq_int4_word(ws[j], t);
#pragma unroll
      for (int i = 0; i < 8; ++i) q[8 * j + i] = t[i];
    }
  } else if constexpr (F == WFormat::W8PC) {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      float t[4];
      dq_int8_word(ws[j], t);
#pragma unroll
      for (int i = 0; i < 4; ++i) q[4 * j + i] = t[i];
    }
  } else {
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      q[2 * j] = bf_lo(ws[j]);
      q[2 * j + 1] = bf_hi(ws[j]);
    }
  }
}

// sum_e qa[e] * x[e] and sum_e qb[e] * x[e] over one chunk of activations.
template <int E>
__device__ __forceinline__ void chunk_dot2(const float (&qa)[E], const float (&qb)[E],
                                           const uint16_t* __restrict__ xr, float& da,
                                           float& db) {
  float a = 0.0f, b = 0.0f;
#pragma unroll
  for (int v = 0; v < E / 8; ++v) {
    const uint4 xv = ldg16(xr + 8 * v);
    const uint32_t xs[4] = {xv.x, xv.y, xv.z, xv.w};
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float x0 = bf_lo(xs[i]), x1 = bf_hi(xs[i]);
      a = fmaf(qa[8 * v + 2 * i], x0, a);
      a = fmaf(qa[8 * v + 2 * i + 1], x1, a);
      b = fmaf(qb[8 * v + 2 * i], x0, b);
      b = fmaf(qb[8 * v + 2 * i + 1], x1, b);
    }
  }
  da = a;
  db = b;
}

template <WFormat F>
__device__ __forceinline__ float group_scale(const void* s, int64_t row, int k, int chunk) {
  if constexpr (F == WFormat::W4G32) {
    return bf2f(reinterpret_cast<const uint16_t*>(s)[row * (k / 32) + chunk]);
  } else {
    return 1.0f;
  }
}

constexpr int kWarps = 8;
constexpr int kUnroll = 4;

// Each warp computes rows (ja, ra) and (jb, rb) for m in [m0, m0 + MT).
template <WFormat F, int MT>
__global__ void __launch_bounds__(kWarps * 32)
    gemv_kernel(const LinearBatch b, int units, int m0) {
  pdl_trigger();
  pdl_wait();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int unit = blockIdx.x * kWarps + warp;
  if (unit >= units) return;

  int ja = 0, ra = 0, jb = 0, rb = 0;
  if (b.epi == Epilogue::SwiGLU) {
    ja = 0, jb = 1, ra = rb = unit;
  } else {
    int u = unit;
    int j = 0;
    while (j + 1 < b.njobs && u >= b.jobs[j].n / 2) u -= b.jobs[j++].n / 2;
    ja = jb = j;
    ra = 2 * u, rb = 2 * u + 1;
  }
  const LinearJob& A = b.jobs[ja];
  const LinearJob& B = b.jobs[jb];
  const int k = b.k;
  const int64_t rbytes = Fmt<F>::row_bytes(k);
  const uint8_t* wa = reinterpret_cast<const uint8_t*>(A.w) + int64_t(ra) * rbytes;
  const uint8_t* wb = reinterpret_cast<const uint8_t*>(B.w) + int64_t(rb) * rbytes;
  const int nchunks = k / Fmt<F>::kPerChunk;
  const int mcount = min(MT, b.m - m0);

  float acc_a[MT], acc_b[MT];
#pragma unroll
  for (int m = 0; m < MT; ++m) acc_a[m] = acc_b[m] = 0.0f;

  for (int c0 = 0; c0 < nchunks; c0 += 32 * kUnroll) {
    uint4 wva[kUnroll], wvb[kUnroll];
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < nchunks) {
        wva[u] = ldg_stream(wa + int64_t(c) * 16);
        wvb[u] = ldg_stream(wb + int64_t(c) * 16);
      }
    }
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int c = c0 + u * 32 + lane;
      if (c < nchunks) {
        const float sa = group_scale<F>(A.s, ra, k, c);
        const float sb_ = group_scale<F>(B.s, rb, k, c);
        float qa[Fmt<F>::kPerChunk], qb[Fmt<F>::kPerChunk];
        dequant_chunk<F>(wva[u], qa);
        dequant_chunk<F>(wvb[u], qb);
#pragma unroll
        for (int m = 0; m < MT; ++m) {
          if (m < mcount) {
            const uint16_t* xr = b.x + int64_t(m0 + m) * k + int64_t(c) * Fmt<F>::kPerChunk;
            float da, db;
            chunk_dot2<Fmt<F>::kPerChunk>(qa, qb, xr, da, db);
            acc_a[m] = fmaf(da, sa, acc_a[m]);
            acc_b[m] = fmaf(db, sb_, acc_b[m]);
          }
        }
      }
    }
  }

#pragma unroll
  for (int m = 0; m < MT; ++m) {
    acc_a[m] = warp_sum(acc_a[m]);
    acc_b[m] = warp_sum(acc_b[m]);
  }

  float sca = 1.0f, scb = 1.0f;
  if constexpr (F == WFormat::W8PC) {
    sca = reinterpret_cast<const float*>(A.s)[ra];
    scb = reinterpret_cast<const float*>(B.s)[rb];
  }
  if (lane < mcount) {
    // Lane m writes row m (registers are indexed statically, so select).
    float va = 0.0f, vb = 0.0f;
#pragma unroll
    for (int m = 0; m < MT; ++m)
      if (m == lane) va = acc_a[m], vb = acc_b[m];
    va *= sca;
    vb *= scb;
    const int64_t mrow = m0 + lane;
    if (b.epi == Epilogue::SwiGLU) {
      const float g = va, up = vb;
      const float silu = g / (1.0f + expf(-g));
      A.y[mrow * A.ldy + ra] = f2bf(silu * up);
    } else {
      if (A.residual) {
        va += bf2f(A.residual[mrow * A.ldr + ra]);
        vb += bf2f(A.residual[mrow * A.ldr + rb]);
      }
      A.y[mrow * A.ldy + ra] = f2bf(va);
      A.y[mrow * A.ldy + rb] = f2bf(vb);
    }
  }
}

template <WFormat F>
int launch_fmt(const LinearBatch& b, cudaStream_t st) {
  int units = 0;
  if (b.epi == Epilogue::SwiGLU) {
    units = b.jobs[0].n;
  } else {
    for (int j = 0; j < b.njobs; ++j) units += b.jobs[j].n / 2;
  }
  if (units == 0 || b.m == 0) return SB_OK;
  const int blocks = ceil_div(units, kWarps);
  for (int m0 = 0; m0 < b.m; m0 += 8) {
    const int left = b.m - m0;
    if (left >= 8) {
      launch_pdl(gemv_kernel<F, 8>, dim3(blocks), dim3(kWarps * 32), 0, st, b, units, m0);
    } else if (left > 2) {
      launch_pdl(gemv_kernel<F, 4>, dim3(blocks), dim3(kWarps * 32), 0, st, b, units, m0);
      if (left > 4) {
        launch_pdl(gemv_kernel<F, 4>, dim3(blocks), dim3(kWarps * 32), 0, st, b, units, m0 + 4);
        SB_LAUNCH_CHECK();
      }
    } else if (left == 2) {
      launch_pdl(gemv_kernel<F, 2>, dim3(blocks), dim3(kWarps * 32), 0, st, b, units, m0);
    } else {
      launch_pdl(gemv_kernel<F, 1>, dim3(blocks), dim3(kWarps * 32), 0, st, b, units, m0);
    }
    SB_LAUNCH_CHECK();
  }
  return SB_OK;
}

}  // namespace

int launch_linear(const LinearBatch& b, cudaStream_t st) {
  if (b.m < 0 || b.k <= 0 || b.njobs < 1 || b.njobs > kMaxJobs) return SB_INVALID_ARGUMENT;
  const int per_chunk = b.fmt == WFormat::W4G32 ? 32 : (b.fmt == WFormat::W8PC ? 16 : 8);
  if (b.k % per_chunk) return SB_INVALID_ARGUMENT;
  if (b.epi == Epilogue::SwiGLU && (b.njobs != 2 || b.jobs[0].n != b.jobs[1].n))
    return SB_INVALID_ARGUMENT;
  for (int j = 0; j < b.njobs; ++j) {
    if (b.jobs[j].n < 0) return SB_INVALID_ARGUMENT;
    if (b.epi != Epilogue::SwiGLU && (b.jobs[j].n % 2)) return SB_INVALID_ARGUMENT;
    if (b.epi == Epilogue::SwiGLU && j == 1) break;
    if (b.jobs[j].y == nullptr) return SB_INVALID_ARGUMENT;
  }
  // 16-byte alignment of every streamed row is required by the vector loads.
  auto misaligned = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) != 0; };
  if (misaligned(b.x)) return SB_INVALID_ARGUMENT;
  for (int j = 0; j < b.njobs; ++j)
    if (misaligned(b.jobs[j].w)) return SB_INVALID_ARGUMENT;
  switch (b.fmt) {
    case WFormat::W4G32: return launch_fmt<WFormat::W4G32>(b, st);
    case WFormat::W8PC: return launch_fmt<WFormat::W8PC>(b, st);
    case WFormat::BF16: return launch_fmt<WFormat::BF16>(b, st);
    default: break;  // MX weights run on the tensor-core GEMV only
  }
  return SB_INVALID_ARGUMENT;
}

}  // namespace sb
