// Row-wise and elementwise kernels: RMSNorm, RoPE, SwiGLU, broadcast add/mul,
// unary maps, softmax, LayerNorm, transpose/slice/broadcast copies, embedding
// gather, argmax, and the small f32 contractions the reference's own op set
// needs (Linear, MatMul).  Templated on the element type: f32 or bf16 (stored
// as uint16_t), always computing in f32.
#include "k_elem.cuh"

namespace sb {

namespace {

template <typename T>
__device__ __forceinline__ float ld(const T* p, int64_t i);
template <>
__device__ __forceinline__ float ld<float>(const float* p, int64_t i) { return p[i]; }
template <>
__device__ __forceinline__ float ld<uint16_t>(const uint16_t* p, int64_t i) { return bf2f(p[i]); }

template <typename T>
__device__ __forceinline__ void st(T* p, int64_t i, float v);
template <>
__device__ __forceinline__ void st<float>(float* p, int64_t i, float v) { p[i] = v; }
template <>
__device__ __forceinline__ void st<uint16_t>(uint16_t* p, int64_t i, float v) { p[i] = f2bf(v); }

// Block-wide sum for blockDim.x <= 1024; all threads get the result.
__device__ float block_sum(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_sum(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = lane < nw ? red[lane] : 0.0f;
  return warp_sum(t);
}

__device__ float block_max(float v, float* red) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  v = warp_max(v);
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  const int nw = (blockDim.x + 31) >> 5;
  float t = lane < nw ? red[lane] : -INFINITY;
  return warp_max(t);
}

// g_ready: gamma is not written by the kernels this one depends on (a graph
// input), so it is read before griddepcontrol.wait and arrives while the
// previous kernel finishes.
template <typename T>
__global__ void rms_norm_kernel(const T* __restrict__ x, const T* __restrict__ g, int64_t cols,
                                float eps, T* __restrict__ y, int g_ready) {
  pdl_trigger();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * cols;
  if constexpr (sizeof(T) == 2) {
    // bf16 rows of up to blockDim * 32 columns: the row stays in registers as
    // 16-byte chunks (read once), gamma is read in 16-byte chunks.
    constexpr int kMax = 4;  // chunks per thread
    const int64_t chunks = cols / 8;
    if (cols % 8 == 0 && chunks <= int64_t(kMax) * blockDim.x &&
        ((reinterpret_cast<uintptr_t>(xr) | reinterpret_cast<uintptr_t>(g) | reinterpret_cast<uintptr_t>(y)) & 15) ==
            0) {
      uint4 gv[kMax];
#pragma unroll
      for (int u = 0; u < kMax; ++u) {
        const int64_t c = threadIdx.x + int64_t(u) * blockDim.x;
        gv[u] = g_ready && c < chunks ? __ldg(reinterpret_cast<const uint4*>(g) + c) : make_uint4(0, 0, 0, 0);
      }
      pdl_wait();
      uint4 v[kMax];
      float ss = 0.0f;
#pragma unroll
      for (int u = 0; u < kMax; ++u) {
        const int64_t c = threadIdx.x + int64_t(u) * blockDim.x;
        v[u] = c < chunks ? __ldg(reinterpret_cast<const uint4*>(xr) + c) : make_uint4(0, 0, 0, 0);
        const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          ss = fmaf(bf_lo(w[e]), bf_lo(w[e]), ss);
          ss = fmaf(bf_hi(w[e]), bf_hi(w[e]), ss);
        }
      }
      ss = block_sum(ss, red);
      const float inv = 1.0f / sqrtf(ss / float(cols) + eps);
#pragma unroll
      for (int u = 0; u < kMax; ++u) {
        const int64_t c = threadIdx.x + int64_t(u) * blockDim.x;
        if (c < chunks) {
          const uint4 g4 = g_ready ? gv[u] : __ldg(reinterpret_cast<const uint4*>(g) + c);
          const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w}, gw[4] = {g4.x, g4.y, g4.z, g4.w};
          uint32_t o[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            o[e] = uint32_t(f2bf((bf_lo(w[e]) * inv) * bf_lo(gw[e]))) |
                   (uint32_t(f2bf((bf_hi(w[e]) * inv) * bf_hi(gw[e]))) << 16);
          reinterpret_cast<uint4*>(y + row * cols)[c] = make_uint4(o[0], o[1], o[2], o[3]);
        }
      }
      return;
    }
  }
  pdl_wait();
  float ss = 0.0f;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    const float v = ld(xr, c);
    ss = fmaf(v, v, ss);
  }
  ss = block_sum(ss, red);
  const float inv = 1.0f / sqrtf(ss / float(cols) + eps);
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x)
    st(y, row * cols + c, (ld(xr, c) * inv) * ld(g, c));
}

// Rotate-half RoPE; angles in double, as the oracle computes them.
constexpr int kRopeRows = 4;  // rows whose cos/sin tables one pass computes (fewer for huge head_dim)

template <typename T>
__global__ void rope_kernel(const T* __restrict__ x, const int32_t* __restrict__ pos, int64_t rows,
                            int heads, int head_dim, double theta, T* __restrict__ y, int nr,
                            const double* __restrict__ inv_freq) {
  pdl_trigger();
  // The inverse frequencies theta^(-2j/d) (from the executable's host-computed
  // table, else pow in double) do not depend on the previous kernel: once per
  // block, before the wait.  Then nr rows at a time: every thread computes one
  // (row, j) angle's cos/sin (rope_cos_sin: reduced in double, evaluated in
  // f32), and the rows' heads are rotated in f32 (B200's FP64 pipe would
  // bound double arithmetic here; the f32 results differ from the oracle's
  // double ones by about 2^-24 relative, far inside bf16 output precision).
  extern __shared__ double sh[];  // inv[half], then cs[nr][2][half] as f32
  const int half = head_dim / 2;
  double* inv = sh;
  float* cs = reinterpret_cast<float*>(sh + half);
  for (int j = threadIdx.x; j < half; j += blockDim.x)
    inv[j] = inv_freq ? inv_freq[j] : pow(theta, -2.0 * double(j) / double(head_dim));
  pdl_wait();
  const int per_row = heads * half;
  const bool vec8 = sizeof(T) == 2 && half % 8 == 0 &&
                    ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
  for (int64_t row0 = int64_t(blockIdx.x) * nr; row0 < rows; row0 += int64_t(gridDim.x) * nr) {
    __syncthreads();  // inv is written; the previous rows' table is no longer read
    for (int t = threadIdx.x; t < nr * half; t += blockDim.x) {
      const int r = t / half, j = t - r * half;
      if (row0 + r < rows) rope_cos_sin(pos[row0 + r], inv[j], cs[(2 * r) * half + j], cs[(2 * r + 1) * half + j]);
    }
    __syncthreads();
    if (vec8) {
      // bf16 rows with half a multiple of 8: 8 pairs per step, as two 16-byte
      // loads and two 16-byte stores, so each thread has whole lines in flight.
      const int per_head = half / 8, units = heads * per_head;
      for (int t = threadIdx.x; t < nr * units; t += blockDim.x) {
        const int r = t / units, u = t - r * units;
        if (row0 + r >= rows) break;
        const int h = u / per_head, j0 = (u - h * per_head) * 8;
        const int64_t b = (row0 + r) * int64_t(heads) * head_dim + int64_t(h) * head_dim + j0;
        const uint4 a = *reinterpret_cast<const uint4*>(x + b), bb = *reinterpret_cast<const uint4*>(x + b + half);
        const uint32_t aw[4] = {a.x, a.y, a.z, a.w}, bw[4] = {bb.x, bb.y, bb.z, bb.w};
        const float* cr = cs + (2 * r) * half + j0;
        const float* sr = cs + (2 * r + 1) * half + j0;
        uint32_t lo[4], hi[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float x1a = bf_lo(aw[e]), x1b = bf_hi(aw[e]), x2a = bf_lo(bw[e]), x2b = bf_hi(bw[e]);
          const float ca = cr[2 * e], cb = cr[2 * e + 1], sa = sr[2 * e], sb2 = sr[2 * e + 1];
          lo[e] = pack_bf2(fmaf(x1a, ca, -x2a * sa), fmaf(x1b, cb, -x2b * sb2));
          hi[e] = pack_bf2(fmaf(x2a, ca, x1a * sa), fmaf(x2b, cb, x1b * sb2));
        }
        *reinterpret_cast<uint4*>(y + b) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        *reinterpret_cast<uint4*>(y + b + half) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
      }
      continue;
    }
    for (int t = threadIdx.x; t < nr * per_row; t += blockDim.x) {
      const int r = t / per_row, i = t - r * per_row;
      if (row0 + r >= rows) break;
      const int h = i / half, j = i - h * half;
      const int64_t b = (row0 + r) * int64_t(heads) * head_dim + int64_t(h) * head_dim;
      const float x1 = ld(x, b + j), x2 = ld(x, b + j + half);
      const float c = cs[(2 * r) * half + j], sn = cs[(2 * r + 1) * half + j];
      st(y, b + j, fmaf(x1, c, -x2 * sn));
      st(y, b + j + half, fmaf(x2, c, x1 * sn));
    }
  }
}

template <typename T>
__global__ void swiglu_kernel(const T* __restrict__ gate, const T* __restrict__ up, int64_t n,
                              T* __restrict__ y) {
  pdl_trigger();
  pdl_wait();
  int64_t start = 0;
  if constexpr (sizeof(T) == 2) {
    // Eight bf16 per 16-byte load when all three arrays are 16-byte aligned.
    if (((reinterpret_cast<uintptr_t>(gate) | reinterpret_cast<uintptr_t>(up) | reinterpret_cast<uintptr_t>(y)) &
         15) == 0) {
      const int64_t n8 = n / 8;
      for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n8; i += int64_t(gridDim.x) * blockDim.x) {
        const uint4 g4 = __ldg(reinterpret_cast<const uint4*>(gate) + i);
        const uint4 u4 = __ldg(reinterpret_cast<const uint4*>(up) + i);
        const uint32_t gw[4] = {g4.x, g4.y, g4.z, g4.w}, uw[4] = {u4.x, u4.y, u4.z, u4.w};
        uint32_t o[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const float g0 = bf_lo(gw[e]), g1 = bf_hi(gw[e]);
          const float r0 = (g0 / (1.0f + expf(-g0))) * bf_lo(uw[e]);
          const float r1 = (g1 / (1.0f + expf(-g1))) * bf_hi(uw[e]);
          o[e] = uint32_t(f2bf(r0)) | (uint32_t(f2bf(r1)) << 16);
        }
        reinterpret_cast<uint4*>(y)[i] = make_uint4(o[0], o[1], o[2], o[3]);
      }
      start = n8 * 8;
    }
  }
  for (int64_t i = start + int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x) {
    const float gv = ld(gate, i);
    st(y, i, (gv / (1.0f + expf(-gv))) * ld(up, i));
  }
}

// NumPy broadcasting through per-axis strides (0 on broadcast axes).
template <typename T>
__global__ void binary_kernel(int op, const T* __restrict__ a, const T* __restrict__ b,
                              T* __restrict__ out, BcastShape sh) {
  pdl_trigger();
  pdl_wait();
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < sh.total;
       i += int64_t(gridDim.x) * blockDim.x) {
    int64_t rem = i, ia = 0, ib = 0;
    for (int ax = sh.rank - 1; ax >= 0; --ax) {
      const int64_t idx = rem % sh.dims[ax];
      rem /= sh.dims[ax];
      ia += idx * sh.sa[ax];
      ib += idx * sh.sb[ax];
    }
    const float va = ld(a, ia), vb = ld(b, ib);
    st(out, i, op == 0 ? va + vb : va * vb);
  }
}

__device__ __forceinline__ float erf_as(float x) {
  // Abramowitz & Stegun 7.1.26, the form the reference CPU backend uses.
  const float sign = x < 0.0f ? -1.0f : 1.0f;
  const float ax = fabsf(x);
  const float t = 1.0f / (1.0f + 0.3275911f * ax);
  const float poly =
      ((((1.0614054f * t - 1.4531521f) * t) + 1.4214138f) * t - 0.28449672f) * t + 0.2548296f;
  return sign * (1.0f - poly * t * expf(-ax * ax));
}

template <typename T>
__global__ void unary_kernel(int op, const T* __restrict__ x, int64_t n, T* __restrict__ y) {
  pdl_trigger();
  pdl_wait();
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x) {
    const float v = ld(x, i);
    float r;
    if (op == 0) r = 0.5f * v * (1.0f + erf_as(v / 1.41421356237309504880f));
    else if (op == 1) r = expf(v);
    else r = logf(v);
    st(y, i, r);
  }
}

template <typename T>
__global__ void softmax_kernel(const T* __restrict__ x, int64_t cols, T* __restrict__ y) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * cols;
  float mx = -INFINITY;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) mx = fmaxf(mx, ld(xr, c));
  mx = block_max(mx, red);
  float sum = 0.0f;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) sum += expf(ld(xr, c) - mx);
  sum = block_sum(sum, red);
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x)
    st(y, row * cols + c, expf(ld(xr, c) - mx) / sum);
}

template <typename T>
__global__ void layer_norm_kernel(const T* __restrict__ x, const T* __restrict__ gamma,
                                  const T* __restrict__ beta, int64_t cols, float eps,
                                  T* __restrict__ y) {
  pdl_trigger();
  pdl_wait();
  __shared__ float red[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * cols;
  float s = 0.0f;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) s += ld(xr, c);
  const float mean = block_sum(s, red) / float(cols);
  float v = 0.0f;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    const float d = ld(xr, c) - mean;
    v = fmaf(d, d, v);
  }
  const float var = block_sum(v, red) / float(cols);
  const float den = sqrtf(var + eps);
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x)
    st(y, row * cols + c, ((ld(xr, c) - mean) / den) * ld(gamma, c) + ld(beta, c));
}

template <typename T>
__global__ void transpose2_kernel(const T* __restrict__ x, int64_t rows, int64_t cols,
                                  T* __restrict__ y) {
  pdl_trigger();
  pdl_wait();
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < rows * cols;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / cols, c = i % cols;
    y[c * rows + r] = x[i];
  }
}

template <typename T>
__global__ void slice_cols_kernel(const T* __restrict__ x, int64_t rows, int64_t cols,
                                  int64_t start, int64_t stride, int64_t out_cols,
                                  T* __restrict__ y) {
  pdl_trigger();
  pdl_wait();
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < rows * out_cols;
       i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t r = i / out_cols, j = i % out_cols;
    y[i] = x[r * cols + start + j * stride];
  }
}

template <typename T>
__global__ void broadcast_kernel(const T* __restrict__ a, T* __restrict__ out, BcastShape sh) {
  pdl_trigger();
  pdl_wait();
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < sh.total;
       i += int64_t(gridDim.x) * blockDim.x) {
    int64_t rem = i, ia = 0;
    for (int ax = sh.rank - 1; ax >= 0; --ax) {
      const int64_t idx = rem % sh.dims[ax];
      rem /= sh.dims[ax];
      ia += idx * sh.sa[ax];
    }
    out[i] = a[ia];
  }
}

template <typename T>
__global__ void embed_kernel(const int32_t* __restrict__ ids, const T* __restrict__ table,
                             int64_t vocab, int64_t dim, T* __restrict__ out, int* err) {
  pdl_trigger();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const int32_t id = ids[row];
  if (id < 0 || id >= vocab) {
    if (threadIdx.x == 0 && err) atomicExch(err, 3);
    for (int64_t c = threadIdx.x; c < dim; c += blockDim.x) out[row * dim + c] = T(0);
    return;
  }
  const T* src = table + int64_t(id) * dim;
  for (int64_t c = threadIdx.x; c < dim; c += blockDim.x) out[row * dim + c] = src[c];
}

// Lowest index among the maxima; NaN never wins; an all-NaN row gives 0.
template <typename T>
__global__ void argmax_kernel(const T* __restrict__ x, int64_t cols, int32_t* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  __shared__ float sv[32];
  __shared__ int32_t si[32];
  const int64_t row = blockIdx.x;
  const T* xr = x + row * cols;
  float bv = -INFINITY;
  int32_t bi = INT32_MAX;
  // Each thread visits its columns in increasing order and keeps the first
  // maximum (strict >); NaNs are skipped.
  auto take = [&](float v, int64_t c) {
    if (v == v && (bi == INT32_MAX || v > bv)) bv = v, bi = int32_t(c);
  };
  constexpr int kVec = 16 / int(sizeof(T));
  int64_t c0 = 0;  // first column of the scalar tail
  if ((reinterpret_cast<uintptr_t>(xr) & 15) == 0) {
    // 16-byte loads, four in flight per thread.
    const int64_t nv = cols / kVec, step = blockDim.x;
    const uint4* xv = reinterpret_cast<const uint4*>(xr);
    int64_t i = threadIdx.x;
    for (; i + 3 * step < nv; i += 4 * step) {
      uint4 a[4];
#pragma unroll
      for (int u = 0; u < 4; ++u) a[u] = __ldg(xv + i + u * step);
#pragma unroll
      for (int u = 0; u < 4; ++u) {
        const T* e = reinterpret_cast<const T*>(&a[u]);
#pragma unroll
        for (int k = 0; k < kVec; ++k) take(ld(e, k), (i + u * step) * kVec + k);
      }
    }
    for (; i < nv; i += step) {
      const uint4 a = __ldg(xv + i);
      const T* e = reinterpret_cast<const T*>(&a);
#pragma unroll
      for (int k = 0; k < kVec; ++k) take(ld(e, k), i * kVec + k);
    }
    c0 = nv * kVec;
  }
  for (int64_t c = c0 + threadIdx.x; c < cols; c += blockDim.x) take(ld(xr, c), c);
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
    const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
    if (oi != INT32_MAX && (bi == INT32_MAX || ov > bv || (ov == bv && oi < bi))) bv = ov, bi = oi;
  }
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  if (lane == 0) sv[warp] = bv, si[warp] = bi;
  __syncthreads();
  if (warp == 0) {
    const int nw = (blockDim.x + 31) >> 5;
    bv = lane < nw ? sv[lane] : -INFINITY;
    bi = lane < nw ? si[lane] : INT32_MAX;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
      const int32_t oi = __shfl_xor_sync(0xffffffffu, bi, o);
      if (oi != INT32_MAX && (bi == INT32_MAX || ov > bv || (ov == bv && oi < bi)))
        bv = ov, bi = oi;
    }
    if (lane == 0) out[row] = bi == INT32_MAX ? 0 : bi;
  }
}

// Tiled f32 GEMM for the reference's own Linear/MatMul ops (small shapes):
// C[m, n] = sum_k A[m, k] * B(k, n), B read through strides so that Linear's
// [out, in] weight and MatMul's [k, n] operand share one kernel.
constexpr int kT = 32;
__global__ void gemm_f32_kernel(const float* __restrict__ a, const float* __restrict__ b,
                                const float* __restrict__ bias, int64_t m, int64_t k, int64_t n,
                                int64_t b_sk, int64_t b_sn, float* __restrict__ c) {
  pdl_trigger();
  pdl_wait();
  __shared__ float as[kT][kT + 1];
  __shared__ float bs[kT][kT + 1];
  const int tx = threadIdx.x % kT, ty = threadIdx.x / kT;  // 32 x 8 threads
  const int64_t row0 = int64_t(blockIdx.y) * kT, col0 = int64_t(blockIdx.x) * kT;
  float acc[4] = {0.0f, 0.0f, 0.0f, 0.0f};
  for (int64_t k0 = 0; k0 < k; k0 += kT) {
    for (int r = ty; r < kT; r += 8) {
      const int64_t ar = row0 + r, ac = k0 + tx;
      as[r][tx] = (ar < m && ac < k) ? a[ar * k + ac] : 0.0f;
      const int64_t bk = k0 + r, bn = col0 + tx;
      bs[r][tx] = (bk < k && bn < n) ? b[bk * b_sk + bn * b_sn] : 0.0f;
    }
    __syncthreads();
    for (int kk = 0; kk < kT; ++kk) {
      const float bv = bs[kk][tx];
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[i] = fmaf(as[ty + 8 * i][kk], bv, acc[i]);
    }
    __syncthreads();
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int64_t r = row0 + ty + 8 * i, cc = col0 + tx;
    if (r < m && cc < n) c[r * n + cc] = acc[i] + (bias ? bias[cc] : 0.0f);
  }
}

__global__ void convert_kernel(int dir, const void* __restrict__ x, int64_t n, void* __restrict__ y) {
  pdl_trigger();
  pdl_wait();
  for (int64_t i = int64_t(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
       i += int64_t(gridDim.x) * blockDim.x) {
    if (dir == 0)
      static_cast<uint16_t*>(y)[i] = f2bf(static_cast<const float*>(x)[i]);
    else
      static_cast<float*>(y)[i] = bf2f(static_cast<const uint16_t*>(x)[i]);
  }
}

inline unsigned grid_for(int64_t n, int threads = 256) {
  int64_t b = (n + threads - 1) / threads;
  const int64_t cap = int64_t(kNumSMs) * 16;
  if (b > cap) b = cap;
  return unsigned(b < 1 ? 1 : b);
}

// Threads per row for rms_norm.  With many bf16 rows of whole 16-byte chunks
// (enough blocks to fill the GPU), four chunks per thread -- 128 threads for
// 4096 columns, 256 for 8192 -- so each thread has four loads in flight and
// the block reduction is short (16384 x 4096: 86 -> 32 us).  A few rows
// (decode) are latency-bound and keep one chunk per thread.
inline int row_threads(int64_t cols, bool chunked = false) {
  if (chunked) {
    const int64_t t = ((cols / 8 + 3) / 4 + 31) / 32 * 32;
    return int(t < 64 ? 64 : t > 1024 ? 1024 : t);
  }
  if (cols >= 1024) return 512;
  if (cols >= 256) return 256;
  return 128;
}

}  // namespace

template <typename T>
int launch_rms_norm(const T* x, const T* g, int64_t rows, int64_t cols, float eps, T* y,
                    cudaStream_t st, bool g_ready) {
  if (rows == 0 || cols == 0) return SB_OK;
  const bool chunked = sizeof(T) == 2 && cols % 8 == 0 && rows >= 4 * kNumSMs;
  launch_pdl(rms_norm_kernel<T>, dim3(unsigned(rows)), dim3(row_threads(cols, chunked)), 0, st, x, g, cols, eps, y,
             g_ready ? 1 : 0);
  SB_LAUNCH_CHECK();
  return SB_OK;
}

template <typename T>
int launch_rope(const T* x, const int32_t* pos, int64_t rows, int64_t heads, int64_t head_dim,
                double theta, T* y, cudaStream_t st, const double* inv_freq) {
  if (head_dim % 2) return SB_INVALID_ARGUMENT;
  if (rows * heads * (head_dim / 2) == 0) return SB_OK;
  // Rows per pass: as many as fit in the default 48 KB of dynamic shared
  // memory, up to kRopeRows.
  const int64_t half = head_dim / 2;
  const int64_t fit = (48 * 1024 / int64_t(sizeof(double)) / half - 1) / 2;
  if (fit < 1) return SB_INVALID_ARGUMENT;
  const int nr = int(fit < kRopeRows ? fit : kRopeRows);
  const int64_t groups = (rows + nr - 1) / nr;
  const unsigned blocks = unsigned(groups < 8 * kNumSMs ? groups : 8 * kNumSMs);
  const size_t smem = size_t(half) * (1 + 2 * nr) * sizeof(double);
  launch_pdl(rope_kernel<T>, dim3(blocks), dim3(256), smem, st, x, pos, rows, int(heads), int(head_dim), theta, y,
             nr, inv_freq);
  SB_LAUNCH_CHECK();
  return SB_OK;
}

template <typename T>
int launch_swiglu(const T* gate, const T* up, int64_t n, T* y, cudaStream_t st) {
  if (n == 0) return SB_OK;
  launch_pdl(swiglu_kernel<T>, dim3(grid_for(n)), dim3(256), 0, st, gate, up, n, y);
  SB_LAUNCH_CHECK();
  return SB_OK;
}

template <typename T>
int launch_binary(int op, const T* a, const T* b, T* out, const BcastShape& sh, cudaStream_t st) {
  if (sh.total == 0) return SB_OK;
  launch_pdl(binary_kernel<T>, dim3(grid_for(sh.total)), dim3(256), 0, st, op, a, b, out, sh);
  SB_LAUNCH_CHECK();
  return SB_OK;
}

template <typename T>
int launch_unary(int op, const T* x, int64_t n, T* y, cudaStream_t st) {
  if (n == 0) return SB_OK;
  launch_pdl(unary_kernel<T>, dim3(grid_for(n)), dim3(256), 0, st, op, x, n, y);
  SB_LAUNCH_CHECK();
  return SB_OK;
}

template <typename T>
int launch_softmax(const T* x, int64_t rows, int64_t cols, T* y, cudaStream_t st) {
  if (rows == 0 || cols == 0) return SB_OK;
  launch_pdl(softmax_kernel<T>, dim3(unsigned(rows)), dim3(row_threads(cols)), 0, st, x, cols, y);
  SB_LAUNCH_CHECK();
  return SB_OK;
}

template <typename T>
int launch_layer_norm(const T* x, const T* gamma, const T* beta, int64_t rows, int64_t cols,
                      float eps, T* y, cudaStream_t st) {
  if (rows == 0 || cols == 0) return SB_OK;
  launch_pdl(layer_norm_kernel<T>, dim3(unsigned(rows)), dim3(row_threads(cols)), 0, st, x, gamma, beta, cols, eps, y);
  SB_LAUNCH_CHECK();
  return SB_OK;
}

template <typename T>
int launch_transpose2(const T* x, int64_t rows, int64_t cols, T* y, cudaStream_t st) {
  if (rows * cols == 0) return SB_OK;
  launch_pdl(transpose2_kernel<T>, dim3(grid_for(rows * cols)), dim3(256), 0, st, x, rows, cols, y);
  SB_LAUNCH_CHECK();
  return SB_OK;
}

template <typename T>
int launch_slice_cols(const T* x, int64_t rows, int64_t cols, int64_t start, int64_t stride,
                      int64_t out_cols, T* y, cudaStream_t st) {
  if (rows * out_cols == 0) return SB_OK;
  launch_pdl(slice_cols_kernel<T>, dim3(grid_for(rows * out_cols)), dim3(256), 0, st, x, rows, cols, start, stride,
                                                                  out_cols, y);
  SB_LAUNCH_CHECK();
  return SB_OK;
}

template <typename T>
int launch_broadcast(const T* a, T* out, const BcastShape& sh, cudaStream_t st) {
  if (sh.total == 0) return SB_OK;
  launch_pdl(broadcast_kernel<T>, dim3(grid_for(sh.total)), dim3(256), 0, st, a, out, sh);
  SB_LAUNCH_CHECK();
  return SB_OK;
}

template <typename T>
int launch_embed(const int32_t* ids, int64_t rows, const T* table, int64_t vocab, int64_t dim,
                 T* out, int* err, cudaStream_t st) {
  if (rows == 0 || dim == 0) return SB_OK;
  launch_pdl(embed_kernel<T>, dim3(unsigned(rows)), dim3(256), 0, st, ids, table, vocab, dim, out, err);
  SB_LAUNCH_CHECK();
  return SB_OK;
}

template <typename T>
int launch_argmax(const T* x, int64_t rows, int64_t cols, int32_t* out, cudaStream_t st) {
  if (rows == 0) return SB_OK;
  launch_pdl(argmax_kernel<T>, dim3(unsigned(rows)), dim3(512), 0, st, x, cols, out);
  SB_LAUNCH_CHECK();
  return SB_OK;
}

template <typename T>
__global__ void last_rows_kernel(const T* __restrict__ x, int64_t batch, int64_t tps, int64_t cols,
                                 T* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int64_t total = batch * cols;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < total; i += int64_t(gridDim.x) * blockDim.x) {
    const int64_t b = i / cols, c = i - b * cols;
    out[i] = x[(b * tps + tps - 1) * cols + c];
  }
}

template <typename T>
int launch_last_rows(const T* x, int64_t batch, int64_t tokens_per_seq, int64_t cols, T* out, cudaStream_t st) {
  if (batch == 0 || cols == 0) return SB_OK;
  launch_pdl(last_rows_kernel<T>, dim3(grid_for(batch * cols)), dim3(256), 0, st, x, batch, tokens_per_seq, cols,
             out);
  SB_LAUNCH_CHECK();
  return SB_OK;
}

int launch_gemm_f32(const float* a, const float* b, const float* bias, int64_t m, int64_t k,
                    int64_t n, bool b_is_nk, float* c, cudaStream_t st) {
  if (m == 0 || n == 0) return SB_OK;
  const dim3 grid(unsigned((n + kT - 1) / kT), unsigned((m + kT - 1) / kT));
  // b_is_nk: B stored [n, k] (Linear weight); else [k, n] (MatMul).
  const int64_t sk = b_is_nk ? 1 : n, sn = b_is_nk ? k : 1;
  launch_pdl(gemm_f32_kernel, dim3(grid), dim3(256), 0, st, a, b, bias, m, k, n, sk, sn, c);
  SB_LAUNCH_CHECK();
  return SB_OK;
}

int launch_convert(int dir, const void* x, int64_t n, void* y, cudaStream_t st) {
  if (n == 0) return SB_OK;
  launch_pdl(convert_kernel, dim3(grid_for(n)), dim3(256), 0, st, dir, x, n, y);
  SB_LAUNCH_CHECK();
  return SB_OK;
}

#define SB_INST(T)                                                                              \
  template int launch_last_rows<T>(const T*, int64_t, int64_t, int64_t, T*, cudaStream_t);       \
  template int launch_rms_norm<T>(const T*, const T*, int64_t, int64_t, float, T*, cudaStream_t, bool); \
  template int launch_rope<T>(const T*, const int32_t*, int64_t, int64_t, int64_t, double, T*,  \
                              cudaStream_t, const double*);                                    \
  template int launch_swiglu<T>(const T*, const T*, int64_t, T*, cudaStream_t);                 \
  template int launch_binary<T>(int, const T*, const T*, T*, const BcastShape&, cudaStream_t);  \
  template int launch_unary<T>(int, const T*, int64_t, T*, cudaStream_t);                       \
  template int launch_softmax<T>(const T*, int64_t, int64_t, T*, cudaStream_t);                 \
  template int launch_layer_norm<T>(const T*, const T*, const T*, int64_t, int64_t, float, T*,  \
                                    cudaStream_t);                                             \
  template int launch_transpose2<T>(const T*, int64_t, int64_t, T*, cudaStream_t);              \
  template int launch_slice_cols<T>(const T*, int64_t, int64_t, int64_t, int64_t, int64_t, T*,  \
                                    cudaStream_t);                                             \
  template int launch_broadcast<T>(const T*, T*, const BcastShape&, cudaStream_t);              \
  template int launch_embed<T>(const int32_t*, int64_t, const T*, int64_t, int64_t, T*, int*,   \
                               cudaStream_t);                                                  \
  template int launch_argmax<T>(const T*, int64_t, int64_t, int32_t*, cudaStream_t);

SB_INST(float)
SB_INST(uint16_t)
#undef SB_INST

}  // namespace sb
