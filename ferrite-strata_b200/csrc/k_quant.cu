// Weight quantisation and dequantisation kernels.
//
// The conventions are this backend's (the reference defines no quantised
// Linear): int8 symmetric per output channel with an f32 scale, and int4
// symmetric in groups of 32 along k with a bf16 scale, two codes per byte,
// low nibble = even k.  Both are bit-exact with the CPU oracle: IEEE division
// (no fast-math), round-to-nearest-even via rintf, and the int4 scale is
// rounded to bf16 before the codes are computed.
#include "common.cuh"

namespace sb {

__global__ void quant_w4g32_kernel(const float* __restrict__ w, int64_t n, int64_t k,
                                   uint8_t* __restrict__ packed, uint16_t* __restrict__ scale) {
  pdl_trigger();
  pdl_wait();
  const int64_t groups = k / 32;
  const int64_t gid = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (gid >= n * groups) return;
  const int64_t row = gid / groups, g = gid % groups;
  const float* src = w + row * k + g * 32;
  float v[32];
  float amax = 0.0f;
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    v[i] = src[i];
    amax = fmaxf(amax, fabsf(v[i]));
  }
  const uint16_t sb = f2bf(amax / 7.0f);
  const float s = bf2f(sb);
  scale[gid] = sb;
  uint8_t out[16];
#pragma unroll
  for (int i = 0; i < 32; i += 2) {
    int lo = 0, hi = 0;
    if (s != 0.0f) {
      lo = int(fminf(fmaxf(rintf(v[i] / s), -8.0f), 7.0f));
      hi = int(fminf(fmaxf(rintf(v[i + 1] / s), -8.0f), 7.0f));
    }
    out[i / 2] = uint8_t((lo & 0xf) | ((hi & 0xf) << 4));
  }
  uint4 o;
  memcpy(&o, out, 16);
  *reinterpret_cast<uint4*>(packed + row * (k / 2) + g * 16) = o;
}

// One block per row: block-wide amax, then codes.
__global__ void quant_w8pc_kernel(const float* __restrict__ w, int64_t n, int64_t k,
                                  int8_t* __restrict__ q, float* __restrict__ scale) {
  pdl_trigger();
  pdl_wait();
  const int64_t row = blockIdx.x;
  const float* src = w + row * k;
  float amax = 0.0f;
  for (int64_t i = threadIdx.x; i < k; i += blockDim.x) amax = fmaxf(amax, fabsf(src[i]));
  __shared__ float red[32];
  amax = warp_max(amax);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = amax;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.0f;
    v = warp_max(v);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float s = red[0] / 127.0f;
  if (threadIdx.x == 0) scale[row] = s;
  for (int64_t i = threadIdx.x; i < k; i += blockDim.x) {
    float c = s == 0.0f ? 0.0f : fminf(fmaxf(rintf(src[i] / s), -127.0f), 127.0f);
    q[row * k + i] = int8_t(c);
  }
}

__global__ void dequant_w4g32_kernel(const uint8_t* __restrict__ packed,
                                     const uint16_t* __restrict__ scale, int64_t n, int64_t k,
                                     float* __restrict__ w) {
  pdl_trigger();
  pdl_wait();
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= n * k) return;
  const int64_t row = idx / k, col = idx % k;
  const uint8_t b = packed[row * (k / 2) + col / 2];
  int v = (col & 1) ? (b >> 4) : (b & 0xf);
  v = v >= 8 ? v - 16 : v;
  w[idx] = float(v) * bf2f(scale[row * (k / 32) + col / 32]);
}

__global__ void dequant_w8pc_kernel(const int8_t* __restrict__ q, const float* __restrict__ scale,
                                    int64_t n, int64_t k, float* __restrict__ w) {
  pdl_trigger();
  pdl_wait();
  const int64_t idx = int64_t(blockIdx.x) * blockDim.x + threadIdx.x;
  if (idx >= n * k) return;
  w[idx] = float(q[idx]) * scale[idx / k];
}

int launch_quant_w4g32(const float* w, int64_t n, int64_t k, uint8_t* packed, uint16_t* scale,
                       cudaStream_t st) {
  if (n < 0 || k <= 0 || k % 32) return SB_INVALID_ARGUMENT;
  const int64_t total = n * (k / 32);
  if (total == 0) return SB_OK;
  launch_pdl(quant_w4g32_kernel, dim3(ceil_div(total, 128)), dim3(128), 0, st, w, n, k, packed, scale);
  SB_LAUNCH_CHECK();
  return SB_OK;
}

int launch_quant_w8pc(const float* w, int64_t n, int64_t k, int8_t* q, float* scale,
                      cudaStream_t st) {
  if (n < 0 || k <= 0) return SB_INVALID_ARGUMENT;
  if (n == 0) return SB_OK;
  launch_pdl(quant_w8pc_kernel, dim3(unsigned(n)), dim3(256), 0, st, w, n, k, q, scale);
  SB_LAUNCH_CHECK();
  return SB_OK;
}

int launch_dequant_w4g32(const uint8_t* packed, const uint16_t* scale, int64_t n, int64_t k,
                         float* w, cudaStream_t st) {
  if (n < 0 || k <= 0 || k % 32) return SB_INVALID_ARGUMENT;
  if (n == 0) return SB_OK;
  launch_pdl(dequant_w4g32_kernel, dim3(ceil_div(n * k, 256)), dim3(256), 0, st, packed, scale, n, k, w);
  SB_LAUNCH_CHECK();
  return SB_OK;
}

int launch_dequant_w8pc(const int8_t* q, const float* scale, int64_t n, int64_t k, float* w,
                        cudaStream_t st) {
  if (n < 0 || k <= 0) return SB_INVALID_ARGUMENT;
  if (n == 0) return SB_OK;
  launch_pdl(dequant_w8pc_kernel, dim3(ceil_div(n * k, 256)), dim3(256), 0, st, q, scale, n, k, w);
  SB_LAUNCH_CHECK();
  return SB_OK;
}

}  // namespace sb
