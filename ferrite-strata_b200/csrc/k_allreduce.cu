// One-shot all-reduce (bf16 sum) over NVLink peer memory, for the
// decode-sized messages of tensor parallelism (a few KB to 1 MB: the o_proj
// and down_proj outputs of a decode step).
//
// Every rank owns an exchange region (CUDA IPC memory, mapped by every other
// rank of the node):
//   [flags: 128 blocks x 8 ranks, uint32][slot 0][slot 1][slot 2][slot 3]
// (slots of kArSlotBytes; 0 and 1 for the plain all-reduce, 2 and 3 for the
// fused all-reduce + add + RMSNorm below)
// Call g of block b (g counts the all-reduces this block has run, kept per
// block on the device so CUDA-graph replays advance it):
//   1. copy this block's slice of x into slot g & 1 of the own region;
//   2. release-store g into flag [b][rank] of every peer's region;
//   3. wait (bounded) until every peer's flag [b][peer] in the own region
//      reaches g;
//   4. sum the slice over all ranks' slots in rank order 0..world-1 (the same
//      order on every rank, so every rank gets bit-identical results).
// A slot is rewritten two calls later; by then every peer has passed call
// g + 1's flag exchange, which it reaches only after finishing call g, so the
// double buffer is safe.  A wait that runs out sets device error word 5 and
// the block returns.
//
// The kernel is launched without programmatic dependent launch and never
// triggers its dependents early: its waits must not hold SMs that a
// dependent kernel is waiting for.
#include "common.cuh"
#include "k_elem.cuh"

namespace sb {

namespace {

constexpr int kArBlocks = 32;
constexpr int kArThreads = 512;
constexpr uint32_t kArSpinLimit = 1u << 24;  // about a second of polling

__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__global__ void __launch_bounds__(kArThreads)
    allreduce_bf16_kernel(const uint16_t* __restrict__ x, uint16_t* __restrict__ y, int64_t n8, int rank,
                          int world, ArPeers peers, uint32_t* __restrict__ counters, int* err) {
  __shared__ uint32_t s_gen;
  __shared__ int s_ok;
  const int b = blockIdx.x, tid = threadIdx.x;
  if (tid == 0) {
    s_gen = counters[b] + 1;
    s_ok = 1;
  }
  __syncthreads();
  const uint32_t gen = s_gen;
  const size_t slot = kArFlagBytes + size_t(gen & 1) * kArSlotBytes;
  const int64_t per = (n8 + kArBlocks - 1) / kArBlocks;
  const int64_t lo = b * per, hi = lo + per < n8 ? lo + per : n8;

  uint4* mine = reinterpret_cast<uint4*>(static_cast<char*>(peers.base[rank]) + slot);
  for (int64_t i = lo + tid; i < hi; i += kArThreads) mine[i] = __ldg(reinterpret_cast<const uint4*>(x) + i);
  __syncthreads();
  if (tid < world && tid != rank) {
    __threadfence_system();
    st_release_sys(static_cast<uint32_t*>(peers.base[tid]) + b * 8 + rank, gen);
  }
  if (tid < world && tid != rank) {
    const uint32_t* f = static_cast<const uint32_t*>(peers.base[rank]) + b * 8 + tid;
    uint32_t spins = 0;
    while (ld_acquire_sys(f) < gen) {
      if (++spins == kArSpinLimit) {
        atomicExch(&s_ok, 0);
        break;
      }
    }
  }
  __syncthreads();
  if (!s_ok) {
    if (tid == 0) {
      if (err) atomicExch(err, 5);
      counters[b] = gen;
    }
    return;
  }
  for (int64_t i = lo + tid; i < hi; i += kArThreads) {
    float acc[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
    for (int r = 0; r < world; ++r) {
      const uint4 v = __ldcv(reinterpret_cast<const uint4*>(static_cast<const char*>(peers.base[r]) + slot) + i);
      const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        acc[2 * e] += bf_lo(w[e]);
        acc[2 * e + 1] += bf_hi(w[e]);
      }
    }
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) o[e] = uint32_t(f2bf(acc[2 * e])) | (uint32_t(f2bf(acc[2 * e + 1])) << 16);
    reinterpret_cast<uint4*>(y)[i] = make_uint4(o[0], o[1], o[2], o[3]);
  }
  if (tid == 0) counters[b] = gen;
}

// All-reduce of one row per block fused with the residual add and the
// RMSNorm that follow it in a tensor-parallel decoder layer:
//   h = bf16(bf16(sum over ranks of x) + r),  n = bf16(h * rsqrt(mean(h^2) + eps) * gamma).
// The exchange is the one above with flags and counters at block index
// kArBlocks + row and its own pair of slots (2 and 3), in which row r always
// owns bytes [r * kArnRowBytes, (r + 1) * kArnRowBytes): only block r of
// every rank touches them, whatever the row count or width of a call, so the
// per-block double-buffer argument holds for each row on its own.  Every
// rank sums in rank order and gets the same h and n.
constexpr int kArnThreads = 512;
constexpr int kArnChunks = 2;  // 16-byte chunks per thread: rows of up to 8192 columns
constexpr size_t kArnRowBytes = size_t(kArnThreads) * kArnChunks * 16;
static_assert(kArnRowBytes * kArMaxRows <= kArSlotBytes, "fused all-reduce rows overflow a slot");
static_assert((kArBlocks + kArMaxRows) * 8 * 4 <= kArFlagBytes, "flag area too small");

__global__ void __launch_bounds__(kArnThreads)
    allreduce_add_norm_bf16_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ r,
                                   const uint16_t* __restrict__ gamma, uint16_t* __restrict__ h_out,
                                   uint16_t* __restrict__ n_out, int cols, float eps, int rank, int world,
                                   ArPeers peers, uint32_t* __restrict__ counters, int* err) {
  __shared__ uint32_t s_gen;
  __shared__ int s_ok;
  __shared__ float red[32];
  const int row = blockIdx.x, fb = kArBlocks + row, tid = threadIdx.x;
  if (tid == 0) {
    s_gen = counters[fb] + 1;
    s_ok = 1;
  }
  __syncthreads();
  const uint32_t gen = s_gen;
  const int c8 = cols / 8;
  const size_t slot = kArFlagBytes + size_t(2 + (gen & 1)) * kArSlotBytes + size_t(row) * kArnRowBytes;
  const uint4* xr = reinterpret_cast<const uint4*>(x + int64_t(row) * cols);
  uint4* mine = reinterpret_cast<uint4*>(static_cast<char*>(peers.base[rank]) + slot);
  for (int i = tid; i < c8; i += kArnThreads) mine[i] = __ldg(xr + i);
  __syncthreads();
  if (tid < world && tid != rank) {
    __threadfence_system();
    st_release_sys(static_cast<uint32_t*>(peers.base[tid]) + fb * 8 + rank, gen);
  }
  if (tid < world && tid != rank) {
    const uint32_t* f = static_cast<const uint32_t*>(peers.base[rank]) + fb * 8 + tid;
    uint32_t spins = 0;
    while (ld_acquire_sys(f) < gen) {
      if (++spins == kArSpinLimit) {
        atomicExch(&s_ok, 0);
        break;
      }
    }
  }
  __syncthreads();
  if (!s_ok) {
    if (tid == 0) {
      if (err) atomicExch(err, 5);
      counters[fb] = gen;
    }
    return;
  }
  uint4 hv[kArnChunks];
  float ss = 0.0f;
#pragma unroll
  for (int u = 0; u < kArnChunks; ++u) {
    const int i = tid + u * kArnThreads;
    hv[u] = make_uint4(0, 0, 0, 0);
    if (i < c8) {
      float acc[8] = {0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f, 0.0f};
      for (int q = 0; q < world; ++q) {
        const uint4 v = __ldcv(reinterpret_cast<const uint4*>(static_cast<const char*>(peers.base[q]) + slot) + i);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          acc[2 * e] += bf_lo(w[e]);
          acc[2 * e + 1] += bf_hi(w[e]);
        }
      }
      const uint4 rv = __ldg(reinterpret_cast<const uint4*>(r + int64_t(row) * cols) + i);
      const uint32_t rw[4] = {rv.x, rv.y, rv.z, rv.w};
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float h0 = bf2f(f2bf(bf2f(f2bf(acc[2 * e])) + bf_lo(rw[e])));
        const float h1 = bf2f(f2bf(bf2f(f2bf(acc[2 * e + 1])) + bf_hi(rw[e])));
        ss = fmaf(h0, h0, ss);
        ss = fmaf(h1, h1, ss);
        o[e] = uint32_t(f2bf(h0)) | (uint32_t(f2bf(h1)) << 16);
      }
      hv[u] = make_uint4(o[0], o[1], o[2], o[3]);
      reinterpret_cast<uint4*>(h_out + int64_t(row) * cols)[i] = hv[u];
    }
  }
  ss = warp_sum(ss);
  if ((tid & 31) == 0) red[tid >> 5] = ss;
  __syncthreads();
  if (tid < 32) {
    float t = tid < kArnThreads / 32 ? red[tid] : 0.0f;
    t = warp_sum(t);
    if (tid == 0) red[0] = t;
  }
  __syncthreads();
  const float inv = 1.0f / sqrtf(red[0] / float(cols) + eps);
#pragma unroll
  for (int u = 0; u < kArnChunks; ++u) {
    const int i = tid + u * kArnThreads;
    if (i < c8) {
      const uint4 gv = __ldg(reinterpret_cast<const uint4*>(gamma) + i);
      const uint32_t hw[4] = {hv[u].x, hv[u].y, hv[u].z, hv[u].w}, gw[4] = {gv.x, gv.y, gv.z, gv.w};
      uint32_t o[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        o[e] = uint32_t(f2bf((bf_lo(hw[e]) * inv) * bf_lo(gw[e]))) |
               (uint32_t(f2bf((bf_hi(hw[e]) * inv) * bf_hi(gw[e]))) << 16);
      reinterpret_cast<uint4*>(n_out + int64_t(row) * cols)[i] = make_uint4(o[0], o[1], o[2], o[3]);
    }
  }
  if (tid == 0) counters[fb] = gen;
}

// Distributed argmax over a vocabulary whose rows (the lm_head's output
// features) are split between the tensor-parallel ranks.  Each row's best
// logit becomes a 64-bit key that orders like (value, then lowest id): the
// value's bits, flipped so that unsigned order is float order (-0 counted as
// +0), over the complement of the vocabulary id; a row with no number (all
// NaN) has key 0.  The largest key over the ranks is the global argmax with
// the replicated argmax's rules (NaN skipped, lowest id on ties, 0 for a row
// of NaNs).  The exchange is the one above with flags and counters at block
// index kAmFlag0 + b and the key slots after the all-reduce's four slots; the
// grid is always kAmBlocks blocks and block b owns rows b, b + kAmBlocks, ...
// in every call, so the per-block double-buffer argument holds.
constexpr int kAmBlocks = 32;
constexpr int kAmThreads = 512;
constexpr int kAmFlag0 = kArBlocks + kArMaxRows;
constexpr size_t kAmSlotBytes = size_t(kAmMaxRows) * sizeof(uint64_t);
static_assert((kAmFlag0 + kAmBlocks) * 8 * 4 <= kArFlagBytes, "flag area too small");

__device__ __forceinline__ uint64_t am_key(float v, uint32_t id) {
  uint32_t u = __float_as_uint(v == 0.0f ? 0.0f : v);
  u = (u & 0x80000000u) ? ~u : (u | 0x80000000u);
  return (uint64_t(u) << 32) | uint64_t(0xFFFFFFFFu - id);
}

__device__ __forceinline__ int32_t am_id(uint64_t key) {
  return key ? int32_t(0xFFFFFFFFu - uint32_t(key)) : 0;
}

template <typename T>
__device__ __forceinline__ float am_ld(const T* p, int64_t i) {
  if constexpr (sizeof(T) == 2)
    return bf2f(p[i]);
  else
    return p[i];
}

__device__ __forceinline__ uint64_t am_max(uint64_t a, uint64_t b) { return a > b ? a : b; }

// The block's largest key of row xr (every thread gets it).
template <typename T>
__device__ uint64_t am_row_key(const T* __restrict__ xr, int64_t cols, int64_t offset, uint64_t* red) {
  uint64_t k = 0;
  for (int64_t c = threadIdx.x; c < cols; c += blockDim.x) {
    const float v = am_ld(xr, c);
    if (v == v) k = am_max(k, am_key(v, uint32_t(offset + c)));
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) k = am_max(k, __shfl_xor_sync(0xffffffffu, k, o));
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  __syncthreads();  // red is reused from the previous row
  if (lane == 0) red[warp] = k;
  __syncthreads();
  k = 0;
  for (int w = 0; w < int(blockDim.x >> 5); ++w) k = am_max(k, red[w]);
  return k;
}

template <typename T>
__global__ void __launch_bounds__(kAmThreads)
    vocab_argmax_kernel(const T* __restrict__ x, int64_t rows, int64_t cols, int64_t offset, int rank, int world,
                        ArPeers peers, uint32_t* __restrict__ counters, uint64_t* __restrict__ keys_out,
                        int32_t* __restrict__ out, int* err) {
  __shared__ uint64_t red[kAmThreads / 32];
  __shared__ uint64_t s_key[kAmMaxRows / kAmBlocks];
  __shared__ uint32_t s_gen;
  __shared__ int s_ok;
  pdl_trigger();
  pdl_wait();  // the logits come from the preceding kernel
  const int b = blockIdx.x, tid = threadIdx.x;
  const int64_t nmine = rows > b ? (rows - b + kAmBlocks - 1) / kAmBlocks : 0;
  if (world <= 1 || keys_out) {
    // No exchange: each row's key (or id) goes straight to global memory,
    // so any number of rows fits.
    for (int64_t j = 0; j < nmine; ++j) {
      const int64_t row = b + j * kAmBlocks;
      const uint64_t k = am_row_key(x + row * cols, cols, offset, red);
      if (tid == 0) {
        if (keys_out)
          keys_out[row] = k;
        else
          out[row] = am_id(k);
      }
    }
    return;
  }
  // The exchange stages this block's keys in s_key; the launcher refuses
  // more than kAmMaxRows rows, and every rank sees the same row count, so
  // all ranks leave here together if that check was bypassed.
  if (nmine > kAmMaxRows / kAmBlocks) {
    if (tid == 0 && err) atomicExch(err, 1);
    return;
  }
  for (int j = 0; j < int(nmine); ++j) {
    const int64_t row = b + int64_t(j) * kAmBlocks;
    const uint64_t k = am_row_key(x + row * cols, cols, offset, red);
    if (tid == 0) s_key[j] = k;
  }
  __syncthreads();
  const int fb = kAmFlag0 + b;
  if (tid == 0) {
    s_gen = counters[fb] + 1;
    s_ok = 1;
  }
  __syncthreads();
  const uint32_t gen = s_gen;
  const size_t slot = kArFlagBytes + 4 * kArSlotBytes + size_t(gen & 1) * kAmSlotBytes;
  uint64_t* mine = reinterpret_cast<uint64_t*>(static_cast<char*>(peers.base[rank]) + slot);
  for (int j = tid; j < nmine; j += blockDim.x) mine[b + j * kAmBlocks] = s_key[j];
  __syncthreads();
  if (tid < world && tid != rank) {
    __threadfence_system();
    st_release_sys(static_cast<uint32_t*>(peers.base[tid]) + fb * 8 + rank, gen);
  }
  if (tid < world && tid != rank) {
    const uint32_t* f = static_cast<const uint32_t*>(peers.base[rank]) + fb * 8 + tid;
    uint32_t spins = 0;
    while (ld_acquire_sys(f) < gen) {
      if (++spins == kArSpinLimit) {
        atomicExch(&s_ok, 0);
        break;
      }
    }
  }
  __syncthreads();
  if (!s_ok) {
    if (tid == 0) {
      if (err) atomicExch(err, 5);
      counters[fb] = gen;
    }
    return;
  }
  for (int j = tid; j < nmine; j += blockDim.x) {
    const int64_t row = b + int64_t(j) * kAmBlocks;
    uint64_t k = 0;
    for (int q = 0; q < world; ++q)
      k = am_max(k, __ldcv(reinterpret_cast<const unsigned long long*>(static_cast<const char*>(peers.base[q]) +
                                                                         slot) +
                           row));
    out[row] = am_id(k);
  }
  if (tid == 0) counters[fb] = gen;
}

__global__ void vocab_argmax_decode_kernel(const uint64_t* __restrict__ keys, int64_t rows, int32_t* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  const int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x;
  if (i < rows) out[i] = am_id(keys[i]);
}

}  // namespace

size_t allreduce_region_bytes() { return kArFlagBytes + 4 * kArSlotBytes + 2 * kAmSlotBytes; }

size_t allreduce_counter_bytes() { return (kArBlocks + kArMaxRows + kAmBlocks) * sizeof(uint32_t); }

template <typename T>
int launch_vocab_argmax(const T* x, int64_t rows, int64_t cols, int64_t offset, int rank, int world,
                        const ArPeers* peers, uint32_t* counters, uint64_t* keys, int32_t* out, int* err,
                        cudaStream_t st) {
  if (rows <= 0 || cols <= 0 || offset < 0 || offset + cols > int64_t(UINT32_MAX)) return SB_INVALID_ARGUMENT;
  const bool exchange = world > 1 && !keys;
  if (exchange && (!peers || !counters || rows > kAmMaxRows || world > 8 || rank < 0 || rank >= world))
    return SB_INVALID_ARGUMENT;
  const ArPeers pr = peers ? *peers : ArPeers{};
  // The exchange waits on the peers: no programmatic early launch of it.
  if (exchange)
    vocab_argmax_kernel<T><<<kAmBlocks, kAmThreads, 0, st>>>(x, rows, cols, offset, rank, world, pr, counters,
                                                             nullptr, out, err);
  else
    launch_pdl(vocab_argmax_kernel<T>, dim3(kAmBlocks), dim3(kAmThreads), 0, st, x, rows, cols, offset, rank,
               world, pr, counters, keys, out, err);
  if (cudaGetLastError() != cudaSuccess) return SB_INTERNAL;
  count_launch();
  return SB_OK;
}

template int launch_vocab_argmax<float>(const float*, int64_t, int64_t, int64_t, int, int, const ArPeers*,
                                        uint32_t*, uint64_t*, int32_t*, int*, cudaStream_t);
template int launch_vocab_argmax<uint16_t>(const uint16_t*, int64_t, int64_t, int64_t, int, int, const ArPeers*,
                                           uint32_t*, uint64_t*, int32_t*, int*, cudaStream_t);

int launch_vocab_argmax_decode(const uint64_t* keys, int64_t rows, int32_t* out, cudaStream_t st) {
  if (rows <= 0) return SB_OK;
  launch_pdl(vocab_argmax_decode_kernel, dim3(unsigned((rows + 255) / 256)), dim3(256), 0, st, keys, rows, out);
  if (cudaGetLastError() != cudaSuccess) return SB_INTERNAL;
  count_launch();
  return SB_OK;
}

bool allreduce_add_norm_supported(int64_t rows, int64_t cols, const void* x, const void* r, const void* gamma,
                                  const void* h, const void* n, int world) {
  const uintptr_t a = reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(r) |
                      reinterpret_cast<uintptr_t>(gamma) | reinterpret_cast<uintptr_t>(h) |
                      reinterpret_cast<uintptr_t>(n);
  return world >= 2 && world <= 8 && rows > 0 && rows <= kArMaxRows && cols > 0 && cols % 8 == 0 &&
         size_t(cols) * 2 <= kArnRowBytes && (a & 15) == 0;
}

int launch_allreduce_add_norm_bf16(const uint16_t* x, const uint16_t* r, const uint16_t* gamma, uint16_t* h,
                                   uint16_t* n, int64_t rows, int64_t cols, float eps, int rank, int world,
                                   const ArPeers& peers, uint32_t* counters, int* err, cudaStream_t st) {
  if (!allreduce_add_norm_supported(rows, cols, x, r, gamma, h, n, world) || rank < 0 || rank >= world)
    return SB_INVALID_ARGUMENT;
  allreduce_add_norm_bf16_kernel<<<unsigned(rows), kArnThreads, 0, st>>>(x, r, gamma, h, n, int(cols), eps, rank,
                                                                          world, peers, counters, err);
  if (cudaGetLastError() != cudaSuccess) return SB_INTERNAL;
  count_launch();
  return SB_OK;
}

bool allreduce_bf16_supported(int64_t n, const void* x, const void* y, int world) {
  return world >= 2 && world <= 8 && n > 0 && n % 8 == 0 && size_t(n) * 2 <= kArSlotBytes &&
         ((reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(y)) & 15) == 0;
}

int launch_allreduce_bf16(const uint16_t* x, uint16_t* y, int64_t n, int rank, int world, const ArPeers& peers,
                          uint32_t* counters, int* err, cudaStream_t st) {
  if (!allreduce_bf16_supported(n, x, y, world) || rank < 0 || rank >= world) return SB_INVALID_ARGUMENT;
  allreduce_bf16_kernel<<<kArBlocks, kArThreads, 0, st>>>(x, y, n / 8, rank, world, peers, counters, err);
  if (cudaGetLastError() != cudaSuccess) return SB_INTERNAL;
  count_launch();
  return SB_OK;
}

}  // namespace sb
