// One-shot all-reduce (bf16 sum) over NVLink peer memory, for the
// decode-sized messages of tensor parallelism (a few KB to 1 MB: the o_proj
// and down_proj outputs of a decode step).
//
// Every rank owns an exchange region (CUDA IPC memory, mapped by every other
// rank of the node):
//   [flags: kArBlocks x 8 ranks, uint32][slot 0: kArSlotBytes][slot 1: kArSlotBytes]
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

}  // namespace

size_t allreduce_region_bytes() { return kArFlagBytes + 2 * kArSlotBytes; }

size_t allreduce_counter_bytes() { return kArBlocks * sizeof(uint32_t); }

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
