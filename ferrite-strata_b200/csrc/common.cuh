// Shared device helpers for the B200 kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>

namespace sb {

// Host-side count of kernel launches enqueued by this library.  Launches
// recorded into a CUDA graph are counted once per replay by the executor.
extern std::atomic<uint64_t> g_launches;

inline void count_launch(uint64_t n = 1) { g_launches.fetch_add(n, std::memory_order_relaxed); }

constexpr int kNumSMs = 148;  // B200: 2 dies x 74 SMs

inline int ceil_div(int64_t a, int64_t b) { return int((a + b - 1) / b); }

// Runs a set-up step (such as raising a kernel's dynamic shared-memory limit,
// which the runtime keeps per device) once on each device that needs it.
// Devices past the 64th run it on every call.
struct PerDeviceOnce {
  std::atomic<uint64_t> done{0};
  template <typename F>
  bool run(F&& setup) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return setup();
    const uint64_t bit = uint64_t(1) << dev;
    if (done.load(std::memory_order_acquire) & bit) return true;
    if (!setup()) return false;
    done.fetch_or(bit, std::memory_order_acq_rel);
    return true;
  }
};

// A paged KV cache.  With a block table the caches are page pools
// [num_pages, kv_heads, page_size, head_dim] and position p of sequence s is
// row p % page_size of page table[s * pages_per_seq + p / page_size], so a
// sequence's cache grows a page at a time and pages can be handed between
// sequences by rewriting the table.  page_size is a power of two from 16 to
// 4096, so a 16-position slab and a 128-position tile never straddle pages
// and a page is either part of a tile or a whole number of tiles.  With no
// table (the default) the caches are contiguous [batch, kv_heads, max_len,
// head_dim].
#if defined(__CUDACC__)
#define SB_HOST_DEVICE __host__ __device__
#else
#define SB_HOST_DEVICE
#endif
struct KvPages {
  const int32_t* table = nullptr;
  int page_size = 0;
  int pages_per_seq = 0;
  int num_pages = 0;
  SB_HOST_DEVICE bool paged() const { return table != nullptr; }
};

inline bool kv_page_size_ok(int64_t ps) { return ps >= 16 && ps <= 4096 && (ps & (ps - 1)) == 0; }

#if !defined(__CUDACC__)
bool pdl_enabled();
#endif

#if defined(__CUDACC__)
// cos and sin of the RoPE angle pos * inv (radians) as f32.  The angle is
// formed and reduced modulo 2 pi in double (a few FP64 operations; exact to
// far below f32 resolution for any position), then evaluated by the f32
// sincosf on |r| <= pi, whose error of about one f32 ulp is what rounding a
// double-precision result to f32 costs anyway.  A double sincos per (row,
// frequency) instead bounds RoPE on B200's narrow FP64 pipe.
__device__ __forceinline__ void rope_cos_sin(int pos, double inv, float& c, float& s) {
  const double a = double(pos) * inv;
  const double k = rint(a * 0.15915494309189535);  // turns: a / (2 pi)
  const float r = float(fma(-k, 6.283185307179586, a));
  sincosf(r, &s, &c);
}

// The cache row (head_dim elements) that holds position p of (seq, kvh), or
// -1 when p lies outside the sequence's pages or its page index is not one of
// the pool's pages.  Callers check 0 <= p < max_len first.
__device__ __forceinline__ int64_t kv_row(const KvPages& kp, int seq, int kvh, int kv_heads, int max_len, int p) {
  if (!kp.table) return (int64_t(seq) * kv_heads + kvh) * max_len + p;
  const int lp = p / kp.page_size;
  if (lp >= kp.pages_per_seq) return -1;
  const int pg = __ldg(kp.table + int64_t(seq) * kp.pages_per_seq + lp);
  if (pg < 0 || pg >= kp.num_pages) return -1;
  return (int64_t(pg) * kv_heads + kvh) * kp.page_size + (p & (kp.page_size - 1));
}


__device__ __forceinline__ float bf2f(uint16_t v) { return __uint_as_float(uint32_t(v) << 16); }

// Round-to-nearest-even f32 -> bf16, matching the oracle bit for bit on
// finite values.
__device__ __forceinline__ uint16_t f2bf(float f) {
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }

__device__ __forceinline__ uint32_t pack_bf2(float lo, float hi) {
  return uint32_t(f2bf(lo)) | (uint32_t(f2bf(hi)) << 16);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// 128-bit read-only load that does not allocate in L1 (streamed weights).
__device__ __forceinline__ uint4 ldg_stream(const void* p) {
  uint4 r;
  asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
               : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
               : "l"(p));
  return r;
}

__device__ __forceinline__ uint4 ldg16(const void* p) {
  return __ldg(reinterpret_cast<const uint4*>(p));
}

// Programmatic dependent launch: let the next kernel in the stream start its
// independent prologue now, then wait until every kernel this one depends on
// has completed and its writes are visible.  Both are no-ops for a launch
// without the programmatic attribute.
__device__ __forceinline__ void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;"); }
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ void cp_async16(void* smem, const void* gmem) {
  const uint32_t s = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(s), "l"(gmem) : "memory");
}
__device__ __forceinline__ void cp_async_commit_wait_all() {
  asm volatile("cp.async.commit_group;\ncp.async.wait_group 0;" ::: "memory");
}

bool pdl_enabled();

// Launch with the programmatic-stream-serialization attribute (when enabled).
template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, dim3 block, size_t smem, cudaStream_t st,
                       Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = pdl_enabled() ? 1 : 0;
  return cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
}

#endif  // __CUDACC__

}  // namespace sb

// Status codes shared with strata_plugin.h.
#define SB_OK 0
#define SB_INVALID_ARGUMENT (-3)
#define SB_RESOURCE_EXHAUSTED (-5)
#define SB_INTERNAL (-6)

#define SB_LAUNCH_CHECK()                                   \
  do {                                                      \
    cudaError_t e_ = cudaGetLastError();                    \
    if (e_ != cudaSuccess) return SB_INTERNAL;              \
    sb::count_launch();                                     \
  } while (0)
