// Decode attention for callers that must not allocate device memory.
//
// The regular entry point, strata_b200_attention_decode_bf16, takes a scratch
// buffer from the caller for the split-KV partial results.  Some callers
// cannot provide one: code that runs while a stream is being captured into a
// CUDA graph in a mode where cudaMalloc is refused, runtimes whose device
// memory is entirely owned by their own pool and may not call cudaMalloc or
// cudaFree (which can also synchronise the whole device), and latency-bound
// loops that are not allowed to allocate at all.  This variant uses a fixed
// scratch area that lives in the library itself instead.
//
// The scratch is a file-scope __device__ array of kNoAllocScratchBytes.
// Every GPU on which the library's kernels are loaded keeps that much memory
// reserved until the process exits.  Host code cannot use the array's name as
// a device address (on the host it names a stand-in object), so the address
// is looked up with cudaGetSymbolAddress once per device, with that device
// current, the first time this entry point runs on it.  The lookup is kept
// together with the CUDA context it was made in: after cudaDeviceReset the
// device gets a new context, the module is loaded again (possibly at another
// address), and the next call looks the address up again.
#include <cuda.h>

#include <mutex>

#include "../../include/strata_b200.h"
#include "k_elem.cuh"

namespace sb {

namespace {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB
constexpr int kMaxDevices = 64;

__device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

struct ScratchAddr {
  CUcontext ctx = nullptr;  // the context the address belongs to
  void* ptr = nullptr;
};

std::mutex g_noalloc_mutex;
ScratchAddr g_noalloc_addr[kMaxDevices];

using CtxGetCurrent = CUresult (*)(CUcontext*);

CtxGetCurrent ctx_get_current() {
  static CtxGetCurrent fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return CtxGetCurrent(nullptr);
    return reinterpret_cast<CtxGetCurrent>(p);
  }();
  return fn;
}

// The device address of the scratch array on the current device.  Returns
// null if it cannot be determined.  Allocates nothing: the lookup only reads
// the address of memory the module already holds.
void* noalloc_scratch() {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  CtxGetCurrent get = ctx_get_current();
  if (!get) return nullptr;
  CUcontext ctx = nullptr;  // null until the runtime has started on this thread's device
  if (get(&ctx) != CUDA_SUCCESS) return nullptr;
  std::lock_guard<std::mutex> lk(g_noalloc_mutex);
  ScratchAddr& a = g_noalloc_addr[dev];
  if (!ctx || a.ctx != ctx || !a.ptr) {
    void* ptr = nullptr;
    if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess) {
      cudaGetLastError();
      return nullptr;
    }
    if (get(&ctx) != CUDA_SUCCESS || !ctx) return nullptr;  // the lookup made the context current
    a.ctx = ctx;
    a.ptr = ptr;
  }
  return a.ptr;
}

}  // namespace

}  // namespace sb

using namespace sb;

extern "C" {

uint64_t strata_b200_noalloc_scratch_capacity(void) { return kNoAllocScratchBytes; }

int32_t strata_b200_attention_decode_bf16_noalloc(const uint16_t* q, const uint16_t* k_new,
                                                  const uint16_t* v_new, uint16_t* k_cache,
                                                  uint16_t* v_cache, const int32_t* pos,
                                                  int64_t batch, int64_t heads, int64_t kv_heads,
                                                  int64_t head_dim, int64_t max_len, uint16_t* out,
                                                  void* stream) {
  if (batch < 0 || heads <= 0 || kv_heads <= 0 || head_dim <= 0 || max_len <= 0)
    return SB_INVALID_ARGUMENT;
  // The partials this call needs: zero when the shape runs on the tensor-core
  // kernel (its splits merge on chip), the split-KV partials of the CUDA-core
  // kernel otherwise (more than 8 query heads per kv head).  Every slot the
  // merge reads is written first by the same call, so nothing has to be
  // cleared between calls.
  if (batch > 65535) return SB_INVALID_ARGUMENT;
  const uint64_t need = attention_v2_scratch_bytes(batch, heads, kv_heads, head_dim, max_len);
  if (need > kNoAllocScratchBytes) return SB_RESOURCE_EXHAUSTED;
  void* scratch = noalloc_scratch();
  if (!scratch) return SB_INTERNAL;
  cudaStream_t st = reinterpret_cast<cudaStream_t>(stream);
  int rc = launch_kv_append<uint16_t>(k_new, v_new, k_cache, v_cache, pos, batch, 1, kv_heads,
                                      head_dim, max_len, nullptr, st);
  if (rc) return rc;
  return launch_attention_v2(q, k_cache, v_cache, pos, batch, 1, heads, kv_heads, head_dim,
                             max_len, true, static_cast<float*>(scratch), out, nullptr, st);
}

}  // extern "C"
