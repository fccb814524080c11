// Internal types of libstrata_b200.so: context, buffers, executables.
#pragma once

#include <cuda_runtime.h>
#include <nccl.h>

#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

#include "../../../include/strata_b200.h"
#include "../k_elem.cuh"
#include "../k_gemv_mma.cuh"
#include "wire.hpp"

namespace sbp {

// A failure with a status code and a message, thrown inside the plugin and
// turned into a StrataError at the ABI boundary.
struct Failure {
  int32_t code;
  std::string msg;
};

[[noreturn]] inline void fail(int32_t code, std::string msg) { throw Failure{code, std::move(msg)}; }

struct Buffer {
  void* ptr = nullptr;
  uint64_t bytes = 0;
  bool owned = true;
};

// NCCL entry points, resolved with dlopen so the library loads on machines
// without NCCL and shares whichever libnccl.so.2 the process already has.
struct Nccl {
  void* lib = nullptr;
  ncclResult_t (*get_unique_id)(ncclUniqueId*) = nullptr;
  ncclResult_t (*comm_init_rank)(ncclComm_t*, int, ncclUniqueId, int) = nullptr;
  ncclResult_t (*all_reduce)(const void*, void*, size_t, ncclDataType_t, ncclRedOp_t, ncclComm_t,
                             cudaStream_t) = nullptr;
  ncclResult_t (*all_gather)(const void*, void*, size_t, ncclDataType_t, ncclComm_t, cudaStream_t) = nullptr;
  ncclResult_t (*comm_destroy)(ncclComm_t) = nullptr;
  const char* (*error_string)(ncclResult_t) = nullptr;
  bool load(std::string* why);
};

struct Ctx {
  std::mutex mu;
  int device = 0;
  bool has_device = false;
  bool device_ready = false;
  std::string device_name = "NVIDIA B200";
  uint64_t memory_bytes = 0;
  cudaStream_t stream = nullptr;
  int* d_err = nullptr;  // device-side error word (0 = none)
  std::vector<uint8_t> caps;  // capability section, built once
  Nccl nccl;
  ncclComm_t comm = nullptr;
  int rank = 0, world = 1;
  // NVLink all-reduce: this rank's IPC exchange region, the peers' regions as
  // mapped here, and the per-block call counters (set up by tp_init).
  bool ar_ready = false;
  void* ar_region = nullptr;
  uint32_t* ar_counters = nullptr;
  sb::ArPeers ar_peers{};
  void setup_allreduce();
  void teardown_allreduce();

  void ensure_device();  // lazily select the device and create the stream
  void check_device_error(const char* where);
};

enum class SK {
  Linear, RmsNorm, Rope, SwiGLU, Binary, Unary, Softmax, LayerNorm, Transpose, Slice,
  Broadcast, Copy, Embed, Argmax, LastToken, GemmF32, KvAppend, Attention, AllReduce, AllReduceAddNorm,
  Quant4, Quant8, Dequant4, Dequant8, QkvRope, VocabArgmax,
};

struct Step {
  SK kind;
  bool bf16 = false;           // float tensors of this step are bf16 (else f32)
  std::vector<uint32_t> v;     // value operands, meaning per kind
  int64_t i[10] = {0};         // integer parameters, meaning per kind
  double d = 0.0;              // theta / eps
  sb::BcastShape bs{};
  // Linear: v = {x, w0, s0, y0, r0, w1, s1, y1, r1, w2, s2, y2, r2}; r = kNone if absent
  sb::WFormat fmt = sb::WFormat::W4G32;
  sb::Epilogue epi = sb::Epilogue::None;
  int njobs = 0;
  uint64_t scratch_off = 0, scratch_bytes = 0;
  uint64_t const_off = UINT64_MAX;     // offset of this step's table in the executable's constants
  std::vector<uint32_t> reads, writes;  // for liveness; writes may include in-place inputs
  int node = -1;                       // originating graph node
  std::string label;
};

constexpr uint32_t kNone = 0xffffffffu;

// Per-class device time of executed steps, for profiling a whole step from
// the outside (STRATA_B200_STEP_TIMES=1: runs are eager, each step is
// bracketed by CUDA events, and the totals accumulate until read).
bool step_times_enabled();
// {"class": [steps, milliseconds], ...} since the last reset.
std::string step_times_json(bool reset);

struct Exe {
  Graph g;
  std::string label;
  std::vector<Step> steps;
  std::vector<uint32_t> alias;      // value -> value whose storage it shares
  std::vector<int64_t> ws_off;      // value -> workspace offset, -1 if none
  uint64_t ws_bytes = 0;
  void* ws = nullptr;
  // Tables computed on the host at lowering (RoPE inverse frequencies), placed
  // after the workspace at consts_off and uploaded with it.
  std::vector<uint8_t> consts;
  uint64_t consts_off = 0;
  std::vector<bool> is_output;
  std::vector<bool> needed_input;   // graph inputs some step reads
  // CUDA graph cache, keyed by the external pointers of a run.
  struct Cached {
    std::vector<void*> key;
    cudaGraphExec_t exec = nullptr;
    uint64_t kernels = 0;
  };
  std::vector<Cached> graphs;
  std::vector<void*> last_key;
  ~Exe();
};

// Lower a decoded graph.  Returns false (and a reason) to decline; throws
// Failure for a malformed graph.
bool lower(const Graph& g, Exe& exe, std::string* reason);

// Enqueue every step on ctx.stream with the given external pointers
// (indexed by value; null = not provided).
void enqueue(Ctx& ctx, Exe& exe, const std::vector<void*>& ext);

// Pattern-table query (the pull `supports`).
uint32_t supports_query(const std::string& pattern, const DType& dt, uint32_t shape_kind,
                        uint8_t shape_rank);
std::vector<uint8_t> build_caps(const Ctx& ctx);

}  // namespace sbp
