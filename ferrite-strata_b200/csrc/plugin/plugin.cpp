// libstrata_b200.so: the Ferrite Strata plugin ABI (StrataPluginV1,
// crates/ferrite-strata-plugin-api/src/raw.rs:591-789) for NVIDIA B200.
//
// Entry point contract, restated from the reference host
// (crates/ferrite-strata-plugin-api/src/host/plugin.rs and host/loader.rs):
//   * the host dlopens the library, reads `strata_plugin_v1`, checks the nine
//     mandatory entries, walks the extension chain and calls plugin_init;
//   * capabilities() returns a framed blob (count + section table + a
//     Capabilities section) that the host copies and then frees with
//     free_blob(ctx, &its_own_copy) -- so the payload is freed through
//     blob->data, never through the header address (plugin.rs:707-733);
//   * compile() is tri-state: OK with an executable, DECLINED with nothing
//     allocated, or a failure with an error object (plugin.rs:289-352);
//   * run() receives StrataBufferRef entries indexed by the decoded subgraph's
//     value indices (plugin.rs:426-534).
#include <cuda_runtime.h>
#include <dlfcn.h>

#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <memory>
#include <new>

#include "plugin.hpp"

using namespace sbp;

struct StrataError {
  uint32_t code;
  std::string msg;
  StrataMessageExt ext;
};

struct StrataBuffer {
  Buffer b;
};

struct StrataExecutable {
  Exe exe;
};

struct StrataEvent {
  cudaEvent_t ev;
};

namespace {

StrataError* make_error(int32_t code, const std::string& msg) {
  auto* e = new (std::nothrow) StrataError;
  if (!e) return nullptr;
  e->code = uint32_t(code);
  e->msg = msg;
  e->ext.base.struct_size = sizeof(StrataMessageExt);
  e->ext.base.ty = STRATA_EXT_MESSAGE;
  e->ext.base.next = nullptr;
  e->ext.message = e->msg.c_str();
  return e;
}

int32_t report(StrataError** out, int32_t code, const std::string& msg) {
  if (out) *out = make_error(code, msg);
  return code;
}

// Run `f`, mapping thrown failures onto status codes and error objects.
template <typename F>
int32_t guarded(StrataError** out_error, F&& f) {
  try {
    return f();
  } catch (const Failure& fl) {
    return report(out_error, fl.code, fl.msg);
  } catch (const WireError& we) {
    return report(out_error, STRATA_INVALID_ARGUMENT, std::string("malformed subgraph blob: ") + we.what());
  } catch (const std::bad_alloc&) {
    return report(out_error, STRATA_RESOURCE_EXHAUSTED, "host memory exhausted");
  } catch (const std::exception& ex) {
    return report(out_error, STRATA_INTERNAL, ex.what());
  }
}

void cuda_check(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return;
  const int32_t code = e == cudaErrorMemoryAllocation ? STRATA_RESOURCE_EXHAUSTED : STRATA_INTERNAL;
  fail(code, std::string(what) + ": " + cudaGetErrorString(e));
}

Ctx* C(void* ctx) {
  if (!ctx) fail(STRATA_INVALID_ARGUMENT, "null plugin context");
  return static_cast<Ctx*>(ctx);
}

int env_int(const char* name, int dflt) {
  const char* v = std::getenv(name);
  return v && *v ? std::atoi(v) : dflt;
}

bool graphs_enabled() { return env_int("STRATA_B200_CUDA_GRAPHS", 1) != 0 && !step_times_enabled(); }

// Cache of device allocations by (device, rounded size), so per-run buffers
// (the reference host allocates one per value per run) do not hit
// cudaMalloc.  Every context of the process shares it, so it has its own
// lock, and a buffer is only handed out again on the device it was made on.
struct Pool {
  std::mutex mu;
  std::multimap<std::pair<int, uint64_t>, void*> free_;
  void* get(int dev, uint64_t bytes) {
    std::lock_guard<std::mutex> lk(mu);
    auto it = free_.find({dev, bytes});
    if (it == free_.end()) return nullptr;
    void* p = it->second;
    free_.erase(it);
    return p;
  }
  void put(int dev, uint64_t bytes, void* p) {
    std::lock_guard<std::mutex> lk(mu);
    free_.emplace(std::make_pair(dev, bytes), p);
  }
  // Frees device dev's cached buffers; the caller has that device current.
  void drain(int dev) {
    std::lock_guard<std::mutex> lk(mu);
    for (auto it = free_.lower_bound({dev, 0}); it != free_.end() && it->first.first == dev;) {
      cudaFree(it->second);
      it = free_.erase(it);
    }
  }
};
Pool g_pool;

uint64_t round_bytes(uint64_t b) { return (std::max<uint64_t>(b, 1) + 255) & ~uint64_t(255); }

void* device_alloc(Ctx& c, uint64_t bytes) {
  const uint64_t rb = round_bytes(bytes);
  if (void* p = g_pool.get(c.device, rb)) return p;
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, rb);
  if (e == cudaErrorMemoryAllocation) {
    cudaGetLastError();
    g_pool.drain(c.device);
    e = cudaMalloc(&p, rb);
  }
  cuda_check(e, "cudaMalloc");
  return p;
}

void device_free(Ctx& c, uint64_t bytes, void* p) {
  if (p) g_pool.put(c.device, round_bytes(bytes), p);
}

}  // namespace

namespace sbp {

void Ctx::ensure_device() {
  if (!has_device) fail(STRATA_INTERNAL, "no CUDA device is visible to this process");
  cuda_check(cudaSetDevice(device), "cudaSetDevice");
  if (device_ready) return;
  cuda_check(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate");
  cuda_check(cudaMalloc(&d_err, sizeof(int)), "cudaMalloc(error word)");
  cuda_check(cudaMemset(d_err, 0, sizeof(int)), "cudaMemset(error word)");
  device_ready = true;
}

// After a synchronize: surface launch/execution errors and the kernels'
// input-validation word.
void Ctx::check_device_error(const char* where) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) fail(STRATA_INTERNAL, std::string(where) + ": " + cudaGetErrorString(e));
  int word = 0;
  cuda_check(cudaMemcpy(&word, d_err, sizeof(int), cudaMemcpyDeviceToHost), "reading the error word");
  if (word) {
    cuda_check(cudaMemset(d_err, 0, sizeof(int)), "clearing the error word");
    if (word == 4)
      fail(STRATA_INTERNAL, std::string(where) + ": a tensor-core pipeline wait ran out (the kernel stopped early)");
    if (word == 5)
      fail(STRATA_INTERNAL, std::string(where) + ": a tensor-parallel peer did not reach the all-reduce in time");
    const char* what = word == 2 ? "a position is outside the KV cache"
                     : word == 3 ? "a token id is outside the embedding table"
                     : word == 6 ? "a block-table entry that a position needs is not a page of the pool"
                                 : "a kernel rejected its input";
    fail(STRATA_INVALID_ARGUMENT, std::string(where) + ": " + what);
  }
}

bool Nccl::load(std::string* why) {
  if (lib) return true;
  for (const char* name : {"libnccl.so.2", "libnccl.so"}) {
    lib = dlopen(name, RTLD_NOW | RTLD_GLOBAL);
    if (lib) break;
  }
  if (!lib) {
    *why = "libnccl.so.2 could not be loaded";
    return false;
  }
  get_unique_id = reinterpret_cast<decltype(get_unique_id)>(dlsym(lib, "ncclGetUniqueId"));
  comm_init_rank = reinterpret_cast<decltype(comm_init_rank)>(dlsym(lib, "ncclCommInitRank"));
  all_reduce = reinterpret_cast<decltype(all_reduce)>(dlsym(lib, "ncclAllReduce"));
  comm_destroy = reinterpret_cast<decltype(comm_destroy)>(dlsym(lib, "ncclCommDestroy"));
  all_gather = reinterpret_cast<decltype(all_gather)>(dlsym(lib, "ncclAllGather"));
  error_string = reinterpret_cast<decltype(error_string)>(dlsym(lib, "ncclGetErrorString"));
  if (!get_unique_id || !comm_init_rank || !all_reduce || !comm_destroy || !error_string || !all_gather) {
    *why = "libnccl.so.2 lacks an expected symbol";
    return false;
  }
  return true;
}

// The exchange regions of the NVLink all-reduce: allocate and zero this
// rank's region, gather every rank's IPC handle over NCCL and map the peers'
// regions.  Any failure leaves ar_ready false and NCCL carries every
// all-reduce.  STRATA_B200_NVLINK_ALLREDUCE=0 turns the custom path off.
void Ctx::setup_allreduce() {
  const char* env = std::getenv("STRATA_B200_NVLINK_ALLREDUCE");
  if ((env && *env == '0') || world < 2 || world > 8 || !comm) return;
  if (cudaMalloc(&ar_region, sb::allreduce_region_bytes()) != cudaSuccess ||
      cudaMalloc(reinterpret_cast<void**>(&ar_counters), sb::allreduce_counter_bytes()) != cudaSuccess ||
      cudaMemset(ar_region, 0, sb::allreduce_region_bytes()) != cudaSuccess ||
      cudaMemset(ar_counters, 0, sb::allreduce_counter_bytes()) != cudaSuccess) {
    cudaGetLastError();
    teardown_allreduce();
    return;
  }
  cudaIpcMemHandle_t mine;
  if (cudaIpcGetMemHandle(&mine, ar_region) != cudaSuccess) {
    cudaGetLastError();
    teardown_allreduce();
    return;
  }
  constexpr size_t kH = sizeof(cudaIpcMemHandle_t);
  void* d_handles = nullptr;
  std::vector<cudaIpcMemHandle_t> all(world);
  bool ok = cudaMalloc(&d_handles, kH * world) == cudaSuccess &&
            cudaMemcpy(static_cast<char*>(d_handles) + kH * rank, &mine, kH, cudaMemcpyHostToDevice) == cudaSuccess;
  // Every rank reaches the all-gather with its region already zeroed.
  ok = ok && cudaDeviceSynchronize() == cudaSuccess &&
       nccl.all_gather(static_cast<char*>(d_handles) + kH * rank, d_handles, kH, ncclUint8, comm, stream) ==
           ncclSuccess &&
       cudaStreamSynchronize(stream) == cudaSuccess &&
       cudaMemcpy(all.data(), d_handles, kH * world, cudaMemcpyDeviceToHost) == cudaSuccess;
  if (d_handles) cudaFree(d_handles);
  for (int r = 0; ok && r < world; ++r) {
    if (r == rank) {
      ar_peers.base[r] = ar_region;
      continue;
    }
    void* p = nullptr;
    ok = cudaIpcOpenMemHandle(&p, all[r], cudaIpcMemLazyEnablePeerAccess) == cudaSuccess;
    ar_peers.base[r] = p;
  }
  if (!ok) {
    cudaGetLastError();
    teardown_allreduce();
    return;
  }
  ar_ready = true;
}

void Ctx::teardown_allreduce() {
  for (int r = 0; r < 8; ++r) {
    if (ar_peers.base[r] && ar_peers.base[r] != ar_region) cudaIpcCloseMemHandle(ar_peers.base[r]);
    ar_peers.base[r] = nullptr;
  }
  if (ar_region) cudaFree(ar_region);
  if (ar_counters) cudaFree(ar_counters);
  ar_region = nullptr;
  ar_counters = nullptr;
  ar_ready = false;
  cudaGetLastError();
}

}  // namespace sbp

// ---------------------------------------------------------------------------
// Error entries (raw.rs:603-616)
// ---------------------------------------------------------------------------

static void sb_error_free(StrataError* e) { delete e; }

static uint32_t sb_error_code(const StrataError* e) { return e ? e->code : uint32_t(STRATA_INTERNAL); }

static void sb_error_payload(const StrataError* e, StrataPayloadVisitor visitor, void* vctx) {
  if (!e || !visitor) return;
  visitor(vctx, const_cast<StrataExtBase*>(&e->ext.base));
}

// ---------------------------------------------------------------------------
// Capability (raw.rs:618-640)
// ---------------------------------------------------------------------------

static int32_t sb_capabilities(void* ctx, StrataWireBlob* out) {
  if (!ctx || !out) return STRATA_INVALID_ARGUMENT;
  try {
    Ctx* c = C(ctx);
    std::lock_guard<std::mutex> lk(c->mu);
    if (c->caps.empty()) c->caps = build_caps(*c);
    const std::vector<uint8_t> framed = frame_payload(kSectionCaps, c->caps);
    uint8_t* data = new uint8_t[framed.size() + 1];
    std::memcpy(data, framed.data(), framed.size());
    data[framed.size()] = 0;
    out->magic = kMagic;
    out->format_major = kFormatMajor;
    out->format_minor = kFormatMinor;
    out->payload_len = framed.size();
    out->data = data;
    out->nul = 0;
    return STRATA_OK;
  } catch (...) {
    return STRATA_INTERNAL;
  }
}

static uint32_t sb_supports(void* ctx, const StrataPatternQuery* q) {
  (void)ctx;
  if (!q || q->struct_size < sizeof(StrataPatternQuery) || (!q->pattern_id && q->pattern_id_len))
    return STRATA_SUPPORT_REFUSE;
  const std::string pattern(reinterpret_cast<const char*>(q->pattern_id), q->pattern_id_len);
  DType dt;
  dt.elem = q->dtype.element;
  dt.qkind = q->dtype.quant.kind;
  dt.block = q->dtype.quant.block_size;
  dt.sym = q->dtype.quant.symmetric;
  return supports_query(pattern, dt, q->shape_class.kind, q->shape_class.rank);
}

// ---------------------------------------------------------------------------
// Compile (raw.rs:642-657)
// ---------------------------------------------------------------------------

// Decode a graph section and lower it; null when the plugin declines.
static std::unique_ptr<StrataExecutable> compile_graph_section(const uint8_t* sec, size_t sec_len) {
  auto holder = std::make_unique<StrataExecutable>();
  holder->exe.g = decode_graph(sec, sec_len);
  holder->exe.label = "b200::" + holder->exe.g.name;
  std::string reason;
  if (!lower(holder->exe.g, holder->exe, &reason)) {
    // DECLINED carries no error object (status.rs); STRATA_B200_EXPLAIN=1
    // prints the reason for whoever is wiring a graph up.
    if (env_int("STRATA_B200_EXPLAIN", 0))
      std::fprintf(stderr, "strata_b200: declined `%s`: %s\n", holder->exe.g.name.c_str(), reason.c_str());
    return nullptr;
  }
  return holder;
}

static void check_blob_header(const StrataWireBlob& b, const char* what) {
  if (b.magic != kMagic) fail(STRATA_INVALID_ARGUMENT, std::string("the ") + what + " blob has the wrong magic");
  if (b.format_major != kFormatMajor)
    fail(STRATA_INVALID_ARGUMENT, "unsupported wire format major " + std::to_string(b.format_major));
  if (!b.data && b.payload_len) fail(STRATA_INVALID_ARGUMENT, std::string("null ") + what + " payload");
}

static int32_t sb_compile(void* ctx, const StrataCompileArgs* a, StrataExecutable** out_exe,
                          StrataError** out_error) {
  if (out_exe) *out_exe = nullptr;
  if (out_error) *out_error = nullptr;
  return guarded(out_error, [&]() -> int32_t {
    C(ctx);
    if (!a || !out_exe) fail(STRATA_INVALID_ARGUMENT, "compile needs arguments and an out-parameter");
    if (a->struct_size < sizeof(StrataCompileArgs))
      fail(STRATA_INVALID_ARGUMENT, "StrataCompileArgs is shorter than this plugin's ABI");
    const StrataWireBlob& b = a->subgraph;
    check_blob_header(b, "subgraph");
    const uint8_t* sec = nullptr;
    size_t sec_len = 0;
    if (!find_section(b.data, size_t(b.payload_len), kSectionGraph, &sec, &sec_len))
      fail(STRATA_INVALID_ARGUMENT, "the subgraph blob carries no graph section");
    auto holder = compile_graph_section(sec, sec_len);
    if (!holder) return STRATA_DECLINED;  // nothing allocated
    *out_exe = holder.release();
    return STRATA_OK;
  });
}

// ---------------------------------------------------------------------------
// Ahead-of-time executables (raw.rs:760-788; the reference host does not call
// these yet).  A serialised executable is a framed blob with two sections:
//   kSectionB200Exe  u32 format version, u32 SM architecture (100),
//                    u32 ABI major, u32 ABI minor, u64 plan fingerprint,
//                    u32 steps, u64 workspace bytes, str label
//   kSectionGraph    the executable's graph, in the reference's encoding.
// Loading decodes and lowers the graph again and accepts the result only if
// its plan has the recorded fingerprint, so a blob from a build that lowers
// differently is refused rather than run.  Weights and caches stay run-time
// buffers; CUDA graphs are captured on the loaded executable's first run.
// abi_compatible answers OK or INVALID_ARGUMENT and touches no device.
// ---------------------------------------------------------------------------

constexpr uint32_t kExeFormat = 1, kExeArch = 100;

// FNV-1a over everything the lowering decided.
static uint64_t plan_fingerprint(const Exe& e) {
  uint64_t h = 1469598103934665603ull;
  auto mix = [&](uint64_t x) {
    for (int k = 0; k < 8; ++k) {
      h ^= (x >> (8 * k)) & 0xff;
      h *= 1099511628211ull;
    }
  };
  mix(e.steps.size());
  mix(e.ws_bytes);
  for (const Step& st : e.steps) {
    mix(uint64_t(st.kind));
    mix(st.bf16);
    mix(st.v.size());
    for (uint32_t v : st.v) mix(v);
    for (int64_t i : st.i) mix(uint64_t(i));
    uint64_t dbits;
    std::memcpy(&dbits, &st.d, sizeof dbits);
    mix(dbits);
    mix(uint64_t(st.fmt));
    mix(uint64_t(st.epi));
    mix(uint64_t(st.njobs));
    mix(st.scratch_bytes);
    for (uint32_t v : st.reads) mix(v);
    for (uint32_t v : st.writes) mix(v);
  }
  return h;
}

struct ExeHeader {
  uint32_t format = 0, arch = 0, abi_major = 0, abi_minor = 0;
  uint64_t fingerprint = 0;
  uint32_t steps = 0;
  uint64_t ws_bytes = 0;
  std::string label;
};

static ExeHeader read_exe_header(const StrataWireBlob& b) {
  check_blob_header(b, "executable");
  const uint8_t* sec = nullptr;
  size_t n = 0;
  if (!find_section(b.data, size_t(b.payload_len), kSectionB200Exe, &sec, &n))
    fail(STRATA_INVALID_ARGUMENT, "the blob is not a serialised B200 executable");
  Reader r(sec, n);
  ExeHeader h;
  h.format = r.u32();
  h.arch = r.u32();
  h.abi_major = r.u32();
  h.abi_minor = r.u32();
  h.fingerprint = r.u64();
  h.steps = r.u32();
  h.ws_bytes = r.u64();
  h.label = r.str();
  if (h.format != kExeFormat) fail(STRATA_INVALID_ARGUMENT, "unknown serialised-executable format");
  if (h.arch != kExeArch) fail(STRATA_INVALID_ARGUMENT, "the executable was built for another architecture");
  if (h.abi_major != STRATA_ABI_MAJOR || h.abi_minor > STRATA_ABI_MINOR)
    fail(STRATA_INVALID_ARGUMENT, "the executable was serialised under an incompatible ABI");
  return h;
}

static int32_t sb_serialize(void* ctx, const StrataExecutable* e, StrataWireBlob* out) {
  if (!ctx || !e || !out) return STRATA_INVALID_ARGUMENT;
  try {
    Writer hw;
    hw.u32(kExeFormat);
    hw.u32(kExeArch);
    hw.u32(STRATA_ABI_MAJOR);
    hw.u32(STRATA_ABI_MINOR);
    hw.u64(plan_fingerprint(e->exe));
    hw.u32(uint32_t(e->exe.steps.size()));
    hw.u64(e->exe.ws_bytes);
    hw.str(e->exe.label);
    const std::vector<uint8_t> framed =
        frame_sections({{kSectionB200Exe, std::move(hw.data())}, {kSectionGraph, encode_graph(e->exe.g)}});
    uint8_t* data = new uint8_t[framed.size() + 1];
    std::memcpy(data, framed.data(), framed.size());
    data[framed.size()] = 0;
    out->magic = kMagic;
    out->format_major = kFormatMajor;
    out->format_minor = kFormatMinor;
    out->payload_len = framed.size();
    out->data = data;
    out->nul = 0;
    return STRATA_OK;
  } catch (const Failure& f) {
    return f.code;
  } catch (...) {
    return STRATA_INTERNAL;
  }
}

static int32_t sb_abi_compatible(void* ctx, const StrataWireBlob* blob) {
  if (!ctx || !blob) return STRATA_INVALID_ARGUMENT;
  try {
    read_exe_header(*blob);
    const uint8_t* sec = nullptr;
    size_t n = 0;
    if (!find_section(blob->data, size_t(blob->payload_len), kSectionGraph, &sec, &n))
      return STRATA_INVALID_ARGUMENT;
    return STRATA_OK;
  } catch (const Failure& f) {
    return f.code;
  } catch (...) {
    return STRATA_INVALID_ARGUMENT;
  }
}

static int32_t sb_deserialize_load(void* ctx, const StrataWireBlob* blob, StrataExecutable** out_exe) {
  if (out_exe) *out_exe = nullptr;
  if (!ctx || !blob || !out_exe) return STRATA_INVALID_ARGUMENT;
  try {
    const ExeHeader h = read_exe_header(*blob);
    const uint8_t* sec = nullptr;
    size_t n = 0;
    if (!find_section(blob->data, size_t(blob->payload_len), kSectionGraph, &sec, &n))
      return STRATA_INVALID_ARGUMENT;
    auto holder = compile_graph_section(sec, n);
    if (!holder || plan_fingerprint(holder->exe) != h.fingerprint || holder->exe.steps.size() != h.steps)
      return STRATA_INVALID_ARGUMENT;  // this build lowers the graph differently
    *out_exe = holder.release();
    return STRATA_OK;
  } catch (const Failure& f) {
    return f.code;
  } catch (const WireError&) {
    return STRATA_INVALID_ARGUMENT;
  } catch (...) {
    return STRATA_INTERNAL;
  }
}

// ---------------------------------------------------------------------------
// Buffers and events (raw.rs:659-725)
// ---------------------------------------------------------------------------

static int32_t sb_alloc(void* ctx, const StrataAllocDesc* d, StrataBuffer** out, StrataError** out_error) {
  if (out) *out = nullptr;
  if (out_error) *out_error = nullptr;
  return guarded(out_error, [&]() -> int32_t {
    Ctx* c = C(ctx);
    if (!d || !out) fail(STRATA_INVALID_ARGUMENT, "alloc needs a descriptor and an out-parameter");
    if (d->struct_size < sizeof(StrataAllocDesc)) fail(STRATA_INVALID_ARGUMENT, "StrataAllocDesc is too short");
    if (d->rank > 8 || (d->rank && !d->dims)) fail(STRATA_INVALID_ARGUMENT, "bad rank or dims");
    DType dt;
    dt.elem = d->dtype.element;
    uint64_t n = 1;
    for (uint32_t i = 0; i < d->rank; ++i) {
      if (d->dims[i] && n > (uint64_t(1) << 46) / d->dims[i])
        fail(STRATA_RESOURCE_EXHAUSTED, "allocation size overflows");
      n *= d->dims[i];
    }
    const uint64_t bytes = dt.byte_len(n);
    std::lock_guard<std::mutex> lk(c->mu);
    c->ensure_device();
    auto buf = std::make_unique<StrataBuffer>();
    buf->b.ptr = device_alloc(*c, bytes);
    buf->b.bytes = bytes;
    buf->b.owned = true;
    *out = buf.release();
    return STRATA_OK;
  });
}

static int32_t sb_buffer_release(void* ctx, StrataBuffer* b) {
  if (!ctx || !b) return STRATA_INVALID_ARGUMENT;
  Ctx* c = static_cast<Ctx*>(ctx);
  std::lock_guard<std::mutex> lk(c->mu);
  if (b->b.owned && b->b.ptr) {
    // The stream may still be reading it; release only after queued work.
    if (c->device_ready) cudaStreamSynchronize(c->stream);
    device_free(*c, b->b.bytes, b->b.ptr);
  }
  delete b;
  return STRATA_OK;
}

static int32_t sb_buffer_write(void* ctx, StrataBuffer* b, uint64_t offset, const uint8_t* data, uint64_t len) {
  if (!ctx || !b || (!data && len)) return STRATA_INVALID_ARGUMENT;
  if (offset > b->b.bytes || len > b->b.bytes - offset) return STRATA_INVALID_ARGUMENT;
  if (len == 0) return STRATA_OK;
  try {
    Ctx* c = C(ctx);
    std::lock_guard<std::mutex> lk(c->mu);
    c->ensure_device();
    cuda_check(cudaMemcpyAsync(static_cast<char*>(b->b.ptr) + offset, data, size_t(len), cudaMemcpyHostToDevice,
                               c->stream),
               "buffer_write");
    cuda_check(cudaStreamSynchronize(c->stream), "buffer_write");
    return STRATA_OK;
  } catch (const Failure& f) {
    return f.code;
  }
}

static int32_t sb_buffer_read(void* ctx, const StrataBuffer* b, uint64_t offset, uint8_t* data, uint64_t len) {
  if (!ctx || !b || (!data && len)) return STRATA_INVALID_ARGUMENT;
  if (offset > b->b.bytes || len > b->b.bytes - offset) return STRATA_INVALID_ARGUMENT;
  if (len == 0) return STRATA_OK;
  try {
    Ctx* c = C(ctx);
    std::lock_guard<std::mutex> lk(c->mu);
    c->ensure_device();
    cuda_check(cudaMemcpyAsync(data, static_cast<const char*>(b->b.ptr) + offset, size_t(len),
                               cudaMemcpyDeviceToHost, c->stream),
               "buffer_read");
    cuda_check(cudaStreamSynchronize(c->stream), "buffer_read");
    return STRATA_OK;
  } catch (const Failure& f) {
    return f.code;
  }
}

static int32_t sb_buffer_event(void* ctx, const StrataBuffer* b, StrataEvent** out) {
  if (!ctx || !b || !out) return STRATA_INVALID_ARGUMENT;
  try {
    Ctx* c = C(ctx);
    std::lock_guard<std::mutex> lk(c->mu);
    c->ensure_device();
    auto ev = std::make_unique<StrataEvent>();
    cuda_check(cudaEventCreateWithFlags(&ev->ev, cudaEventDisableTiming), "cudaEventCreate");
    cuda_check(cudaEventRecord(ev->ev, c->stream), "cudaEventRecord");
    *out = ev.release();
    return STRATA_OK;
  } catch (const Failure& f) {
    return f.code;
  }
}

static int32_t sb_event_ready(void* ctx, const StrataEvent* e) {
  if (!ctx || !e) return STRATA_INVALID_ARGUMENT;
  const cudaError_t r = cudaEventQuery(e->ev);
  if (r == cudaSuccess) return 1;
  if (r == cudaErrorNotReady) {
    cudaGetLastError();
    return 0;
  }
  return STRATA_INTERNAL;
}

static int32_t sb_event_await(void* ctx, const StrataEvent* e) {
  if (!ctx || !e) return STRATA_INVALID_ARGUMENT;
  return cudaEventSynchronize(e->ev) == cudaSuccess ? STRATA_OK : STRATA_INTERNAL;
}

static int32_t sb_event_free(void* ctx, StrataEvent* e) {
  if (!ctx || !e) return STRATA_INVALID_ARGUMENT;
  cudaEventDestroy(e->ev);
  delete e;
  return STRATA_OK;
}

// ---------------------------------------------------------------------------
// Run (raw.rs:727-735)
// ---------------------------------------------------------------------------

namespace {

// Enqueue one run on the context's stream.  Caller holds c.mu.
void enqueue_run(Ctx& c, const StrataRunArgs* a) {
  if (!a) fail(STRATA_INVALID_ARGUMENT, "run needs arguments");
  if (a->struct_size < sizeof(StrataRunArgs)) fail(STRATA_INVALID_ARGUMENT, "StrataRunArgs is too short");
  if (!a->executable) fail(STRATA_INVALID_ARGUMENT, "run was given a null executable");
  if (a->arg_count && !a->args) fail(STRATA_INVALID_ARGUMENT, "run was given a null argument array");
  Exe& e = const_cast<StrataExecutable*>(a->executable)->exe;
  const size_t nv = e.g.values.size();
  std::vector<void*> ext(nv, nullptr);
  for (uint32_t i = 0; i < a->arg_count; ++i) {
    const StrataBufferRef& r = a->args[i];
    if (r.value_index >= nv)
      fail(STRATA_INVALID_ARGUMENT, "argument names value " + std::to_string(r.value_index) +
                                        ", which this executable does not have");
    if (!r.buffer) continue;
    const uint32_t v = r.value_index;
    const bool is_in = e.g.values[v].producer < 0 || e.needed_input[v];
    const bool is_out = e.is_output[v];
    if (!is_in && !is_out) continue;  // intermediates live in the plugin's workspace
    if (r.buffer->b.bytes < e.g.values[v].bytes())
      fail(STRATA_INVALID_ARGUMENT, "the buffer for `" + e.g.values[v].name + "` holds " +
                                        std::to_string(r.buffer->b.bytes) + " bytes, it needs " +
                                        std::to_string(e.g.values[v].bytes()));
    ext[v] = r.buffer->b.ptr;
  }
  for (size_t v = 0; v < nv; ++v)
    if (e.needed_input[v] && !ext[v] && e.g.values[v].bytes() > 0)
      fail(STRATA_INVALID_ARGUMENT, "no buffer for input `" + e.g.values[v].name + "` of `" + e.label + "`");
  c.ensure_device();
  if (!e.ws && e.ws_bytes) {
    cuda_check(cudaMalloc(&e.ws, e.ws_bytes), "workspace cudaMalloc");
    if (!e.consts.empty())
      cuda_check(cudaMemcpy(static_cast<char*>(e.ws) + e.consts_off, e.consts.data(), e.consts.size(),
                            cudaMemcpyHostToDevice),
                 "uploading the executable's constants");
  }

  if (!graphs_enabled()) {
    enqueue(c, e, ext);
    return;
  }
  for (auto& cg : e.graphs) {
    if (cg.key == ext) {
      cuda_check(cudaGraphLaunch(cg.exec, c.stream), "cudaGraphLaunch");
      sb::count_launch(cg.kernels);
      return;
    }
  }
  if (ext != e.last_key) {
    // First time with these pointers: run eagerly, capture if they repeat.
    e.last_key = ext;
    enqueue(c, e, ext);
    return;
  }
  cuda_check(cudaStreamBeginCapture(c.stream, cudaStreamCaptureModeThreadLocal), "cudaStreamBeginCapture");
  const uint64_t before = sb::g_launches.load();
  try {
    enqueue(c, e, ext);
  } catch (...) {
    cudaGraph_t dead = nullptr;
    cudaStreamEndCapture(c.stream, &dead);
    if (dead) cudaGraphDestroy(dead);
    cudaGetLastError();
    throw;
  }
  const uint64_t kernels = sb::g_launches.load() - before;
  sb::g_launches.fetch_sub(kernels);
  cudaGraph_t graph = nullptr;
  cuda_check(cudaStreamEndCapture(c.stream, &graph), "cudaStreamEndCapture");
  cudaGraphExec_t exec = nullptr;
  const cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
  cudaGraphDestroy(graph);
  cuda_check(ie, "cudaGraphInstantiate");
  if (e.graphs.size() >= 4) {
    cudaGraphExecDestroy(e.graphs.front().exec);
    e.graphs.erase(e.graphs.begin());
  }
  e.graphs.push_back(Exe::Cached{ext, exec, kernels});
  cuda_check(cudaGraphLaunch(exec, c.stream), "cudaGraphLaunch");
  sb::count_launch(kernels);
}

void copy_to_host_arena(Ctx& c, const StrataRunArgs* a) {
  if (!a->host_arena || !a->host_arena->entries) return;
  const Exe& e = a->executable->exe;
  // Entries are indexed by value index; an output whose entry is present and
  // sized for it is copied out.
  std::vector<void*> ext(e.g.values.size(), nullptr);
  for (uint32_t i = 0; i < a->arg_count; ++i)
    if (a->args[i].buffer && a->args[i].value_index < ext.size())
      ext[a->args[i].value_index] = a->args[i].buffer->b.ptr;
  for (auto o : e.g.outputs) {
    if (o >= a->host_arena->entry_count) continue;
    StrataArenaEntryView& ent = a->host_arena->entries[o];
    if (!ent.data || ent.element_count != uint64_t(e.g.values[o].elements())) continue;
    const uint32_t b = e.alias[o];
    const void* src = ext[o] ? ext[o] : (e.ws_off[b] >= 0 ? static_cast<const char*>(e.ws) + e.ws_off[b] : nullptr);
    if (!src) continue;
    cuda_check(cudaMemcpyAsync(ent.data, src, e.g.values[o].bytes(), cudaMemcpyDeviceToHost, c.stream),
               "host arena copy");
  }
  cuda_check(cudaStreamSynchronize(c.stream), "host arena copy");
}

}  // namespace

static int32_t sb_run(void* ctx, const StrataRunArgs* a, StrataError** out_error) {
  if (out_error) *out_error = nullptr;
  return guarded(out_error, [&]() -> int32_t {
    Ctx* c = C(ctx);
    std::lock_guard<std::mutex> lk(c->mu);
    enqueue_run(*c, a);
    cuda_check(cudaStreamSynchronize(c->stream), "run");
    c->check_device_error(a->executable->exe.label.c_str());
    copy_to_host_arena(*c, a);
    return STRATA_OK;
  });
}

static int32_t sb_run_async(void* ctx, const StrataRunArgs* a, StrataError** out_error) {
  if (out_error) *out_error = nullptr;
  return guarded(out_error, [&]() -> int32_t {
    Ctx* c = C(ctx);
    std::lock_guard<std::mutex> lk(c->mu);
    enqueue_run(*c, a);
    return STRATA_OK;
  });
}

static int32_t sb_synchronize(void* ctx, StrataError** out_error) {
  if (out_error) *out_error = nullptr;
  return guarded(out_error, [&]() -> int32_t {
    Ctx* c = C(ctx);
    std::lock_guard<std::mutex> lk(c->mu);
    c->ensure_device();
    cuda_check(cudaStreamSynchronize(c->stream), "synchronize");
    c->check_device_error("synchronize");
    return STRATA_OK;
  });
}

// ---------------------------------------------------------------------------
// Teardown (raw.rs:737-757)
// ---------------------------------------------------------------------------

static void sb_free_executable(void* ctx, StrataExecutable* e) {
  if (!e) return;
  if (ctx) {
    Ctx* c = static_cast<Ctx*>(ctx);
    std::lock_guard<std::mutex> lk(c->mu);
    if (c->device_ready) cudaStreamSynchronize(c->stream);
  }
  delete e;
}

static void sb_free_blob(void* ctx, StrataWireBlob* blob) {
  (void)ctx;
  if (!blob) return;
  delete[] const_cast<uint8_t*>(blob->data);
  blob->data = nullptr;
}

static void* sb_plugin_init(void) {
  auto* c = new (std::nothrow) Ctx;
  if (!c) return nullptr;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess) {
    cudaGetLastError();
    count = 0;
  }
  c->has_device = count > 0;
  c->device = env_int("STRATA_B200_DEVICE", env_int("LOCAL_RANK", 0));
  if (c->has_device) {
    if (c->device >= count) c->device = c->device % count;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, c->device) == cudaSuccess) {
      c->device_name = prop.name;
      c->memory_bytes = prop.totalGlobalMem;
    }
  }
  return c;
}

static void sb_plugin_free(void* ctx) {
  if (!ctx) return;
  Ctx* c = static_cast<Ctx*>(ctx);
  if (c->device_ready) {
    cudaSetDevice(c->device);
    cudaStreamSynchronize(c->stream);
    c->teardown_allreduce();
    if (c->comm) c->nccl.comm_destroy(c->comm);
    g_pool.drain(c->device);
    cudaFree(c->d_err);
    cudaStreamDestroy(c->stream);
  }
  delete c;
}

// ---------------------------------------------------------------------------
// Extension chain: plugin version, then the B200 device extension
// ---------------------------------------------------------------------------

static int32_t ext_buffer_wrap(void* ctx, void* ptr, uint64_t bytes, StrataBuffer** out) {
  if (!ctx || !out || (!ptr && bytes)) return STRATA_INVALID_ARGUMENT;
  auto* b = new (std::nothrow) StrataBuffer;
  if (!b) return STRATA_RESOURCE_EXHAUSTED;
  b->b.ptr = ptr;
  b->b.bytes = bytes;
  b->b.owned = false;
  *out = b;
  return STRATA_OK;
}

static int32_t ext_buffer_device_ptr(void* ctx, const StrataBuffer* b, void** out_ptr, uint64_t* out_bytes) {
  if (!ctx || !b) return STRATA_INVALID_ARGUMENT;
  if (out_ptr) *out_ptr = b->b.ptr;
  if (out_bytes) *out_bytes = b->b.bytes;
  return STRATA_OK;
}

static void* ext_stream(void* ctx) {
  if (!ctx) return nullptr;
  Ctx* c = static_cast<Ctx*>(ctx);
  try {
    std::lock_guard<std::mutex> lk(c->mu);
    c->ensure_device();
  } catch (...) {
    return nullptr;
  }
  return c->stream;
}

static uint64_t ext_launch_count(void* ctx) {
  (void)ctx;
  return sb::g_launches.load();
}

static int32_t ext_tp_unique_id(void* ctx, uint8_t out[128]) {
  if (!ctx || !out) return STRATA_INVALID_ARGUMENT;
  Ctx* c = static_cast<Ctx*>(ctx);
  std::string why;
  if (!c->nccl.load(&why)) return STRATA_UNIMPLEMENTED;
  ncclUniqueId id;
  if (c->nccl.get_unique_id(&id) != ncclSuccess) return STRATA_INTERNAL;
  static_assert(sizeof(id) == 128, "ncclUniqueId is 128 bytes");
  std::memcpy(out, &id, 128);
  return STRATA_OK;
}

static int32_t ext_tp_init(void* ctx, int32_t rank, int32_t world, const uint8_t id[128], StrataError** out_error) {
  if (out_error) *out_error = nullptr;
  return guarded(out_error, [&]() -> int32_t {
    Ctx* c = C(ctx);
    if (!id || world < 1 || rank < 0 || rank >= world) fail(STRATA_INVALID_ARGUMENT, "bad tensor-parallel rank");
    std::lock_guard<std::mutex> lk(c->mu);
    c->ensure_device();
    if (world == 1) {
      c->rank = 0;
      c->world = 1;
      return STRATA_OK;
    }
    std::string why;
    if (!c->nccl.load(&why)) fail(STRATA_UNIMPLEMENTED, why);
    ncclUniqueId uid;
    std::memcpy(&uid, id, 128);
    ncclComm_t comm = nullptr;
    const ncclResult_t r = c->nccl.comm_init_rank(&comm, world, uid, rank);
    if (r != ncclSuccess) fail(STRATA_INTERNAL, std::string("ncclCommInitRank: ") + c->nccl.error_string(r));
    c->comm = comm;
    c->rank = rank;
    c->world = world;
    c->setup_allreduce();
    return STRATA_OK;
  });
}

static int32_t ext_set_device(void* ctx, int32_t device) {
  if (!ctx) return STRATA_INVALID_ARGUMENT;
  Ctx* c = static_cast<Ctx*>(ctx);
  std::lock_guard<std::mutex> lk(c->mu);
  if (c->device_ready && c->device != device) return STRATA_INVALID_ARGUMENT;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || device < 0 || device >= count) {
    cudaGetLastError();
    return STRATA_INVALID_ARGUMENT;
  }
  c->device = device;
  cudaDeviceProp prop;
  if (cudaGetDeviceProperties(&prop, device) == cudaSuccess) {
    c->device_name = prop.name;
    c->memory_bytes = prop.totalGlobalMem;
  }
  c->caps.clear();
  return STRATA_OK;
}

static StrataB200DeviceExt g_device_ext = {
    {sizeof(StrataB200DeviceExt), STRATA_B200_EXT_DEVICE, nullptr},
    STRATA_B200_EXT_DEVICE_VERSION,
    0,
    ext_buffer_wrap,
    ext_buffer_device_ptr,
    sb_run_async,
    sb_synchronize,
    ext_stream,
    ext_launch_count,
    ext_tp_unique_id,
    ext_tp_init,
    ext_set_device,
};

static StrataPluginVersionExt g_version_ext = {
    {sizeof(StrataPluginVersionExt), STRATA_EXT_PLUGIN_VERSION,
     reinterpret_cast<StrataExtBase*>(&g_device_ext)},
    0,
    1,
    0,
    {STRATA_ABI_MAJOR, STRATA_ABI_MINOR},
};

extern "C" {
// Per-class device time of the steps run since the last reset (see
// step_times_enabled), as JSON into buf (NUL-terminated when it fits).
// Returns the bytes the JSON needs, without the NUL.
__attribute__((visibility("default"))) uint64_t strata_b200_step_times(char* buf, uint64_t cap, int32_t reset) {
  const std::string j = sbp::step_times_json(reset != 0);
  if (buf && cap) {
    const size_t n = j.size() < cap ? j.size() : size_t(cap - 1);
    std::memcpy(buf, j.data(), n);
    buf[n] = '\0';
  }
  return j.size();
}

__attribute__((visibility("default"))) StrataPluginV1 strata_plugin_v1 = {
    sizeof(StrataPluginV1),
    reinterpret_cast<StrataExtBase*>(&g_version_ext),
    {STRATA_ABI_MAJOR, STRATA_ABI_MINOR},
    sb_error_free,
    sb_error_code,
    sb_error_payload,
    sb_capabilities,
    sb_supports,
    sb_compile,
    sb_alloc,
    sb_buffer_release,
    sb_buffer_write,
    sb_buffer_read,
    sb_buffer_event,
    sb_event_ready,
    sb_event_await,
    sb_event_free,
    sb_run,
    sb_free_executable,
    sb_free_blob,
    sb_plugin_init,
    sb_plugin_free,
    sb_serialize,
    sb_deserialize_load,
    sb_abi_compatible,
};
}  // extern "C"
