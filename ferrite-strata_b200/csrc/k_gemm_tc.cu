// Tensor-core GEMM on the 5th-generation tensor cores (tcgen05, TMEM, TMA)
// for prefill-sized batches:
//
//   y[m, n] = scale[n] * sum_k x[m, k] * w[n, k]   (+ residual[m, n])
//
// x and w are bf16 and K-major (row-major [M, K] and [N, K]); int8 weights
// reach this kernel as their exact bf16 codes (prepared once per launch by
// launch_codes_to_bf16), so the per-channel scale is applied in f32 in the
// epilogue and the product matches the oracle's code * scale.
//
// Persistent: one CTA per SM walks 128 x BN tiles of y (tokens x features; BN
// 256 for prefill-sized launches, down to 32 for small ones, choose_bn):
//   warp 0      one thread issues TMA loads of the x tile (128 x 64) and the
//               w tile (BN x 64), 128-byte swizzled, into a 4- to 8-stage
//               ring that runs continuously across the CTA's tiles;
//   warp 1      allocates 2 BN TMEM columns (two f32 accumulators: TMEM lane =
//               token row, column = feature) and one thread issues
//               tcgen05.mma (M 128, N BN, K 16; four per stage) and
//               tcgen05.commit to release each stage and each finished
//               accumulator;
//   warps 2-5   the epilogue: tcgen05.ld 32 columns at a time from their
//               TMEM lane quarter, scale, residual or SwiGLU, bf16 -- while
//               the MMA thread already fills the other accumulator.
// Every mbarrier wait is bounded; a wait that runs out records error code 4
// in *err and the CTA winds down (the TMEM owner still frees its columns).
#include <cuda.h>

#include <mutex>

#include "common.cuh"
#include "k_elem.cuh"
#include "k_int4.cuh"
#include "k_tc.cuh"

namespace sb {

namespace {

constexpr int kBM = 128, kBK = 64;
constexpr int kGThreads = 192;
constexpr int kABytes = kBM * kBK * 2;            // 16 KB

// Tile width BN (256, 128, 64 or 32 weight rows): narrower tiles give small-M
// launches enough tiles to fill the SMs, and use the shared memory they free
// for a deeper ring.
template <int BN>
struct GL {
  static constexpr int kBBytes = BN * kBK * 2;                                  // 32 KB at BN = 256
  static constexpr int kStageBytes = kABytes + kBBytes;
  static constexpr int kStages = BN == 256 ? 4 : BN == 128 ? 6 : 8;
  static constexpr int kSmem = kStages * kStageBytes + 1024 + 256;             // ring + alignment + barriers
  static constexpr uint32_t kTmemCols = 2 * BN;                                // two f32 accumulators
  static constexpr uint32_t kIdesc = tc::idesc_bf16(kBM, BN);
};

struct GemmArgs {
  int m, n, k;               // n: output features (for SwiGLU: of the gate and of the up matrix)
  const float* scale;        // [n] or null (SwiGLU: gate scales)
  const float* scale2;       // SwiGLU: up scales [n] or null
  const uint16_t* residual;  // [m, ldr] or null
  int ldr;
  uint16_t* y;               // [m, ldy]
  int ldy;
  int* err;
};

using namespace tc;

// Epilogue of one tile for one token row: TMEM columns [col0, col0 + BN) of
// this warp's lane quarter.  EPI 0: y = scale * acc (+ residual); EPI 1: the
// gate in columns 0..BN/2-1 and the up in BN/2..BN-1, each rounded to bf16 as
// the graph's gate and up values are, then silu(gate) * up.
template <int EPI, int BN>
__device__ __forceinline__ void gemm_epilogue(const GemmArgs& p, uint32_t taddr, int row, int n0) {
  if constexpr (EPI == 1) {
    for (int c = 0; c < BN / 64; ++c) {
      uint32_t gr[32], ur[32];
      tmem_ld32(taddr + uint32_t(c * 32), gr);
      tmem_ld32(taddr + uint32_t(BN / 2 + c * 32), ur);
      const int nb = n0 + c * 32;
      if (row >= p.m || nb >= p.n) continue;
      uint16_t* yr = p.y + int64_t(row) * p.ldy + nb;
      float out[32];
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        const int n = nb + j < p.n ? nb + j : p.n - 1;
        float g = __uint_as_float(gr[j]), u = __uint_as_float(ur[j]);
        if (p.scale) g *= p.scale[n];
        if (p.scale2) u *= p.scale2[n];
        g = bf2f(f2bf(g));
        u = bf2f(f2bf(u));
        out[j] = (g / (1.0f + expf(-g))) * u;
      }
      if (nb + 32 <= p.n && (reinterpret_cast<uintptr_t>(yr) & 15) == 0) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            w[e] = uint32_t(f2bf(out[8 * v + 2 * e])) | (uint32_t(f2bf(out[8 * v + 2 * e + 1])) << 16);
          *reinterpret_cast<uint4*>(yr + 8 * v) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      } else {
        for (int j = 0; j < 32 && nb + j < p.n; ++j) yr[j] = f2bf(out[j]);
      }
    }
  } else {
    for (int c = 0; c < BN / 32; ++c) {
      uint32_t r[32];
      tmem_ld32(taddr + uint32_t(c * 32), r);
      const int nb = n0 + c * 32;
      if (row >= p.m || nb >= p.n) continue;
      uint16_t* yr = p.y + int64_t(row) * p.ldy + nb;
      const uint16_t* rr = p.residual ? p.residual + int64_t(row) * p.ldr + nb : nullptr;
      if (nb + 32 <= p.n && (reinterpret_cast<uintptr_t>(yr) & 15) == 0 &&
          (!rr || (reinterpret_cast<uintptr_t>(rr) & 15) == 0)) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint32_t w[4];
          const uint4 res = rr ? *reinterpret_cast<const uint4*>(rr + 8 * v) : make_uint4(0, 0, 0, 0);
          const uint32_t rw[4] = {res.x, res.y, res.z, res.w};
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const int j = 8 * v + 2 * e;
            float lo = __uint_as_float(r[j]), hi = __uint_as_float(r[j + 1]);
            if (p.scale) {
              lo *= p.scale[nb + j];
              hi *= p.scale[nb + j + 1];
            }
            if (rr) {
              lo = bf2f(f2bf(lo)) + bf_lo(rw[e]);
              hi = bf2f(f2bf(hi)) + bf_hi(rw[e]);
            }
            w[e] = uint32_t(f2bf(lo)) | (uint32_t(f2bf(hi)) << 16);
          }
          *reinterpret_cast<uint4*>(yr + 8 * v) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      } else {
        for (int j = 0; j < 32 && nb + j < p.n; ++j) {
          float v = __uint_as_float(r[j]);
          if (p.scale) v *= p.scale[nb + j];
          if (rr) v = bf2f(f2bf(v)) + bf2f(rr[j]);
          yr[j] = f2bf(v);
        }
      }
    }
  }
}

// Persistent: CTA b computes tiles b, b + grid, ... (features fastest, so a
// wave of CTAs shares its x rows and walks all of W).  Two TMEM accumulators
// of BN columns alternate between tiles: the epilogue warps drain tile i
// while the MMA thread fills the other accumulator with tile i + 1.
//
// EPI 0: y = scale * (x W^T) (+ residual).  EPI 1 (SwiGLU): the B tile is
// BN/2 rows of the gate matrix over BN/2 rows of the up matrix for the same
// output features, and y = silu(gate) * up for those BN/2 features.
template <int EPI, int BN>
__global__ void __launch_bounds__(kGThreads, 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap tmap_x, const __grid_constant__ CUtensorMap tmap_w,
                   const __grid_constant__ CUtensorMap tmap_w2, const GemmArgs p) {
  using L = GL<BN>;
  constexpr int kGStages = L::kStages, kGStageBytes = L::kStageBytes, kBBytes = L::kBBytes;
  constexpr uint32_t kTmemCols = L::kTmemCols, kIdesc = L::kIdesc;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kGStages * kGStageBytes);
  uint64_t* empty = full + kGStages;
  uint64_t* acc_full = empty + kGStages;   // [2]: accumulator b holds a finished tile
  uint64_t* acc_empty = acc_full + 2;      // [2]: the epilogue has drained accumulator b
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  __shared__ int s_fail;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  constexpr int kOutCols = EPI == 1 ? BN / 2 : BN;  // output features per tile
  const int tiles_n = (p.n + kOutCols - 1) / kOutCols;
  const int tiles = tiles_n * ((p.m + kBM - 1) / kBM);
  const int nk = (p.k + kBK - 1) / kBK;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kGStages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], kGThreads / 32 - 2);  // one arrival per epilogue warp
    }
    s_fail = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                 "r"(kTmemCols)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
  const uint32_t tmem = *tmem_slot;
  pdl_trigger();
  pdl_wait();  // x comes from the previous kernel

  if (warp == 0) {
    if (lane == 0) {
      // Producer: one continuous ring over every (tile, k-block) of this CTA.
      uint32_t c = 0;
      bool ok = true;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x) {
        const int m0 = (t / tiles_n) * kBM, n0 = (t % tiles_n) * kOutCols;
        for (int kb = 0; kb < nk; ++kb, ++c) {
          const int s = int(c % kGStages);
          if (!mbar_wait(&empty[s], ((c / kGStages) & 1) ^ 1)) {  // first pass: free
            atomicExch(&s_fail, 1);
            ok = false;
            break;
          }
          uint8_t* sa = smem + s * kGStageBytes;
          mbar_expect_tx(&full[s], kGStageBytes);
          tma_load_2d(sa, &tmap_x, &full[s], kb * kBK, m0);
          if constexpr (EPI == 1) {
            tma_load_2d(sa + kABytes, &tmap_w, &full[s], kb * kBK, n0);
            tma_load_2d(sa + kABytes + kBBytes / 2, &tmap_w2, &full[s], kb * kBK, n0);
          } else {
            tma_load_2d(sa + kABytes, &tmap_w, &full[s], kb * kBK, n0);
          }
        }
      }
      // Let the copies still in flight land before the CTA can exit.
      for (uint32_t d = c >= kGStages ? c - kGStages : 0; d < c; ++d)
        mbar_wait(&full[d % kGStages], (d / kGStages) & 1);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      // MMA issuer.
      uint32_t c = 0;
      bool ok = true;
      int i = 0;
      for (int t = blockIdx.x; ok && t < tiles; t += gridDim.x, ++i) {
        const int b = i & 1;
        if (!mbar_wait(&acc_empty[b], ((i >> 1) & 1) ^ 1)) {  // first use of each accumulator: free
          atomicExch(&s_fail, 1);
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
        const uint32_t acc = tmem + uint32_t(b * BN);
        for (int kb = 0; kb < nk; ++kb, ++c) {
          const int s = int(c % kGStages);
          if (!mbar_wait(&full[s], (c / kGStages) & 1)) {
            atomicExch(&s_fail, 1);
            ok = false;
            break;
          }
          asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
          const uint8_t* sa = smem + s * kGStageBytes;
          const uint64_t da = sw128_desc(sa), db = sw128_desc(sa + kABytes);
#pragma unroll
          for (int kk = 0; kk < kBK / 16; ++kk)  // +32 bytes along K per step
            umma_bf16(acc, da + uint64_t(2 * kk), db + uint64_t(2 * kk), kIdesc, (kb | kk) != 0);
          umma_commit(&empty[s]);
        }
        if (ok) umma_commit(&acc_full[b]);
      }
    }
  } else {
    // Epilogue warps 2..5: TMEM lane quarter = warp % 4.
    const int quarter = warp & 3;
    int i = 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++i) {
      const int b = i & 1;
      if (!mbar_wait_warp(&acc_full[b], (i >> 1) & 1)) {
        atomicExch(&s_fail, 1);
        break;
      }
      asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
      const int m0 = (t / tiles_n) * kBM, n0 = (t % tiles_n) * kOutCols;
      gemm_epilogue<EPI, BN>(p, tmem + (uint32_t(quarter * 32) << 16) + uint32_t(b * BN), m0 + quarter * 32 + lane,
                             n0);
      asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
  __syncthreads();
  if (warp == 1) {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols) : "memory");
  }
  if (threadIdx.x == 0 && s_fail && p.err) atomicExch(p.err, 4);
}

// int8 codes (or int4 codes times their bf16 group scale) as bf16 [n, k].
__global__ void codes_i8_to_bf16_kernel(const int8_t* __restrict__ q, int64_t count, uint16_t* __restrict__ out) {
  pdl_trigger();
  pdl_wait();  // `out` may still be read by the previous GEMM
  const int64_t n8 = count / 8;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n8; i += int64_t(gridDim.x) * blockDim.x) {
    const uint2 v = __ldg(reinterpret_cast<const uint2*>(q) + i);
    const int8_t* b = reinterpret_cast<const int8_t*>(&v);
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e)
      w[e] = uint32_t(f2bf(float(b[2 * e]))) | (uint32_t(f2bf(float(b[2 * e + 1]))) << 16);
    reinterpret_cast<uint4*>(out)[i] = make_uint4(w[0], w[1], w[2], w[3]);
  }
  for (int64_t i = n8 * 8 + blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < count;
       i += int64_t(gridDim.x) * blockDim.x)
    out[i] = f2bf(float(q[i]));
}

__global__ void w4g32_to_bf16_kernel(const uint8_t* __restrict__ packed, const uint16_t* __restrict__ scale,
                                     int64_t n, int64_t k, uint16_t* __restrict__ out) {
  pdl_trigger();
  pdl_wait();  // `out` may still be read by the previous GEMM
  const int64_t words = n * k / 8;  // 8 codes per 32-bit word
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < words; i += int64_t(gridDim.x) * blockDim.x) {
    const uint32_t u = __ldg(reinterpret_cast<const uint32_t*>(packed) + i);
    const int64_t e0 = i * 8, row = e0 / k, col = e0 % k;
    const float s = bf2f(scale[row * (k / 32) + col / 32]);
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int lo = int((u >> (8 * e)) & 0xF), hi = int((u >> (8 * e + 4)) & 0xF);
      const float clo = float(lo >= 8 ? lo - 16 : lo), chi = float(hi >= 8 ? hi - 16 : hi);
      w[e] = uint32_t(f2bf(clo * s)) | (uint32_t(f2bf(chi * s)) << 16);
    }
    reinterpret_cast<uint4*>(out)[i] = make_uint4(w[0], w[1], w[2], w[3]);
  }
}

// MX codes (fmt 2: E4M3 bytes; fmt 3: E2M1 nibbles, even k low) times their
// E8M0 scale: exact in f32, and the product of a code and a power of two is
// a bf16 value, so the expansion is exact.
template <int FMT>
__global__ void mx_to_bf16_kernel(const uint8_t* __restrict__ codes, const uint8_t* __restrict__ scale, int64_t n,
                                  int64_t k, uint16_t* __restrict__ out) {
  pdl_trigger();
  pdl_wait();  // `out` may still be read by the previous GEMM
  constexpr int kPer = FMT == 2 ? 4 : 8;  // codes per 32-bit word
  const int64_t words = n * k / kPer;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < words; i += int64_t(gridDim.x) * blockDim.x) {
    const uint32_t u = __ldg(reinterpret_cast<const uint32_t*>(codes) + i);
    const int64_t e0 = i * kPer, row = e0 / k, col = e0 % k;
    const float s = e8m0_f32(scale[row * (k / 32) + col / 32]);
    if constexpr (FMT == 2) {
      const uint32_t w0 = uint32_t(f2bf(e4m3_f32(u & 0xFF) * s)) | (uint32_t(f2bf(e4m3_f32((u >> 8) & 0xFF) * s)) << 16);
      const uint32_t w1 =
          uint32_t(f2bf(e4m3_f32((u >> 16) & 0xFF) * s)) | (uint32_t(f2bf(e4m3_f32(u >> 24) * s)) << 16);
      reinterpret_cast<uint2*>(out)[i] = make_uint2(w0, w1);
    } else {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        w[e] = uint32_t(f2bf(e2m1_f32((u >> (8 * e)) & 0xF) * s)) |
               (uint32_t(f2bf(e2m1_f32((u >> (8 * e + 4)) & 0xF) * s)) << 16);
      reinterpret_cast<uint4*>(out)[i] = make_uint4(w[0], w[1], w[2], w[3]);
    }
  }
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
  static EncodeTiled fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiled>(p);
  });
  return fn;
}

// A bf16 [rows, k] row-major operand as 64 x box_rows tiles, 128-byte swizzled.
bool make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t k, uint32_t box_rows) {
  EncodeTiled enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {cuuint64_t(k), cuuint64_t(rows)};
  const cuuint64_t strides[1] = {cuuint64_t(k) * 2};
  const cuuint32_t box[2] = {uint32_t(kBK), box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool gemm_tc_supported(int64_t m, int64_t n, int64_t k, const void* x, const void* w) {
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  return m > 0 && n > 0 && k > 0 && k % 8 == 0 && a16(x) && a16(w) && m <= int64_t(65535) * kBM &&
         encode_fn() != nullptr;
}

namespace {

template <int EPI, int BN>
int launch_gemm(const CUtensorMap& mx, const CUtensorMap& mw, const CUtensorMap& mw2, const GemmArgs& a,
                cudaStream_t st) {
  static PerDeviceOnce configured;
  if (!configured.run([] {
        return cudaFuncSetAttribute(gemm_tc_kernel<EPI, BN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    GL<BN>::kSmem) == cudaSuccess;
      }))
    return SB_INTERNAL;
  constexpr int cols = EPI == 1 ? BN / 2 : BN;
  const int tiles = (a.n + cols - 1) / cols * ((a.m + kBM - 1) / kBM);
  const dim3 grid{unsigned(tiles < kNumSMs ? tiles : kNumSMs), 1u, 1u};  // persistent: one CTA per SM
  if (launch_pdl(gemm_tc_kernel<EPI, BN>, grid, dim3(kGThreads), size_t(GL<BN>::kSmem), st, mx, mw, mw2, a) !=
      cudaSuccess)
    return SB_INTERNAL;
  count_launch();
  return SB_OK;
}

// The tile width for an m x n launch (n output features; a SwiGLU tile holds
// BN/2 of them): a persistent CTA's time goes with (tiles per CTA, rounded
// up) x (BN + 32) -- the B tile plus about 32 rows' worth of A tile and
// epilogue -- so small m takes narrow tiles that fill the 148 SMs, and
// prefill-sized m keeps 256 (at m = 16384 every 7B projection does).  Ties
// keep the wider tile.
int choose_bn(int64_t m, int64_t n, bool swiglu) {
  int best = 256;
  int64_t best_cost = -1;
  for (int bn : {256, 128, 64, 32}) {
    if (swiglu && bn < 64) continue;
    const int64_t cols = swiglu ? bn / 2 : bn;
    const int64_t tiles = (n + cols - 1) / cols * ((m + kBM - 1) / kBM);
    const int64_t cost = (tiles + kNumSMs - 1) / kNumSMs * (bn + 32);
    if (best_cost < 0 || cost < best_cost) {
      best = bn;
      best_cost = cost;
    }
  }
  return best;
}

}  // namespace

int launch_gemm_tc_bf16(const uint16_t* x, int64_t m, int64_t k, const uint16_t* w, int64_t n, const float* scale,
                        const uint16_t* residual, int64_t ldr, uint16_t* y, int64_t ldy, int* err, cudaStream_t st) {
  if (!gemm_tc_supported(m, n, k, x, w)) return SB_INVALID_ARGUMENT;
  const int bn = choose_bn(m, n, false);
  CUtensorMap mx, mw;
  if (!make_map(&mx, x, m, k, kBM) || !make_map(&mw, w, n, k, uint32_t(bn))) return SB_INTERNAL;
  GemmArgs a{};
  a.m = int(m);
  a.n = int(n);
  a.k = int(k);
  a.scale = scale;
  a.residual = residual;
  a.ldr = int(ldr);
  a.y = y;
  a.ldy = int(ldy);
  a.err = err;
  switch (bn) {
    case 32: return launch_gemm<0, 32>(mx, mw, mw, a, st);
    case 64: return launch_gemm<0, 64>(mx, mw, mw, a, st);
    case 128: return launch_gemm<0, 128>(mx, mw, mw, a, st);
    default: return launch_gemm<0, 256>(mx, mw, mw, a, st);
  }
}

int launch_gemm_tc_swiglu(const uint16_t* x, int64_t m, int64_t k, const uint16_t* w_gate, const uint16_t* w_up,
                          int64_t n, const float* s_gate, const float* s_up, uint16_t* y, int64_t ldy, int* err,
                          cudaStream_t st) {
  if (!gemm_tc_supported(m, n, k, x, w_gate) || !gemm_tc_supported(m, n, k, x, w_up)) return SB_INVALID_ARGUMENT;
  const int bn = choose_bn(m, n, true);
  CUtensorMap mx, mg, mu;
  if (!make_map(&mx, x, m, k, kBM) || !make_map(&mg, w_gate, n, k, uint32_t(bn / 2)) ||
      !make_map(&mu, w_up, n, k, uint32_t(bn / 2)))
    return SB_INTERNAL;
  GemmArgs a{};
  a.m = int(m);
  a.n = int(n);
  a.k = int(k);
  a.scale = s_gate;
  a.scale2 = s_up;
  a.y = y;
  a.ldy = int(ldy);
  a.err = err;
  switch (bn) {
    case 64: return launch_gemm<1, 64>(mx, mg, mu, a, st);
    case 128: return launch_gemm<1, 128>(mx, mg, mu, a, st);
    default: return launch_gemm<1, 256>(mx, mg, mu, a, st);
  }
}

int launch_codes_to_bf16(const void* w, const void* scale, int fmt, int64_t n, int64_t k, uint16_t* out,
                         cudaStream_t st) {
  const int threads = 256, blocks = 4 * kNumSMs;
  cudaError_t e;
  if (fmt == 1) {  // int8 per channel: the codes themselves
    e = launch_pdl(codes_i8_to_bf16_kernel, dim3(blocks), dim3(threads), 0, st, static_cast<const int8_t*>(w),
                   n * k, out);
  } else if (fmt == 0) {  // int4 group 32: code * bf16 scale, rounded to bf16
    if (k % 32) return SB_INVALID_ARGUMENT;
    e = launch_pdl(w4g32_to_bf16_kernel, dim3(blocks), dim3(threads), 0, st, static_cast<const uint8_t*>(w),
                   static_cast<const uint16_t*>(scale), n, k, out);
  } else if (fmt == 2 || fmt == 3) {  // MX: code * 2^(e - 127), exact
    if (k % 32) return SB_INVALID_ARGUMENT;
    auto kern = fmt == 2 ? mx_to_bf16_kernel<2> : mx_to_bf16_kernel<3>;
    e = launch_pdl(kern, dim3(blocks), dim3(threads), 0, st, static_cast<const uint8_t*>(w),
                   static_cast<const uint8_t*>(scale), n, k, out);
  } else {
    return SB_INVALID_ARGUMENT;
  }
  if (e != cudaSuccess) return SB_INTERNAL;
  count_launch();
  return SB_OK;
}

}  // namespace sb
