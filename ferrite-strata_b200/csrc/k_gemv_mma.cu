// Tensor-core GEMV for decode (M <= 16 rows of x per launch), int4 group-32
// and int8 per-channel weights, with fused epilogues.
//
// Work decomposition.  The output is cut into 16-row mma.m16n8k16 tiles.  The
// grid is persistent (at most one wave of resident blocks); block b computes
// tiles b, b + grid, b + 2 grid, ...  Within a tile the 8 warps split K into 8
// slices of whole 32-code groups and the 8 partial fragments are summed
// through shared memory by finish_tile.
//
// Memory pipeline.  Each warp copies its slice of the 16 weight rows to its
// own shared-memory ring with 16-byte cp.async (a row's slice is contiguous,
// so every copy instruction moves whole 32-byte sectors), two chunks of 8
// groups deep, together with the int4 scales of those groups.  The ring runs
// over the block's whole tile sequence, so the next tile's weights stream in
// while the current tile is reduced.  The first two chunks are issued before
// griddepcontrol.wait: under programmatic dependent launch the weight stream
// overlaps the tail of the previous kernel, and only the activations, which
// that kernel produces, are read after the wait.  ldmatrix m8n8 (b16) then
// hands thread (g, q) exactly the 32-bit word q of rows g and g + 8 of a group,
// which is the fragment the dequantisation below needs.
//
// Dequantisation.  Thread (g, q) holds, per row and group, the word q: eight
// int4 codes at k offsets 8q..8q+7.  XOR 0x88888888 turns each code c into
// c + 8; OR-ing nibble pairs (j, j+4) into the mantissa of bf16 128.0 and
// subtracting 136.0 gives the exact codes as bf16x2 pairs.  The MMA's k order
// inside a group is permuted to match (virtual k 2q,2q+1 <-> real 8q+2s,
// 8q+2s+4 for k16 step s) and the activations are permuted the same way with
// byte permutes, so the dot product is unchanged.  Each group's two MMAs
// accumulate into a fresh fragment that is scaled by the group's bf16 scale in
// f32: dequantisation is exactly code * scale, as in the oracle.
#include <cstdlib>
#include <string>

#include "k_gemv_mma.cuh"

namespace sb {

namespace {

constexpr int kWarps = 8;      // K-slices per block
constexpr int kTileRows = 16;  // output rows per block
constexpr int kChunk = 8;      // groups per pipeline stage
constexpr int kStages = 2;

struct Params {
  const uint16_t* x;
  int m, k;          // rows of x in this launch (<= 16), inner dimension
  int groups;        // k / 32
  int gpw;           // groups per warp (K-slice)
  int njobs;
  const uint8_t* w[3];
  const void* s[3];
  int n[3];
  uint16_t* y[3];
  const uint16_t* res[3];
  int m_base;        // absolute row of this launch's first x row (sequence index)
  int tiles;         // 16-row output tiles
  QkvExtra qkv;
};

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

__device__ __forceinline__ void mma_bf16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2,
                                         uint32_t a3, uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
      "{%8,%9}, {%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ uint32_t bf16x2_sub(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}

// Nibble pair (j, j+4) of a code word already XOR-ed with 0x88888888.
__device__ __forceinline__ uint32_t int4_pair(uint32_t u, int j) {
  return bf16x2_sub(((u >> (4 * j)) & 0x000F000Fu) | 0x43004300u, 0x43084308u);
}

__device__ __forceinline__ float int8_code(uint32_t u, int j) {
  return __uint_as_float(((u >> (8 * j)) & 0xFFu) | 0x4B000000u) - 8388736.0f;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

// Job and matrix row of tile row t (0..15) in block y.  Tile rows t and t + 8
// form one epilogue pair.
template <int MODE>
__device__ __forceinline__ void row_of(const Params& p, int y, int t, int& job, int& row) {
  if constexpr (MODE == 0) {
    int r = y * kTileRows + t;
    job = 0;
    while (job + 1 < p.njobs && r >= p.n[job]) r -= p.n[job++];
    row = r;
  } else if constexpr (MODE == 1) {
    job = t < 8 ? 0 : 1;
    row = y * 8 + (t & 7);
  } else {
    const int hd = p.qkv.head_dim;
    const int bph = hd / 16;  // blocks per head: 8 rotate-half pairs per block
    const int head = y / bph, j = y % bph;
    const int in_head = 8 * j + (t & 7) + (t < 8 ? 0 : hd / 2);
    if (head < p.qkv.hq) {
      job = 0;
      row = head * hd + in_head;
    } else if (head < p.qkv.hq + p.qkv.hkv) {
      job = 1;
      row = (head - p.qkv.hq) * hd + in_head;
    } else {
      job = 2;
      row = (head - p.qkv.hq - p.qkv.hkv) * hd + in_head;
    }
  }
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* smem) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

// Sum the 8 K-slice partials of tile y through shared memory and run the
// epilogue.  Every thread of the block calls this once per tile.
template <int FMT, int NT, int MODE>
__device__ __forceinline__ void finish_tile(const Params& p, int y, float (&red)[kWarps][kTileRows][16],
                                            const float (&acc)[NT][4], int warp, int g, int q, int tid) {
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    red[warp][g][t * 8 + 2 * q] = acc[t][0];
    red[warp][g][t * 8 + 2 * q + 1] = acc[t][1];
    red[warp][g + 8][t * 8 + 2 * q] = acc[t][2];
    red[warp][g + 8][t * 8 + 2 * q + 1] = acc[t][3];
  }
  __syncthreads();
  const int items = 8 * p.m;
  for (int it = tid; it < items; it += kWarps * 32) {
    const int pp = it / p.m, m = it % p.m;
    float vlo = 0.0f, vhi = 0.0f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      vlo += red[w][pp][m];
      vhi += red[w][pp + 8][m];
    }
    int jl, nlo, jh, nhi;
    row_of<MODE>(p, y, pp, jl, nlo);
    row_of<MODE>(p, y, pp + 8, jh, nhi);
    if (FMT == 1) {
      vlo *= reinterpret_cast<const float*>(p.s[jl])[nlo];
      vhi *= reinterpret_cast<const float*>(p.s[jh])[nhi];
    }
    if constexpr (MODE == 0) {
      if (p.res[jl]) vlo += bf2f(p.res[jl][int64_t(m) * p.n[jl] + nlo]);
      if (p.res[jh]) vhi += bf2f(p.res[jh][int64_t(m) * p.n[jh] + nhi]);
      p.y[jl][int64_t(m) * p.n[jl] + nlo] = f2bf(vlo);
      p.y[jh][int64_t(m) * p.n[jh] + nhi] = f2bf(vhi);
    } else if constexpr (MODE == 1) {
      const float silu = vlo / (1.0f + expf(-vlo));
      p.y[0][int64_t(m) * p.n[0] + nlo] = f2bf(silu * vhi);
    } else {
      const QkvExtra& e = p.qkv;
      const int hd = e.head_dim, half = hd / 2;
      const int head_in_job = nlo / hd, i = nlo % hd;  // i < half: the pair's first row
      // The projection output is a bf16 value: round before the rotation.
      double xlo = bf2f(f2bf(vlo)), xhi = bf2f(f2bf(vhi));
      const int pos = e.pos[m];
      if (jl < 2) {
        const double inv = pow(e.theta, -2.0 * double(i) / double(hd));
        double sn, cs;
        sincos(double(pos) * inv, &sn, &cs);
        const double a = xlo * cs - xhi * sn, b = xhi * cs + xlo * sn;
        xlo = double(float(a));
        xhi = double(float(b));
      }
      const uint16_t olo = f2bf(float(xlo)), ohi = f2bf(float(xhi));
      if (jl == 0) {
        uint16_t* qo = e.q_out + int64_t(m) * e.hq * hd + head_in_job * hd;
        qo[i] = olo;
        qo[i + half] = ohi;
      } else {
        uint16_t* side = jl == 1 ? e.k_out : e.v_out;
        if (side) {
          uint16_t* so = side + int64_t(m) * e.hkv * hd + head_in_job * hd;
          so[i] = olo;
          so[i + half] = ohi;
        }
        if (pos >= 0 && pos < e.max_len) {
          const int seq = (p.m_base + m) / e.tokens_per_seq;
          uint16_t* cache = jl == 1 ? e.k_cache : e.v_cache;
          uint16_t* dst = cache + ((int64_t(seq) * e.hkv + head_in_job) * e.max_len + pos) * hd;
          dst[i] = olo;
          dst[i + half] = ohi;
        } else if (e.err) {
          atomicExch(e.err, 2);
        }
      }
    }
  }
  __syncthreads();  // red is reused by the next tile
}

template <int FMT>
struct Stage {
  static constexpr int kBPG = FMT == 0 ? 16 : 32;            // bytes per row per group
  static constexpr int kW = kChunk * kTileRows * kBPG;        // weight bytes of one stage
  static constexpr int kS = FMT == 0 ? kTileRows * kChunk * 2 : 0;  // bf16 scales of one stage
  static constexpr int kBytes = kW + kS;
};

// Per warp: the ring of kStages stages (weights, then bf16 scales [16][kChunk]).
__host__ __device__ constexpr size_t warp_smem_bytes(int fmt) {
  return size_t(kStages) * (fmt == 0 ? Stage<0>::kBytes : Stage<1>::kBytes);
}

template <int FMT, int NT, int MODE>
__global__ void __launch_bounds__(kWarps * 32) gemv_mma_kernel(const __grid_constant__ Params p) {
  __shared__ float red[kWarps][kTileRows][16];
  extern __shared__ __align__(128) uint8_t dsm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q = lane & 3;
  constexpr int BPG = Stage<FMT>::kBPG;
  uint8_t* ring = dsm + size_t(warp) * warp_smem_bytes(FMT);

  const int64_t row_bytes = int64_t(p.k) * BPG / 32;
  const int gb = warp * p.gpw;
  const int ng = max(0, min(p.groups, gb + p.gpw) - gb);
  const int nchunks = max(1, (ng + kChunk - 1) / kChunk);  // a warp with no groups still steps
  // This block's tiles: blockIdx.x, blockIdx.x + gridDim.x, ...
  const int my_tiles = (p.tiles - int(blockIdx.x) + int(gridDim.x) - 1) / int(gridDim.x);
  const int items = my_tiles * nchunks;

  // Copy item it (tile it / nchunks, chunk it % nchunks) into stage it % kStages:
  // 16 rows x nj groups of weights (16 B copies, consecutive lanes along a
  // row) and, for int4, the matching bf16 scales (4 B copies).
  auto issue = [&](int it) {
    if (it < items) {
      const int y = int(blockIdx.x) + (it / nchunks) * int(gridDim.x);
      const int c = it % nchunks;
      const int nj = max(0, min(kChunk, ng - c * kChunk));
      uint8_t* dst = ring + (it % kStages) * Stage<FMT>::kBytes;
      const int per_row = nj * (BPG / 16);
      for (int e = lane; e < kTileRows * per_row; e += 32) {
        const int r = e / per_row, i = e % per_row;
        const int j = i / (BPG / 16), h = i % (BPG / 16);
        int job, row;
        row_of<MODE>(p, y, r, job, row);
        cp_async16(dst + ((j * kTileRows + r) * BPG) + h * 16,
                   p.w[job] + int64_t(row) * row_bytes + int64_t(gb + c * kChunk + j) * BPG + h * 16);
      }
      if constexpr (FMT == 0) {
        // Scales as bf16 pairs: needs an even group count and an even slice start.
        uint8_t* sdst = dst + Stage<FMT>::kW;
        const int pairs = (nj + 1) / 2;
        for (int e = lane; e < kTileRows * pairs; e += 32) {
          const int r = e / pairs, i = e % pairs;
          int job, row;
          row_of<MODE>(p, y, r, job, row);
          const uint8_t* src = reinterpret_cast<const uint8_t*>(p.s[job]) +
                               (int64_t(row) * p.groups + gb + c * kChunk + 2 * i) * 2;
          const uint32_t sa = static_cast<uint32_t>(__cvta_generic_to_shared(sdst + (r * kChunk + 2 * i) * 2));
          asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(sa), "l"(src) : "memory");
        }
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  pdl_trigger();
  for (int it = 0; it < kStages; ++it) issue(it);
  pdl_wait();  // activations come from the previous kernel

  float acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;
  // x row used by this thread's B fragment for n-tile t: rows past M repeat
  // the last row (their output columns are never written).
  const uint16_t* xrow[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) xrow[t] = p.x + int64_t(min(t * 8 + g, p.m - 1)) * p.k + int64_t(gb) * 32;
  const int mi = lane >> 3, rr = lane & 7;  // ldmatrix: matrix mi, row rr

  for (int it = 0; it < items; ++it) {
    const int c = it % nchunks;
    const int y = int(blockIdx.x) + (it / nchunks) * int(gridDim.x);
    asm volatile("cp.async.wait_group %0;" ::"n"(kStages - 1) : "memory");
    __syncwarp();
    const uint8_t* st = ring + (it % kStages) * Stage<FMT>::kBytes;
    const int nj = max(0, min(kChunk, ng - c * kChunk));
#pragma unroll
    for (int j = 0; j < kChunk; j += 2) {
      if (j < nj) {
        if constexpr (FMT == 0) {
          uint32_t f[4];
          ldsm_x4(f, st + (((j + (mi >> 1)) * kTileRows + (mi & 1) * 8 + rr) * BPG));
          const uint16_t* ss = reinterpret_cast<const uint16_t*>(st + Stage<FMT>::kW);
#pragma unroll
          for (int jj = 0; jj < 2; ++jj) {
            if (j + jj < nj) {
              const int gi = c * kChunk + j + jj;  // group within the slice
              const uint32_t ul = f[2 * jj] ^ 0x88888888u, uh = f[2 * jj + 1] ^ 0x88888888u;
              const uint32_t p0 = int4_pair(ul, 0), p1 = int4_pair(ul, 1), p2 = int4_pair(ul, 2),
                             p3 = int4_pair(ul, 3);
              const uint32_t h0 = int4_pair(uh, 0), h1 = int4_pair(uh, 1), h2 = int4_pair(uh, 2),
                             h3 = int4_pair(uh, 3);
              const float sl = bf2f(ss[g * kChunk + j + jj]), sh = bf2f(ss[(g + 8) * kChunk + j + jj]);
#pragma unroll
              for (int t = 0; t < NT; ++t) {
                const uint4 xv = ldg16(xrow[t] + int64_t(gi) * 32 + 8 * q);
                float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                mma_bf16(d, p0, h0, p1, h1, prmt(xv.x, xv.z, 0x5410), prmt(xv.x, xv.z, 0x7632));
                mma_bf16(d, p2, h2, p3, h3, prmt(xv.y, xv.w, 0x5410), prmt(xv.y, xv.w, 0x7632));
                acc[t][0] = fmaf(d[0], sl, acc[t][0]);
                acc[t][1] = fmaf(d[1], sl, acc[t][1]);
                acc[t][2] = fmaf(d[2], sh, acc[t][2]);
                acc[t][3] = fmaf(d[3], sh, acc[t][3]);
              }
            }
          }
        } else {
#pragma unroll
          for (int jj = 0; jj < 2; ++jj) {
            if (j + jj < nj) {
              const int gi = c * kChunk + j + jj;
              // int8: a group is 32 B per row = two 16 B halves, one k16 step each.
              uint32_t f[4];
              ldsm_x4(f, st + (((j + jj) * kTileRows + (mi & 1) * 8 + rr) * BPG) + (mi >> 1) * 16);
#pragma unroll
              for (int s = 0; s < 2; ++s) {
                const uint32_t ul = f[2 * s] ^ 0x80808080u, uh = f[2 * s + 1] ^ 0x80808080u;
                const uint32_t a0 = pack_bf16x2(int8_code(ul, 0), int8_code(ul, 2));
                const uint32_t a2 = pack_bf16x2(int8_code(ul, 1), int8_code(ul, 3));
                const uint32_t a1 = pack_bf16x2(int8_code(uh, 0), int8_code(uh, 2));
                const uint32_t a3 = pack_bf16x2(int8_code(uh, 1), int8_code(uh, 3));
#pragma unroll
                for (int t = 0; t < NT; ++t) {
                  const uint2 xv =
                      __ldg(reinterpret_cast<const uint2*>(xrow[t] + int64_t(gi) * 32 + 16 * s + 4 * q));
                  mma_bf16(acc[t], a0, a1, a2, a3, prmt(xv.x, xv.y, 0x5410), prmt(xv.x, xv.y, 0x7632));
                }
              }
            }
          }
        }
      }
    }
    __syncwarp();
    issue(it + kStages);  // keeps the ring full across tile boundaries
    if (c == nchunks - 1) {
      finish_tile<FMT, NT, MODE>(p, y, red, acc, warp, g, q, tid);
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;
    }
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
}

template <int FMT, int NT, int MODE>
int launch_one(const Params& p, int blocks, bool pdl, cudaStream_t st) {
  auto kern = gemv_mma_kernel<FMT, NT, MODE>;
  const size_t smem = kWarps * warp_smem_bytes(FMT);
  static int per_sm = 0;
  if (per_sm == 0) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
      return SB_INTERNAL;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kWarps * 32, smem) != cudaSuccess ||
        per_sm < 1)
      per_sm = 1;
  }
  // Persistent: at most one full wave of blocks, each walking tiles.
  const int grid = blocks < per_sm * kNumSMs ? blocks : per_sm * kNumSMs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(kWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, kern, p) != cudaSuccess) return SB_INTERNAL;
  count_launch();
  return SB_OK;
}

template <int FMT, int NT>
int dispatch_mode(GemvMode mode, const Params& p, int blocks, bool pdl, cudaStream_t st) {
  switch (mode) {
    case GemvMode::Plain: return launch_one<FMT, NT, 0>(p, blocks, pdl, st);
    case GemvMode::SwiGLU: return launch_one<FMT, NT, 1>(p, blocks, pdl, st);
    case GemvMode::QkvRope: return launch_one<FMT, NT, 2>(p, blocks, pdl, st);
  }
  return SB_INVALID_ARGUMENT;
}

}  // namespace

// STRATA_B200_GEMV=cudacore routes every batch to the CUDA-core GEMV (for A/B measurements).
static bool tensor_core_gemv_enabled() {
  static const bool on = [] {
    const char* v = std::getenv("STRATA_B200_GEMV");
    return !(v && std::string(v) == "cudacore");
  }();
  return on;
}

bool gemv_mma_supported(const GemvMmaArgs& a) {
  if (!tensor_core_gemv_enabled() && a.mode != GemvMode::QkvRope) return false;
  const LinearBatch& b = a.lb;
  if (b.fmt != WFormat::W4G32 && b.fmt != WFormat::W8PC) return false;
  if (b.k % 32 || b.m <= 0) return false;
  if (b.fmt == WFormat::W4G32 && (b.k / 32) % 2) return false;  // scales copied as bf16 pairs
  auto aligned = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (!aligned(b.x)) return false;
  for (int j = 0; j < b.njobs; ++j)
    if (!aligned(b.jobs[j].w)) return false;
  switch (a.mode) {
    case GemvMode::Plain:
      if (b.epi == Epilogue::SwiGLU) return false;
      for (int j = 0; j < b.njobs; ++j)
        if (b.jobs[j].n % kTileRows || b.jobs[j].n <= 0) return false;
      return true;
    case GemvMode::SwiGLU:
      return b.njobs == 2 && b.jobs[0].n == b.jobs[1].n && b.jobs[0].n % 8 == 0 && b.jobs[0].n > 0;
    case GemvMode::QkvRope: {
      const QkvExtra& e = a.qkv;
      if (b.njobs != 3 || (e.head_dim != 64 && e.head_dim != 128)) return false;
      return b.jobs[0].n == e.hq * e.head_dim && b.jobs[1].n == e.hkv * e.head_dim &&
             b.jobs[2].n == e.hkv * e.head_dim && e.tokens_per_seq > 0;
    }
  }
  return false;
}

int launch_gemv_mma(const GemvMmaArgs& a, cudaStream_t st) {
  if (!gemv_mma_supported(a)) return SB_INVALID_ARGUMENT;
  const LinearBatch& b = a.lb;
  const int fmt = b.fmt == WFormat::W4G32 ? 0 : 1;
  const int groups = b.k / 32;
  int gpw = (groups + kWarps - 1) / kWarps;
  gpw += gpw & 1;  // even slice starts keep the bf16 scale pairs 4-byte aligned
  int rows = 0;
  switch (a.mode) {
    case GemvMode::Plain:
      for (int j = 0; j < b.njobs; ++j) rows += b.jobs[j].n;
      break;
    case GemvMode::SwiGLU: rows = 2 * b.jobs[0].n; break;
    case GemvMode::QkvRope: rows = b.jobs[0].n + b.jobs[1].n + b.jobs[2].n; break;
  }
  const int blocks = rows / kTileRows;

  for (int m0 = 0; m0 < b.m; m0 += 16) {
    Params p{};
    p.m = b.m - m0 < 16 ? b.m - m0 : 16;
    p.x = b.x + int64_t(m0) * b.k;
    p.k = b.k;
    p.groups = groups;
    p.gpw = gpw;
    p.njobs = b.njobs;
    for (int j = 0; j < b.njobs; ++j) {
      const LinearJob& J = b.jobs[j];
      p.w[j] = static_cast<const uint8_t*>(J.w);
      p.s[j] = J.s;
      p.n[j] = J.n;
      p.y[j] = J.y ? J.y + int64_t(m0) * J.ldy : nullptr;
      p.res[j] = J.residual ? J.residual + int64_t(m0) * J.ldr : nullptr;
    }
    p.qkv = a.qkv;
    p.m_base = m0;
    p.tiles = blocks;
    if (a.mode == GemvMode::QkvRope) {
      const QkvExtra& e = a.qkv;
      p.qkv.pos = e.pos + m0;
      p.qkv.q_out = e.q_out + int64_t(m0) * e.hq * e.head_dim;
      p.qkv.k_out = e.k_out ? e.k_out + int64_t(m0) * e.hkv * e.head_dim : nullptr;
      p.qkv.v_out = e.v_out ? e.v_out + int64_t(m0) * e.hkv * e.head_dim : nullptr;
    }
    const bool two = p.m > 8;
    int rc;
    if (fmt == 0)
      rc = two ? dispatch_mode<0, 2>(a.mode, p, blocks, a.pdl, st) : dispatch_mode<0, 1>(a.mode, p, blocks, a.pdl, st);
    else
      rc = two ? dispatch_mode<1, 2>(a.mode, p, blocks, a.pdl, st) : dispatch_mode<1, 1>(a.mode, p, blocks, a.pdl, st);
    if (rc) return rc;
  }
  return SB_OK;
}

}  // namespace sb
