// Tensor-core GEMV for decode (M <= 16 rows of x per launch), int4 group-32
// and int8 per-channel weights, with fused epilogues.
//
// Work decomposition.  A block computes one 16-row mma.m16n8k16 tile of the
// output.  Its 8 warps split K into 8 slices of whole 32-code groups; each
// warp streams its slice of the 16 weight rows straight from HBM into mma
// fragment registers (no shared-memory staging), and the 8 partial fragments
// are summed through shared memory at the end.  A 4096 x 4096 matrix is 256
// blocks x 8 warps = 2048 streaming warps.
//
// Memory pipeline.  Each warp issues the loads for its first 16 groups (and
// their scales) before griddepcontrol.wait, so under programmatic dependent
// launch the weight stream of this kernel overlaps the tail of the previous
// kernel; only the activations, which the previous kernel produces, are read
// after the wait.
//
// Dequantisation.  Thread (g, q) of the fragment holds, per row and group,
// the 32-bit word q: eight int4 codes at k offsets 8q..8q+7.  XOR 0x88888888
// turns each code c into c + 8; OR-ing nibble pairs (j, j+4) into the mantissa
// of bf16 128.0 and subtracting 136.0 gives the exact codes as bf16x2 pairs.
// The MMA's k order inside a group is permuted to match (virtual k 2q,2q+1 <->
// real 8q+2s, 8q+2s+4 for k16 step s) and the activations are permuted the
// same way with byte permutes, so the dot product is unchanged.  Each group's
// two MMAs accumulate into a fresh fragment that is scaled by the group's
// bf16 scale in f32: dequantisation is exactly code * scale, as in the oracle.
#include "k_gemv_mma.cuh"

namespace sb {

namespace {

constexpr int kWarps = 8;      // K-slices per block
constexpr int kTileRows = 16;  // output rows per block
constexpr int kChunk = 16;     // groups loaded per batch of loads

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

__device__ __forceinline__ uint32_t ldg32_stream(const void* p) {
  uint32_t r;
  asm volatile("ld.global.nc.L1::evict_first.u32 %0, [%1];" : "=r"(r) : "l"(p));
  return r;
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

template <int FMT, int NT, int MODE>
__global__ void __launch_bounds__(kWarps * 32) gemv_mma_kernel(const __grid_constant__ Params p) {
  __shared__ float red[kWarps][kTileRows][16];
  const int y = blockIdx.x;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q = lane & 3;
  constexpr int BPG = FMT == 0 ? 16 : 32;  // bytes per row per 32-code group

  int jlo, rlo, jhi, rhi;
  row_of<MODE>(p, y, g, jlo, rlo);
  row_of<MODE>(p, y, g + 8, jhi, rhi);
  const int64_t row_bytes = int64_t(p.k) * BPG / 32;
  const uint8_t* wlo = p.w[jlo] + int64_t(rlo) * row_bytes;
  const uint8_t* whi = p.w[jhi] + int64_t(rhi) * row_bytes;
  const int gb = warp * p.gpw;
  const int ge = min(p.groups, gb + p.gpw);

  pdl_trigger();

  float acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;

  // x row used by this thread's B fragment for n-tile t: rows past M repeat
  // the last row (their output columns are never written).
  const uint16_t* xrow[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t) xrow[t] = p.x + int64_t(min(t * 8 + g, p.m - 1)) * p.k;

  bool waited = false;
  for (int c0 = gb; c0 < ge; c0 += kChunk) {
    const int nc = min(kChunk, ge - c0);
    // ---- weights and scales: independent of the previous kernel
    uint32_t wl[kChunk][BPG / 16], wh[kChunk][BPG / 16];
    float sl[kChunk], sh[kChunk];
#pragma unroll
    for (int i = 0; i < kChunk; ++i) {
      if (i < nc) {
#pragma unroll
        for (int s = 0; s < BPG / 16; ++s) {
          wl[i][s] = ldg32_stream(wlo + int64_t(c0 + i) * BPG + 16 * s + 4 * q);
          wh[i][s] = ldg32_stream(whi + int64_t(c0 + i) * BPG + 16 * s + 4 * q);
        }
        if constexpr (FMT == 0) {
          const unsigned short* s_lo = reinterpret_cast<const unsigned short*>(p.s[jlo]);
          const unsigned short* s_hi = reinterpret_cast<const unsigned short*>(p.s[jhi]);
          sl[i] = bf2f(__ldg(s_lo + int64_t(rlo) * p.groups + c0 + i));
          sh[i] = bf2f(__ldg(s_hi + int64_t(rhi) * p.groups + c0 + i));
        }
      }
    }
    if (!waited) {
      pdl_wait();  // the activations come from the previous kernel
      waited = true;
    }
#pragma unroll
    for (int i = 0; i < kChunk; ++i) {
      if (i < nc) {
        const int gi = c0 + i;
        if constexpr (FMT == 0) {
          const uint32_t ul = wl[i][0] ^ 0x88888888u, uh = wh[i][0] ^ 0x88888888u;
          const uint32_t p0 = int4_pair(ul, 0), p1 = int4_pair(ul, 1), p2 = int4_pair(ul, 2),
                         p3 = int4_pair(ul, 3);
          const uint32_t h0 = int4_pair(uh, 0), h1 = int4_pair(uh, 1), h2 = int4_pair(uh, 2),
                         h3 = int4_pair(uh, 3);
#pragma unroll
          for (int t = 0; t < NT; ++t) {
            const uint4 xv = ldg16(xrow[t] + int64_t(gi) * 32 + 8 * q);
            float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
            mma_bf16(d, p0, h0, p1, h1, prmt(xv.x, xv.z, 0x5410), prmt(xv.x, xv.z, 0x7632));
            mma_bf16(d, p2, h2, p3, h3, prmt(xv.y, xv.w, 0x5410), prmt(xv.y, xv.w, 0x7632));
            acc[t][0] = fmaf(d[0], sl[i], acc[t][0]);
            acc[t][1] = fmaf(d[1], sl[i], acc[t][1]);
            acc[t][2] = fmaf(d[2], sh[i], acc[t][2]);
            acc[t][3] = fmaf(d[3], sh[i], acc[t][3]);
          }
        } else {
#pragma unroll
          for (int s = 0; s < 2; ++s) {
            const uint32_t ul = wl[i][s] ^ 0x80808080u, uh = wh[i][s] ^ 0x80808080u;
            const uint32_t a0 = pack_bf16x2(int8_code(ul, 0), int8_code(ul, 2));
            const uint32_t a2 = pack_bf16x2(int8_code(ul, 1), int8_code(ul, 3));
            const uint32_t a1 = pack_bf16x2(int8_code(uh, 0), int8_code(uh, 2));
            const uint32_t a3 = pack_bf16x2(int8_code(uh, 1), int8_code(uh, 3));
#pragma unroll
            for (int t = 0; t < NT; ++t) {
              const uint2 xv = __ldg(reinterpret_cast<const uint2*>(xrow[t] + int64_t(gi) * 32 + 16 * s + 4 * q));
              mma_bf16(acc[t], a0, a1, a2, a3, prmt(xv.x, xv.y, 0x5410), prmt(xv.x, xv.y, 0x7632));
            }
          }
        }
      }
    }
  }
  if (!waited) pdl_wait();

  // ---- sum the 8 K-slice partials
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
}

template <int FMT, int NT, int MODE>
int launch_one(const Params& p, int blocks, bool pdl, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(blocks, 1, 1);
  cfg.blockDim = dim3(kWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = st;
  cudaLaunchAttribute attr;
  attr.id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr.val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = &attr;
  cfg.numAttrs = pdl ? 1 : 0;
  if (cudaLaunchKernelEx(&cfg, gemv_mma_kernel<FMT, NT, MODE>, p) != cudaSuccess) return SB_INTERNAL;
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

bool gemv_mma_supported(const GemvMmaArgs& a) {
  const LinearBatch& b = a.lb;
  if (b.fmt != WFormat::W4G32 && b.fmt != WFormat::W8PC) return false;
  if (b.k % 32 || b.m <= 0) return false;
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
  const int gpw = (groups + kWarps - 1) / kWarps;
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
