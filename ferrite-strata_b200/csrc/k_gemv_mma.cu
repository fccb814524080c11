// Tensor-core GEMV for decode (M <= 16 rows of x per launch), int4 group-32
// and int8 per-channel weights, with fused epilogues.
//
// Work decomposition.  A block owns 64 output rows (4 warps x 16 rows, one
// mma.m16n8k16 row tile per warp) and one K-slice of whole 32-wide groups.
// The K-slices of the same 64 rows form one thread-block cluster (up to 8
// CTAs); partial sums are reduced through distributed shared memory, so no
// partials reach HBM.
//
// Memory pipeline.  Every block first issues cp.async copies of its whole
// weight slice (and loads its scales), then executes griddepcontrol.wait: with
// programmatic dependent launch the weight stream of this kernel overlaps the
// tail of the previous kernel, and only the activations (which the previous
// kernel produces) are read after the wait.
//
// Dequantisation.  A thread of the mma fragment reads one 32-bit word per row
// per group: eight int4 codes at k offsets 8q..8q+7.  XOR 0x88888888 turns each
// code c into c + 8; OR-ing nibble pairs (j, j+4) into the mantissa of bf16
// 128.0 and subtracting 136.0 yields the exact codes as a bf16x2 pair.  The
// MMA's k order inside a group is permuted to match (virtual k 2q,2q+1 <->
// real 8q+2s, 8q+2s+4 for k16 step s), and the activations are permuted the
// same way with byte permutes, so the dot product is unchanged.  Each group's
// two MMAs accumulate into a fresh fragment that is scaled by the group's bf16
// scale in f32, so dequantisation is exact (code * scale) as in the oracle.
#include <cooperative_groups.h>

#include "k_gemv_mma.cuh"

namespace cg = cooperative_groups;

namespace sb {

namespace {

constexpr int kWarps = 4;
constexpr int kRows = 64;      // output rows per block
constexpr int kMaxCluster = 8;
constexpr int kMaxGroupsPerBlock = 48;
constexpr int kScalesPerThread = kRows * kMaxGroupsPerBlock / (kWarps * 32);

struct Params {
  const uint16_t* x;
  int m, k;          // rows of x in this launch (<= 16), inner dimension
  int groups;        // k / 32
  int gpb;           // groups per block (K-slice)
  int xs_stride;     // bytes per row of the staged activations
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

// Nibble pair (j, j+4) of a code word (already XOR-ed with 0x88888888).
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

// Global row of tile row `t` (0..15) of warp `w` in row block `y`: the job it
// belongs to and the row inside that job's matrix.  Tile rows t and t + 8
// form one epilogue pair.
template <int MODE>
__device__ __forceinline__ void row_of(const Params& p, int y, int w, int t, int& job, int& row) {
  if constexpr (MODE == 0) {
    int r = y * kRows + w * 16 + t;
    job = 0;
    while (job + 1 < p.njobs && r >= p.n[job]) r -= p.n[job++];
    row = r;
  } else if constexpr (MODE == 1) {
    job = t < 8 ? 0 : 1;
    row = y * 32 + w * 8 + (t & 7);
  } else {
    const int hd = p.qkv.head_dim;
    const int bph = hd / 64;  // blocks per head
    const int head = y / bph, j = y % bph;
    const int pi = 32 * j + 8 * w + (t & 7);  // rotate-half pair index in the head
    const int in_head = pi + (t < 8 ? 0 : hd / 2);
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

template <int FMT>
struct WF {
  static constexpr int kBytesPerGroupRow = FMT == 0 ? 16 : 32;  // 32 codes
};

template <int FMT, int NT, int MODE>
__global__ void __launch_bounds__(kWarps * 32) gemv_mma_kernel(const __grid_constant__ Params p) {
  extern __shared__ __align__(128) uint8_t smem[];
  constexpr int BPG = WF<FMT>::kBytesPerGroupRow;
  cg::cluster_group cluster = cg::this_cluster();
  const int crank = int(cluster.block_rank());
  const int csize = int(cluster.num_blocks());
  const int y = blockIdx.y;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q = lane & 3;

  const int g0 = crank * p.gpb;
  const int ng = max(0, min(p.gpb, p.groups - g0));

  uint8_t* sW = smem;                                              // [warp][gi][16][BPG]
  float* sS = reinterpret_cast<float*>(sW + kRows * p.gpb * BPG);  // [64][gpb] or [64]
  const int s_len = FMT == 0 ? kRows * p.gpb : kRows;
  uint8_t* sX = reinterpret_cast<uint8_t*>(sS + s_len);              // [16][xs_stride]
  float* sP = reinterpret_cast<float*>(sX + NT * 8 * p.xs_stride);  // [64][16]

  asm volatile("griddepcontrol.launch_dependents;");

  // ---- weights (independent of the previous kernel): issue before the wait
  {
    const int chunks_per_row = ng * (BPG / 16);
    const int total = kRows * chunks_per_row;
    for (int c = tid; c < total; c += kWarps * 32) {
      const int r = c / chunks_per_row, rem = c % chunks_per_row;
      const int gi = rem / (BPG / 16), sub = rem % (BPG / 16);
      int job, row;
      row_of<MODE>(p, y, r / 16, r % 16, job, row);
      const uint8_t* src = p.w[job] + int64_t(row) * (int64_t(p.k) * BPG / 32) +
                           int64_t(g0 + gi) * BPG + sub * 16;
      uint8_t* dst = sW + ((size_t(r / 16) * p.gpb + gi) * 16 + (r % 16)) * BPG + sub * 16;
      cp_async16(dst, src);
    }
    if (FMT == 0) {
      // All scale loads of a thread are issued before any is consumed, so
      // their latencies overlap (at most kScalesPerThread per thread).
      uint16_t sv[kScalesPerThread];
#pragma unroll
      for (int i = 0; i < kScalesPerThread; ++i) {
        const int c = tid + i * kWarps * 32;
        if (c < kRows * ng) {
          const int r = c / ng, gi = c % ng;
          int job, row;
          row_of<MODE>(p, y, r / 16, r % 16, job, row);
          sv[i] = __ldg(reinterpret_cast<const unsigned short*>(p.s[job]) + int64_t(row) * p.groups + g0 + gi);
        }
      }
#pragma unroll
      for (int i = 0; i < kScalesPerThread; ++i) {
        const int c = tid + i * kWarps * 32;
        if (c < kRows * ng) sS[(c / ng) * p.gpb + c % ng] = bf2f(sv[i]);
      }
    } else {
      for (int r = tid; r < kRows; r += kWarps * 32) {
        int job, row;
        row_of<MODE>(p, y, r / 16, r % 16, job, row);
        sS[r] = reinterpret_cast<const float*>(p.s[job])[row];
      }
    }
  }

  // ---- activations come from the previous kernel
  asm volatile("griddepcontrol.wait;" ::: "memory");
  {
    const int chunks = ng * 4;  // 32 bf16 = 64 B = 4 chunks per group
    // Rows m >= p.m of the staged tile are left unset: they only feed output
    // columns that are never written.
    for (int c = tid; c < p.m * chunks; c += kWarps * 32) {
      const int m = c / chunks, rem = c % chunks;
      cp_async16(sX + m * p.xs_stride + rem * 16,
                 reinterpret_cast<const uint8_t*>(p.x + int64_t(m) * p.k + int64_t(g0) * 32) + rem * 16);
    }
  }
  cp_async_commit_wait_all();
  __syncthreads();

  // ---- tensor-core main loop over this block's groups
  float acc[NT][4];
#pragma unroll
  for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;

  const uint8_t* wt = sW + size_t(warp) * p.gpb * 16 * BPG;
  for (int gi = 0; gi < ng; ++gi) {
    const uint8_t* wg = wt + size_t(gi) * 16 * BPG;
    if constexpr (FMT == 0) {
      const uint32_t ulo = *reinterpret_cast<const uint32_t*>(wg + g * BPG + 4 * q) ^ 0x88888888u;
      const uint32_t uhi = *reinterpret_cast<const uint32_t*>(wg + (g + 8) * BPG + 4 * q) ^ 0x88888888u;
      const uint32_t p0 = int4_pair(ulo, 0), p1 = int4_pair(ulo, 1), p2 = int4_pair(ulo, 2),
                     p3 = int4_pair(ulo, 3);
      const uint32_t h0 = int4_pair(uhi, 0), h1 = int4_pair(uhi, 1), h2 = int4_pair(uhi, 2),
                     h3 = int4_pair(uhi, 3);
      const float s_lo = sS[(warp * 16 + g) * p.gpb + gi];
      const float s_hi = sS[(warp * 16 + g + 8) * p.gpb + gi];
#pragma unroll
      for (int t = 0; t < NT; ++t) {
        const uint4 xv = *reinterpret_cast<const uint4*>(sX + (t * 8 + g) * p.xs_stride + gi * 64 + q * 16);
        float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
        mma_bf16(d, p0, h0, p1, h1, prmt(xv.x, xv.z, 0x5410), prmt(xv.x, xv.z, 0x7632));
        mma_bf16(d, p2, h2, p3, h3, prmt(xv.y, xv.w, 0x5410), prmt(xv.y, xv.w, 0x7632));
        acc[t][0] = fmaf(d[0], s_lo, acc[t][0]);
        acc[t][1] = fmaf(d[1], s_lo, acc[t][1]);
        acc[t][2] = fmaf(d[2], s_hi, acc[t][2]);
        acc[t][3] = fmaf(d[3], s_hi, acc[t][3]);
      }
    } else {
#pragma unroll
      for (int s = 0; s < 2; ++s) {
        const uint32_t ulo = *reinterpret_cast<const uint32_t*>(wg + g * BPG + 16 * s + 4 * q) ^ 0x80808080u;
        const uint32_t uhi = *reinterpret_cast<const uint32_t*>(wg + (g + 8) * BPG + 16 * s + 4 * q) ^ 0x80808080u;
        const uint32_t a0 = pack_bf16x2(int8_code(ulo, 0), int8_code(ulo, 2));
        const uint32_t a2 = pack_bf16x2(int8_code(ulo, 1), int8_code(ulo, 3));
        const uint32_t a1 = pack_bf16x2(int8_code(uhi, 0), int8_code(uhi, 2));
        const uint32_t a3 = pack_bf16x2(int8_code(uhi, 1), int8_code(uhi, 3));
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const uint2 xv = *reinterpret_cast<const uint2*>(sX + (t * 8 + g) * p.xs_stride + gi * 64 + s * 32 + q * 8);
          mma_bf16(acc[t], a0, a1, a2, a3, prmt(xv.x, xv.y, 0x5410), prmt(xv.x, xv.y, 0x7632));
        }
      }
    }
  }

  // ---- partials to shared memory, reduced across the cluster
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    float* lo = sP + (warp * 16 + g) * 16 + t * 8 + 2 * q;
    float* hi = sP + (warp * 16 + g + 8) * 16 + t * 8 + 2 * q;
    lo[0] = acc[t][0];
    lo[1] = acc[t][1];
    hi[0] = acc[t][2];
    hi[1] = acc[t][3];
  }
  cluster.sync();

  const int pair_begin = crank * 32 / csize, pair_end = (crank + 1) * 32 / csize;
  const int items = (pair_end - pair_begin) * p.m;
  for (int it = tid; it < items; it += kWarps * 32) {
    const int pp = pair_begin + it / p.m, m = it % p.m;
    const int w = pp / 8, gg = pp % 8;
    const int rlo = w * 16 + gg, rhi = rlo + 8;
    float plo[kMaxCluster], phi[kMaxCluster];
#pragma unroll
    for (int r = 0; r < kMaxCluster; ++r) {
      if (r < csize) {
        const float* rp = cluster.map_shared_rank(sP, r);
        plo[r] = rp[rlo * 16 + m];
        phi[r] = rp[rhi * 16 + m];
      }
    }
    float vlo = 0.0f, vhi = 0.0f;
#pragma unroll
    for (int r = 0; r < kMaxCluster; ++r) {
      if (r < csize) {
        vlo += plo[r];
        vhi += phi[r];
      }
    }
    int jlo, nlo, jhi, nhi;
    row_of<MODE>(p, y, w, gg, jlo, nlo);
    row_of<MODE>(p, y, w, gg + 8, jhi, nhi);
    if (FMT == 1) {
      vlo *= sS[rlo];
      vhi *= sS[rhi];
    }
    if constexpr (MODE == 0) {
      if (p.res[jlo]) vlo += bf2f(p.res[jlo][int64_t(m) * p.n[jlo] + nlo]);
      if (p.res[jhi]) vhi += bf2f(p.res[jhi][int64_t(m) * p.n[jhi] + nhi]);
      p.y[jlo][int64_t(m) * p.n[jlo] + nlo] = f2bf(vlo);
      p.y[jhi][int64_t(m) * p.n[jhi] + nhi] = f2bf(vhi);
    } else if constexpr (MODE == 1) {
      const float silu = vlo / (1.0f + expf(-vlo));
      p.y[0][int64_t(m) * p.n[0] + nlo] = f2bf(silu * vhi);
    } else {
      const QkvExtra& e = p.qkv;
      const int hd = e.head_dim, half = hd / 2;
      const int head_in_job = nlo / hd, i = nlo % hd;  // i < half: the pair's first row
      // The linear output is a bf16 value; round before the rotation.
      double xlo = bf2f(f2bf(vlo)), xhi = bf2f(f2bf(vhi));
      const int pos = e.pos[m];
      if (jlo < 2) {
        const double inv = pow(e.theta, -2.0 * double(i) / double(hd));
        double sn, cs;
        sincos(double(pos) * inv, &sn, &cs);
        const double a = xlo * cs - xhi * sn, b = xhi * cs + xlo * sn;
        xlo = double(float(a));
        xhi = double(float(b));
      }
      const uint16_t olo = f2bf(float(xlo)), ohi = f2bf(float(xhi));
      if (jlo == 0) {
        uint16_t* qo = e.q_out + int64_t(m) * e.hq * hd + head_in_job * hd;
        qo[i] = olo;
        qo[i + half] = ohi;
      } else {
        uint16_t* side = jlo == 1 ? e.k_out : e.v_out;
        if (side) {
          uint16_t* so = side + int64_t(m) * e.hkv * hd + head_in_job * hd;
          so[i] = olo;
          so[i + half] = ohi;
        }
        if (pos >= 0 && pos < e.max_len) {
          const int seq = (p.m_base + m) / e.tokens_per_seq;
          uint16_t* cache = jlo == 1 ? e.k_cache : e.v_cache;
          uint16_t* dst = cache + ((int64_t(seq) * e.hkv + head_in_job) * e.max_len + pos) * hd;
          dst[i] = olo;
          dst[i + half] = ohi;
        } else if (e.err) {
          atomicExch(e.err, 2);
        }
      }
    }
  }
  cluster.sync();  // keep this block's partials alive until every rank has read them
}

template <int FMT, int NT, int MODE>
int launch_one(const Params& p, int cluster, int row_blocks, size_t smem, bool pdl, cudaStream_t st) {
  auto kern = gemv_mma_kernel<FMT, NT, MODE>;
  static bool configured = false;
  if (!configured) {
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024) != cudaSuccess)
      return SB_INTERNAL;
    configured = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(cluster, row_blocks, 1);
  cfg.blockDim = dim3(kWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  attrs[na].id = cudaLaunchAttributeClusterDimension;
  attrs[na].val.clusterDim.x = cluster;
  attrs[na].val.clusterDim.y = 1;
  attrs[na].val.clusterDim.z = 1;
  ++na;
  if (pdl) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  if (cudaLaunchKernelEx(&cfg, kern, p) != cudaSuccess) return SB_INTERNAL;
  count_launch();
  return SB_OK;
}

template <int FMT, int NT>
int dispatch_mode(GemvMode mode, const Params& p, int cluster, int rb, size_t smem, bool pdl,
                  cudaStream_t st) {
  switch (mode) {
    case GemvMode::Plain: return launch_one<FMT, NT, 0>(p, cluster, rb, smem, pdl, st);
    case GemvMode::SwiGLU: return launch_one<FMT, NT, 1>(p, cluster, rb, smem, pdl, st);
    case GemvMode::QkvRope: return launch_one<FMT, NT, 2>(p, cluster, rb, smem, pdl, st);
  }
  return SB_INVALID_ARGUMENT;
}

}  // namespace

bool gemv_mma_supported(const GemvMmaArgs& a) {
  const LinearBatch& b = a.lb;
  if (b.fmt != WFormat::W4G32 && b.fmt != WFormat::W8PC) return false;
  if (b.k % 32 || b.m <= 0) return false;
  if (b.k / 32 > kMaxCluster * kMaxGroupsPerBlock) return false;
  auto aligned = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (!aligned(b.x)) return false;
  for (int j = 0; j < b.njobs; ++j)
    if (!aligned(b.jobs[j].w)) return false;
  switch (a.mode) {
    case GemvMode::Plain:
      if (b.epi == Epilogue::SwiGLU) return false;
      for (int j = 0; j < b.njobs; ++j)
        if (b.jobs[j].n % kRows || b.jobs[j].n <= 0) return false;
      return true;
    case GemvMode::SwiGLU:
      return b.njobs == 2 && b.jobs[0].n == b.jobs[1].n && b.jobs[0].n % 32 == 0 && b.jobs[0].n > 0;
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
  int cluster = (groups + 15) / 16;
  if (cluster > kMaxCluster) cluster = kMaxCluster;
  if (cluster < 1) cluster = 1;
  const int gpb = (groups + cluster - 1) / cluster;
  if (gpb > kMaxGroupsPerBlock) return SB_INVALID_ARGUMENT;
  int rows = 0;
  switch (a.mode) {
    case GemvMode::Plain:
      for (int j = 0; j < b.njobs; ++j) rows += b.jobs[j].n;
      break;
    case GemvMode::SwiGLU: rows = 2 * b.jobs[0].n; break;
    case GemvMode::QkvRope: rows = b.jobs[0].n + b.jobs[1].n + b.jobs[2].n; break;
  }
  const int row_blocks = rows / kRows;
  const int bpg = fmt == 0 ? 16 : 32;
  const int xs_stride = ((gpb * 64 + 127) / 128) * 128 + 64;
  auto smem_for = [&](int nt) {
    return size_t(kRows) * gpb * bpg + (fmt == 0 ? kRows * gpb : kRows) * sizeof(float) +
           size_t(nt) * 8 * xs_stride + kRows * 16 * sizeof(float);
  };
  if (smem_for(2) > 200 * 1024) return SB_INVALID_ARGUMENT;

  for (int m0 = 0; m0 < b.m; m0 += 16) {
    Params p{};
    p.m = b.m - m0 < 16 ? b.m - m0 : 16;
    p.x = b.x + int64_t(m0) * b.k;
    p.k = b.k;
    p.groups = groups;
    p.gpb = gpb;
    p.xs_stride = xs_stride;
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
      // Row offsets of this chunk: positions and outputs advance by m0 rows;
      // cache rows are addressed by sequence, which also advances.
      p.qkv.pos = e.pos + m0;
      p.qkv.q_out = e.q_out + int64_t(m0) * e.hq * e.head_dim;
      p.qkv.k_out = e.k_out ? e.k_out + int64_t(m0) * e.hkv * e.head_dim : nullptr;
      p.qkv.v_out = e.v_out ? e.v_out + int64_t(m0) * e.hkv * e.head_dim : nullptr;
    }
    const bool two = p.m > 8;
    const size_t smem = smem_for(two ? 2 : 1);
    int rc;
    if (fmt == 0)
      rc = two ? dispatch_mode<0, 2>(a.mode, p, cluster, row_blocks, smem, a.pdl, st)
               : dispatch_mode<0, 1>(a.mode, p, cluster, row_blocks, smem, a.pdl, st);
    else
      rc = two ? dispatch_mode<1, 2>(a.mode, p, cluster, row_blocks, smem, a.pdl, st)
               : dispatch_mode<1, 1>(a.mode, p, cluster, row_blocks, smem, a.pdl, st);
    if (rc) return rc;
  }
  return SB_OK;
}

}  // namespace sb
