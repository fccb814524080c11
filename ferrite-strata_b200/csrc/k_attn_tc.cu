// Tensor-core decode attention: bf16 KV cache, head_dim 64 or 128, up to 8
// query heads per kv head (MHA and GQA).
//
// Grid (split, kv head, query row).  A CTA owns `span` consecutive cache
// positions of one (row, kv head) and its 4 warps take 16-position slabs of
// that span in turn (slab w, w + 4, ...).  Each warp streams its slabs
// through its own 3-deep cp.async ring (K and V rows, padded so that ldmatrix
// rows land in distinct banks) and runs, per slab,
//
//   S^T[16 heads x 16 positions] = Q[16 x D] . K^T        (mma.sync m16n8k16)
//   online softmax per head row, in base 2
//   O[16 heads x D] += P[16 x 16] . V[16 x D]              (V via ldmatrix.trans)
//
// Q rows beyond the group size are zero, so one m16 tile covers any group of
// up to 8 heads.  Computing S transposed makes the score accumulators exactly
// the A fragment of P . V, so P never leaves registers.  At the end the warps
// merge their (max, sum, O) through shared memory.  The splits of one
// (row, kv head) -- at most 8 -- are launched as one thread-block cluster, and
// CTA 0 of the cluster merges the splits through distributed shared memory
// and writes the output: no partials reach HBM and no merge kernel runs.
//
// In a decode step (one token per sequence) the cache rows below the row's
// position were written by earlier steps, so when positions are a graph input
// the first slabs below the position are requested before griddepcontrol.wait
// and stream in while the previous kernel (the q/k/v projection that writes
// row `pos`) finishes.
#include <cooperative_groups.h>

#include "common.cuh"
#include "k_elem.cuh"

namespace sb {

namespace {

constexpr int kTcWarps = 4;
constexpr int kSlab = 16;    // positions per warp step
constexpr int kTcDepth = 3;  // slabs in flight per warp
constexpr float kLog2e = 1.4426950408889634f;
constexpr int kMaxSplits = 8;  // splits of one (row, kv head) form one thread-block cluster (portable size)

template <int D>
struct TcLayout {
  static constexpr int kRow = D * 2 + 16;              // padded row bytes
  static constexpr int kSlabBytes = 2 * kSlab * kRow;  // K rows, then V rows
  static constexpr int kWarpBytes = kTcDepth * kSlabBytes;
  static constexpr int kBytes = kTcWarps * kWarpBytes;
  // The final merges reuse the ring: per warp O [warps][8][D], max and sum
  // [warps][8]; then the CTA's merged O [8][D], max and sum [8].
  static_assert((kTcWarps * 8 * D + 2 * kTcWarps * 8 + 8 * D + 16) * 4 <= kBytes, "merge area");
};

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a2, uint32_t b0, uint32_t b1) {
  // Rows 8..15 of A are zero (a1 = a3 = 0).
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(0u), "r"(a2), "r"(0u), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void ldsm4(uint32_t (&r)[4], const void* p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

__device__ __forceinline__ void ldsm4t(uint32_t (&r)[4], const void* p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

// 16-byte copy that reads `src_bytes` (16 or 0) and zero-fills the rest.
__device__ __forceinline__ void cp16z(void* smem, const void* gmem, int src_bytes) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(a), "l"(gmem), "r"(src_bytes) : "memory");
}

__device__ __forceinline__ uint32_t pack2(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

template <int D>
__global__ void __launch_bounds__(kTcWarps * 32)
    attn_tc_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ kc,
                   const uint16_t* __restrict__ vc, const int32_t* __restrict__ pos, int tokens_per_seq,
                   int heads, int kv_heads, int max_len, int span, int splits, int pos_external,
                   int cluster_merge, float* __restrict__ partial, uint16_t* __restrict__ out, int* err,
                   KvPages kp) {
  using Lay = TcLayout<D>;
  constexpr int kCpr = D / 8;  // 16-byte chunks per row
  extern __shared__ __align__(128) uint8_t smem[];
  const int split = blockIdx.x, kvh = blockIdx.y, row = blockIdx.z;
  const int G = heads / kv_heads;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, qd = lane & 3;
  uint8_t* ring = smem + warp * Lay::kWarpBytes;
  const int seq = row / tokens_per_seq;
  const int t0 = split * span;

  pdl_trigger();

  // Copy slab i of this warp (global slab warp + 4 i of the span): rows below
  // `valid` are read, the rest zero-filled (their scores are masked and their
  // V rows must be finite zeros).  A slab's 16 positions are consecutive rows
  // of one page (spans are whole multiples of 64 positions, pages of 16 or
  // more); a slab whose page index is bad is zero-filled and sets error word 6.
  // Always commits one group.
  auto issue = [&](int i, int lim) {
    const int s = t0 + (warp + kTcWarps * i) * kSlab;
    const int valid = min(kSlab, max(0, lim - s));
    if (valid > 0) {
      const int64_t srow = kv_row(kp, seq, kvh, kv_heads, max_len, s);
      const int rd = srow < 0 ? 0 : valid;  // rows read
      if (srow < 0 && lane == 0 && err) atomicExch(err, 6);
      const uint8_t* kb = reinterpret_cast<const uint8_t*>(kc + (srow < 0 ? 0 : srow * D));
      const uint8_t* vb = reinterpret_cast<const uint8_t*>(vc + (srow < 0 ? 0 : srow * D));
      uint8_t* dst = ring + (i % kTcDepth) * Lay::kSlabBytes;
#pragma unroll
      for (int j = 0; j < 2 * kSlab * kCpr / 32; ++j) {
        const int c = lane + 32 * j;             // chunk: K rows first, then V rows
        const int isv = c >= kSlab * kCpr;
        const int cc = c - isv * kSlab * kCpr;
        const int r = cc / kCpr, col = cc % kCpr;
        const int rr = r < rd ? r : 0;           // a readable address for zero-filled rows
        const uint8_t* src = (isv ? vb : kb) + int64_t(rr) * (D * 2) + col * 16;
        cp16z(dst + (isv * kSlab + r) * Lay::kRow + col * 16, src, r < rd ? 16 : 0);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  // Before the wait: slabs entirely below the row's position.
  int issued = 0;
  if (pos_external && tokens_per_seq == 1) {
    const int p_early = pos[row];
    if (p_early > 0 && p_early < max_len) {
      const int lim_pre = min(p_early, t0 + span);
      while (issued < kTcDepth && t0 + (warp + kTcWarps * issued + 1) * kSlab <= lim_pre) {
        issue(issued, lim_pre);
        ++issued;
      }
    }
  }
  pdl_wait();
  const int p = pos[row];
  const bool bad = p < 0 || p >= max_len;
  if (bad && tid == 0 && err) atomicExch(err, 2);
  const int lim = bad ? t0 : min(p + 1, t0 + span);  // positions [t0, lim) of this CTA
  const int slabs = (max(0, lim - t0) + kSlab - 1) / kSlab;
  const int mine = max(0, (slabs - warp + kTcWarps - 1) / kTcWarps);
  for (int i = issued; i < kTcDepth; ++i) issue(i, lim);

  // Q as the A fragment (head row g of the group; rows >= G are zero).
  uint32_t qa0[D / 16], qa2[D / 16];
  {
    const bool live = g < G;
    const uint32_t* qr =
        reinterpret_cast<const uint32_t*>(q + int64_t(row) * heads * D + int64_t(kvh * G + (live ? g : 0)) * D);
#pragma unroll
    for (int k = 0; k < D / 16; ++k) {
      qa0[k] = live ? qr[k * 8 + qd] : 0u;
      qa2[k] = live ? qr[k * 8 + 4 + qd] : 0u;
    }
  }
  const float scale = kLog2e * (D == 128 ? 0.08838834764831845f : 0.125f);  // log2(e) / sqrt(D)

  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  float m_run = -INFINITY, l_run = 0.0f;
  const int mi = lane >> 3, rr = lane & 7;

  for (int i = 0; i < mine; ++i) {
    asm volatile("cp.async.wait_group %0;" ::"n"(kTcDepth - 1) : "memory");
    __syncwarp();
    const uint8_t* sK = ring + (i % kTcDepth) * Lay::kSlabBytes;
    const uint8_t* sV = sK + kSlab * Lay::kRow;
    const int s0 = t0 + (warp + kTcWarps * i) * kSlab;

    float sc[2][4] = {{0.0f, 0.0f, 0.0f, 0.0f}, {0.0f, 0.0f, 0.0f, 0.0f}};
#pragma unroll
    for (int k = 0; k < D / 16; ++k) {
      uint32_t b[4];
      ldsm4(b, sK + ((mi >> 1) * 8 + rr) * Lay::kRow + k * 32 + (mi & 1) * 16);
      mma16816(sc[0], qa0[k], qa2[k], b[0], b[1]);
      mma16816(sc[1], qa0[k], qa2[k], b[2], b[3]);
    }
    // sc[n][0..1]: head g, positions s0 + 8n + 2qd + {0, 1}.
    float pv[2][2];
    float mx = -INFINITY;
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        const int t = s0 + 8 * n + 2 * qd + e;
        pv[n][e] = t < lim ? sc[n][e] * scale : -INFINITY;
        mx = fmaxf(mx, pv[n][e]);
      }
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 1));
    mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, 2));
    const float m_new = fmaxf(m_run, mx);
    const float m_use = m_new == -INFINITY ? 0.0f : m_new;
    const float corr = exp2f(m_run - m_use);
    float psum = 0.0f;
#pragma unroll
    for (int n = 0; n < 2; ++n)
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        pv[n][e] = exp2f(pv[n][e] - m_use);
        psum += pv[n][e];
      }
    l_run = l_run * corr + psum;
    m_run = m_new;
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      o[n][0] *= corr;
      o[n][1] *= corr;
    }
    const uint32_t pa0 = pack2(pv[0][0], pv[0][1]), pa2 = pack2(pv[1][0], pv[1][1]);
#pragma unroll
    for (int nb = 0; nb < D / 16; ++nb) {
      uint32_t v[4];
      ldsm4t(v, sV + ((mi & 1) * 8 + rr) * Lay::kRow + (2 * nb + (mi >> 1)) * 16);
      mma16816(o[2 * nb], pa0, pa2, v[0], v[1]);
      mma16816(o[2 * nb + 1], pa0, pa2, v[2], v[3]);
    }
    __syncwarp();
    issue(i + kTcDepth, lim);
  }
  asm volatile("cp.async.wait_group 0;" ::: "memory");
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 1);
  l_run += __shfl_xor_sync(0xffffffffu, l_run, 2);
  __syncthreads();  // every warp is done with its ring

  float* sO = reinterpret_cast<float*>(smem);     // [warps][8][D]
  float* sM = sO + kTcWarps * 8 * D;              // [warps][8]
  float* sL = sM + kTcWarps * 8;                  // [warps][8]
  float* cO = sL + kTcWarps * 8;                  // [8][D]: this CTA's merged O (cluster merge)
  float* cM = cO + 8 * D;                         // [8]
  float* cL = cM + 8;                             // [8]
  if (g < G) {
#pragma unroll
    for (int n = 0; n < D / 8; ++n) {
      sO[(warp * 8 + g) * D + n * 8 + 2 * qd] = o[n][0];
      sO[(warp * 8 + g) * D + n * 8 + 2 * qd + 1] = o[n][1];
    }
    if (qd == 0) {
      sM[warp * 8 + g] = m_run;
      sL[warp * 8 + g] = l_run;
    }
  }
  __syncthreads();
  for (int it = tid; it < G * D; it += kTcWarps * 32) {
    const int h = it / D, d = it % D;
    float M = -INFINITY;
#pragma unroll
    for (int w = 0; w < kTcWarps; ++w) M = fmaxf(M, sM[w * 8 + h]);
    float acc = 0.0f, L = 0.0f;
#pragma unroll
    for (int w = 0; w < kTcWarps; ++w) {
      const float mw = sM[w * 8 + h];
      const float wt = mw == -INFINITY ? 0.0f : exp2f(mw - M);
      acc = fmaf(wt, sO[(w * 8 + h) * D + d], acc);
      L = fmaf(wt, sL[w * 8 + h], L);
    }
    const int hh = kvh * G + h;
    if (cluster_merge) {
      cO[h * D + d] = acc;
      if (d == 0) {
        cM[h] = M;
        cL[h] = L;
      }
    } else if (splits == 1) {
      out[int64_t(row) * heads * D + int64_t(hh) * D + d] = f2bf(L > 0.0f ? acc / L : 0.0f);
    } else {
      float* pp = partial + ((int64_t(row) * heads + hh) * splits + split) * (D + 2);
      pp[2 + d] = acc;
      if (d == 0) {
        pp[0] = M == -INFINITY ? -INFINITY : M / kLog2e;  // natural-log units for the merge
        pp[1] = L;
      }
    }
  }
  if (cluster_merge) {
    // The splits of this (row, kv head) are one cluster: after the cluster
    // barrier CTA 0 reads every CTA's (max, sum, O) through distributed
    // shared memory and writes the output; the second barrier keeps the
    // other CTAs' shared memory alive until it has.
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    cluster.sync();
    if (split == 0) {
      for (int it = tid; it < G * D; it += kTcWarps * 32) {
        const int h = it / D, d = it % D;
        float M = -INFINITY;
        for (int r = 0; r < splits; ++r) M = fmaxf(M, cluster.map_shared_rank(cM, r)[h]);
        float acc = 0.0f, L = 0.0f;
        for (int r = 0; r < splits; ++r) {
          const float mr = cluster.map_shared_rank(cM, r)[h];
          const float wt = mr == -INFINITY ? 0.0f : exp2f(mr - M);
          acc = fmaf(wt, cluster.map_shared_rank(cO, r)[h * D + d], acc);
          L = fmaf(wt, cluster.map_shared_rank(cL, r)[h], L);
        }
        out[int64_t(row) * heads * D + int64_t(kvh * G + h) * D + d] = f2bf(L > 0.0f ? acc / L : 0.0f);
      }
    }
    cluster.sync();
  }
}

template <int D>
int launch_tc(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int32_t* pos, int64_t rows,
              int64_t tps, int64_t heads, int64_t kv_heads, int64_t max_len, bool pos_external, float* scratch,
              uint16_t* out, int* err, cudaStream_t st, const KvPages& kp) {
  using Lay = TcLayout<D>;
  static PerDeviceOnce configured;
  if (!configured.run([] {
        return cudaFuncSetAttribute(attn_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kBytes) ==
               cudaSuccess;
      }))
    return SB_INTERNAL;
  const int span = attention_tc_span(rows, kv_heads, max_len);
  const int splits = int((max_len + span - 1) / span);
  // Splits merge inside their cluster; no partials reach memory.
  const int cluster_merge = splits > 1 ? 1 : 0;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(splits), unsigned(kv_heads), unsigned(rows));
  cfg.blockDim = dim3(kTcWarps * 32, 1, 1);
  cfg.dynamicSmemBytes = size_t(Lay::kBytes);
  cfg.stream = st;
  cudaLaunchAttribute attrs[2];
  int na = 0;
  if (pdl_enabled()) {
    attrs[na].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attrs[na].val.programmaticStreamSerializationAllowed = 1;
    ++na;
  }
  if (cluster_merge) {
    attrs[na].id = cudaLaunchAttributeClusterDimension;
    attrs[na].val.clusterDim.x = unsigned(splits);
    attrs[na].val.clusterDim.y = 1;
    attrs[na].val.clusterDim.z = 1;
    ++na;
  }
  cfg.attrs = attrs;
  cfg.numAttrs = na;
  if (cudaLaunchKernelEx(&cfg, attn_tc_kernel<D>, q, kc, vc, pos, int(tps), int(heads), int(kv_heads),
                         int(max_len), span, splits, pos_external ? 1 : 0, cluster_merge, scratch, out, err, kp) !=
      cudaSuccess)
    return SB_INTERNAL;
  count_launch();
  return SB_OK;
}

}  // namespace

int attention_tc_span(int64_t rows, int64_t kv_heads, int64_t max_len) {
  // About one wave (two 104 KB CTAs per SM), at most one cluster's worth of
  // splits, whole slabs of 64 positions per CTA.  Splitting further only
  // adds cluster merges: at 2049 cached positions, 256 (row, kv head) pairs
  // (7B batch 8; 70B batch 32 GQA) ran in 51 / 101 us with 2 splits against
  // 54 / 112 us with 3 and 60 / 119 us with 4; 32 pairs (7B batch 1) kept
  // improving up to 7-8 splits (26 -> 11 us).
  const int64_t pairs = rows * kv_heads;
  const int64_t most = (max_len + 63) / 64;
  int64_t splits = (2 * kNumSMs + pairs - 1) / pairs;
  if (splits > kMaxSplits) splits = kMaxSplits;
  if (splits > most) splits = most;
  if (splits < 1) splits = 1;
  const int64_t per = (max_len + splits - 1) / splits;
  return int((per + 63) / 64 * 64);
}

bool attention_tc_supported(int64_t heads, int64_t kv_heads, int64_t head_dim) {
  return kv_heads > 0 && heads % kv_heads == 0 && heads / kv_heads <= 8 && (head_dim == 64 || head_dim == 128);
}

int launch_attention_tc(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* pos,
                        int64_t rows, int64_t tokens_per_seq, int64_t heads, int64_t kv_heads, int64_t head_dim,
                        int64_t max_len, bool pos_external, float* scratch, uint16_t* out, int* err,
                        cudaStream_t st, const KvPages& kp) {
  if (rows == 0) return SB_OK;
  if (!attention_tc_supported(heads, kv_heads, head_dim) || rows > 65535 || kv_heads > 65535)
    return SB_INVALID_ARGUMENT;
  if (kp.paged() && (!kv_page_size_ok(kp.page_size) || int64_t(kp.page_size) * kp.pages_per_seq != max_len))
    return SB_INVALID_ARGUMENT;
  if (head_dim == 128)
    return launch_tc<128>(q, k_cache, v_cache, pos, rows, tokens_per_seq, heads, kv_heads, max_len, pos_external,
                          scratch, out, err, st, kp);
  return launch_tc<64>(q, k_cache, v_cache, pos, rows, tokens_per_seq, heads, kv_heads, max_len, pos_external,
                       scratch, out, err, st, kp);
}

}  // namespace sb
