// Prefill attention on tensor cores (bf16, head_dim 64 or 128, MHA and GQA).
//
// Same semantics as the decode kernels: query row r of sequence r / S
// (S = tokens per sequence) attends to cache positions 0..pos[r] of that
// sequence, after the step's KV append has written every row's k and v.
// With pos = 0..S-1 this is causal self-attention over the prompt.
//
// Grid (64-row query tile, query head, sequence); 4 warps, 16 query rows
// each.  The CTA walks 64-position K/V tiles up to the largest position of
// its rows, double-buffered in shared memory with cp.async (rows padded so
// that ldmatrix reads are free of bank conflicts).  Per KV tile each warp
// runs S = Q K^T (mma.sync m16n8k16, Q held in registers), an online softmax
// in base 2 with the per-row causal mask, and O += P V with P taken straight
// from the score accumulators and V through ldmatrix.trans.
#include "common.cuh"
#include "k_elem.cuh"

namespace sb {

namespace {

constexpr int kPfWarps = 4;
constexpr int kPfRows = 16 * kPfWarps;  // query rows per CTA
constexpr int kPfKv = 64;               // positions per KV tile
constexpr float kPfLog2e = 1.4426950408889634f;

template <int D>
struct PfLayout {
  static constexpr int kRow = D * 2 + 16;
  static constexpr int kTile = kPfKv * kRow;      // one K or V tile
  static constexpr int kStage = 2 * kTile;        // K then V
  static constexpr int kBytes = 2 * kStage + kPfRows * 4;  // two stages + row positions
};

__device__ __forceinline__ void pf_mma(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                       uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

__device__ __forceinline__ void pf_ldsm4(uint32_t (&r)[4], const void* p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

__device__ __forceinline__ void pf_ldsm4t(uint32_t (&r)[4], const void* p) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(p));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

__device__ __forceinline__ void pf_cp16z(void* smem, const void* gmem, int src_bytes) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(a), "l"(gmem), "r"(src_bytes) : "memory");
}

__device__ __forceinline__ uint32_t pf_pack(float lo, float hi) {
  const __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&v);
}

template <int D>
__global__ void __launch_bounds__(kPfWarps * 32)
    attn_prefill_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ kc,
                        const uint16_t* __restrict__ vc, const int32_t* __restrict__ pos, int tokens_per_seq,
                        int heads, int kv_heads, int max_len, uint16_t* __restrict__ out, int* err) {
  using Lay = PfLayout<D>;
  constexpr int kCpr = D / 8;  // 16-byte chunks per row
  extern __shared__ __align__(128) uint8_t smem[];
  int* s_pos = reinterpret_cast<int*>(smem + 2 * Lay::kStage);
  __shared__ int s_len;
  const int tile = blockIdx.x, h = blockIdx.y, seq = blockIdx.z;
  const int G = heads / kv_heads, kvh = h / G;
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, qd = lane & 3;
  const int t_first = tile * kPfRows;                    // first query token of the tile in its sequence
  const int n_rows = min(kPfRows, tokens_per_seq - t_first);
  const int64_t row0 = int64_t(seq) * tokens_per_seq + t_first;
  const int64_t head_off = (int64_t(seq) * kv_heads + kvh) * int64_t(max_len) * D;
  const uint8_t* kb = reinterpret_cast<const uint8_t*>(kc + head_off);
  const uint8_t* vb = reinterpret_cast<const uint8_t*>(vc + head_off);

  pdl_trigger();
  pdl_wait();  // q and the appended cache rows come from the previous kernels

  if (tid == 0) s_len = 0;
  __syncthreads();
  if (tid < kPfRows) {
    int p = -1;
    if (tid < n_rows) {
      p = pos[row0 + tid];
      if (p < 0 || p >= max_len) {
        if (err) atomicExch(err, 2);
        p = -1;
      }
    }
    s_pos[tid] = p;
    if (p >= 0) atomicMax(&s_len, p + 1);
  }
  __syncthreads();
  const int len = s_len;
  const int ntiles = (len + kPfKv - 1) / kPfKv;

  auto load_tile = [&](int t, int stage) {
    uint8_t* sk = smem + stage * Lay::kStage;
    uint8_t* sv = sk + Lay::kTile;
    const int base = t * kPfKv;
    for (int c = tid; c < 2 * kPfKv * kCpr; c += kPfWarps * 32) {
      const int isv = c >= kPfKv * kCpr;
      const int cc = c - isv * kPfKv * kCpr;
      const int r = cc / kCpr, col = cc % kCpr;
      const bool ok = base + r < len;
      const uint8_t* src = (isv ? vb : kb) + int64_t(ok ? base + r : 0) * (D * 2) + col * 16;
      pf_cp16z((isv ? sv : sk) + r * Lay::kRow + col * 16, src, ok ? 16 : 0);
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
  };

  // Q fragments of the warp's 16 rows (rows g and g + 8), zero beyond the tile.
  const int lr0 = warp * 16 + g, lr1 = lr0 + 8;
  uint32_t qa[D / 16][4];
  {
    const uint32_t* q0 = reinterpret_cast<const uint32_t*>(q + (row0 + lr0) * int64_t(heads) * D + int64_t(h) * D);
    const uint32_t* q1 = reinterpret_cast<const uint32_t*>(q + (row0 + lr1) * int64_t(heads) * D + int64_t(h) * D);
    const bool v0 = lr0 < n_rows, v1 = lr1 < n_rows;
#pragma unroll
    for (int k = 0; k < D / 16; ++k) {
      qa[k][0] = v0 ? q0[k * 8 + qd] : 0u;
      qa[k][1] = v1 ? q1[k * 8 + qd] : 0u;
      qa[k][2] = v0 ? q0[k * 8 + 4 + qd] : 0u;
      qa[k][3] = v1 ? q1[k * 8 + 4 + qd] : 0u;
    }
  }
  const int p0 = s_pos[lr0], p1 = s_pos[lr1];
  const int wmax = __reduce_max_sync(0xffffffffu, max(p0, p1));  // last position any row of the warp sees
  const float scale = kPfLog2e * (D == 128 ? 0.08838834764831845f : 0.125f);  // log2(e) / sqrt(D)

  float o[D / 8][4];
#pragma unroll
  for (int n = 0; n < D / 8; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.0f;
  float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.0f, l1 = 0.0f;
  const int mi = lane >> 3, rr = lane & 7;

  if (ntiles > 0) load_tile(0, 0);
  for (int t = 0; t < ntiles; ++t) {
    if (t + 1 < ntiles) {
      load_tile(t + 1, (t + 1) & 1);
      asm volatile("cp.async.wait_group 1;" ::: "memory");
    } else {
      asm volatile("cp.async.wait_group 0;" ::: "memory");
    }
    __syncthreads();
    const uint8_t* sk = smem + (t & 1) * Lay::kStage;
    const uint8_t* sv = sk + Lay::kTile;
    const int base = t * kPfKv;
    if (base <= wmax) {  // warp-uniform: tiles past every row of this warp are skipped
      float s[kPfKv / 8][4];
#pragma unroll
      for (int j = 0; j < kPfKv / 8; ++j) s[j][0] = s[j][1] = s[j][2] = s[j][3] = 0.0f;
#pragma unroll
      for (int k = 0; k < D / 16; ++k) {
#pragma unroll
        for (int j = 0; j < kPfKv / 8; j += 2) {
          uint32_t b[4];
          pf_ldsm4(b, sk + (j * 8 + (mi >> 1) * 8 + rr) * Lay::kRow + k * 32 + (mi & 1) * 16);
          pf_mma(s[j], qa[k][0], qa[k][1], qa[k][2], qa[k][3], b[0], b[1]);
          pf_mma(s[j + 1], qa[k][0], qa[k][1], qa[k][2], qa[k][3], b[2], b[3]);
        }
      }
      // Mask, scale, row maxima (rows g: elements 0-1, g + 8: elements 2-3).
      float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
      for (int j = 0; j < kPfKv / 8; ++j)
#pragma unroll
        for (int e = 0; e < 2; ++e) {
          const int tpos = base + j * 8 + 2 * qd + e;
          s[j][e] = tpos <= p0 ? s[j][e] * scale : -INFINITY;
          s[j][2 + e] = tpos <= p1 ? s[j][2 + e] * scale : -INFINITY;
          mx0 = fmaxf(mx0, s[j][e]);
          mx1 = fmaxf(mx1, s[j][2 + e]);
        }
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
      mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
      mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
      const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
      const float u0 = n0 == -INFINITY ? 0.0f : n0, u1 = n1 == -INFINITY ? 0.0f : n1;
      const float c0 = exp2f(m0 - u0), c1 = exp2f(m1 - u1);
      float ps0 = 0.0f, ps1 = 0.0f;
#pragma unroll
      for (int j = 0; j < kPfKv / 8; ++j) {
        s[j][0] = exp2f(s[j][0] - u0);
        s[j][1] = exp2f(s[j][1] - u0);
        s[j][2] = exp2f(s[j][2] - u1);
        s[j][3] = exp2f(s[j][3] - u1);
        ps0 += s[j][0] + s[j][1];
        ps1 += s[j][2] + s[j][3];
      }
      l0 = l0 * c0 + ps0;
      l1 = l1 * c1 + ps1;
      m0 = n0;
      m1 = n1;
#pragma unroll
      for (int n = 0; n < D / 8; ++n) {
        o[n][0] *= c0;
        o[n][1] *= c0;
        o[n][2] *= c1;
        o[n][3] *= c1;
      }
      // O += P V, 16 positions per k-step.
#pragma unroll
      for (int ks = 0; ks < kPfKv / 16; ++ks) {
        const uint32_t a0 = pf_pack(s[2 * ks][0], s[2 * ks][1]);
        const uint32_t a1 = pf_pack(s[2 * ks][2], s[2 * ks][3]);
        const uint32_t a2 = pf_pack(s[2 * ks + 1][0], s[2 * ks + 1][1]);
        const uint32_t a3 = pf_pack(s[2 * ks + 1][2], s[2 * ks + 1][3]);
#pragma unroll
        for (int nb = 0; nb < D / 16; ++nb) {
          uint32_t v[4];
          pf_ldsm4t(v, sv + (ks * 16 + (mi & 1) * 8 + rr) * Lay::kRow + (2 * nb + (mi >> 1)) * 16);
          pf_mma(o[2 * nb], a0, a1, a2, a3, v[0], v[1]);
          pf_mma(o[2 * nb + 1], a0, a1, a2, a3, v[2], v[3]);
        }
      }
    }
    __syncthreads();  // the stage is refilled two tiles later
  }

  l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
  l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
  l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
  const float i0 = l0 > 0.0f ? 1.0f / l0 : 0.0f, i1 = l1 > 0.0f ? 1.0f / l1 : 0.0f;
  if (lr0 < n_rows) {
    uint32_t* o0 = reinterpret_cast<uint32_t*>(out + (row0 + lr0) * int64_t(heads) * D + int64_t(h) * D);
#pragma unroll
    for (int n = 0; n < D / 8; ++n) o0[n * 4 + qd] = pf_pack(o[n][0] * i0, o[n][1] * i0);
  }
  if (lr1 < n_rows) {
    uint32_t* o1 = reinterpret_cast<uint32_t*>(out + (row0 + lr1) * int64_t(heads) * D + int64_t(h) * D);
#pragma unroll
    for (int n = 0; n < D / 8; ++n) o1[n * 4 + qd] = pf_pack(o[n][2] * i1, o[n][3] * i1);
  }
}

template <int D>
int launch_pf(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int32_t* pos, int64_t batch,
              int64_t tps, int64_t heads, int64_t kv_heads, int64_t max_len, uint16_t* out, int* err,
              cudaStream_t st) {
  using Lay = PfLayout<D>;
  static PerDeviceOnce configured;
  if (!configured.run([] {
        return cudaFuncSetAttribute(attn_prefill_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, Lay::kBytes) ==
               cudaSuccess;
      }))
    return SB_INTERNAL;
  const dim3 grid{unsigned((tps + kPfRows - 1) / kPfRows), unsigned(heads), unsigned(batch)};
  if (launch_pdl(attn_prefill_kernel<D>, grid, dim3(kPfWarps * 32), size_t(Lay::kBytes), st, q, kc, vc, pos,
                 int(tps), int(heads), int(kv_heads), int(max_len), out, err) != cudaSuccess)
    return SB_INTERNAL;
  count_launch();
  return SB_OK;
}

}  // namespace

bool attention_prefill_supported(int64_t rows, int64_t tokens_per_seq, int64_t heads, int64_t kv_heads,
                                 int64_t head_dim) {
  return tokens_per_seq >= 16 && rows % tokens_per_seq == 0 && attention_tc_supported(heads, kv_heads, head_dim) &&
         heads <= 65535 && rows / tokens_per_seq <= 65535;
}

int launch_attention_prefill(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* pos,
                             int64_t rows, int64_t tokens_per_seq, int64_t heads, int64_t kv_heads, int64_t head_dim,
                             int64_t max_len, uint16_t* out, int* err, cudaStream_t st) {
  if (!attention_prefill_supported(rows, tokens_per_seq, heads, kv_heads, head_dim)) return SB_INVALID_ARGUMENT;
  const int64_t batch = rows / tokens_per_seq;
  if (head_dim == 128)
    return launch_pf<128>(q, k_cache, v_cache, pos, batch, tokens_per_seq, heads, kv_heads, max_len, out, err, st);
  return launch_pf<64>(q, k_cache, v_cache, pos, batch, tokens_per_seq, heads, kv_heads, max_len, out, err, st);
}

}  // namespace sb
