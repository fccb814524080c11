// Prefill attention on the 5th-generation tensor cores (tcgen05, TMEM, TMA):
// bf16, head_dim 64 or 128, MHA and GQA.
//
// Same semantics as the decode kernels: query row r of sequence r / S
// (S = tokens per sequence) attends to cache positions 0..pos[r] of that
// sequence, after the step's KV append has written every row's k and v.
// With pos = 0..S-1 this is causal self-attention over the prompt.
//
// One CTA per (128-row query tile, query head, sequence), heaviest tiles
// first; 128-position K/V tiles up to the largest position of its rows.
// Per KV tile j, FlashAttention-style with both products on tcgen05.mma
// (kind::f16, M = 128, f32 accumulators in TMEM):
//   S = Q K^T        A = Q (loaded once), B = K tile, S in TMEM;
//   softmax          one thread per query row reads its S row from TMEM,
//                    masks positions past pos[r], and keeps a running row
//                    maximum in base 2; the probabilities P are written as
//                    bf16 into shared memory in the K-major 128-byte-swizzled
//                    layout the MMA reads.  O is rescaled (read, scaled,
//                    written back in TMEM) only when a row's maximum grows
//                    by more than 8 (a factor of 256), so P stays below 2^8;
//                    the row sum uses the same reference maximum, so the
//                    final O / l is exact;
//   O += P V         A = P, B = V^T: the V tile as loaded is [position][d],
//                    and a transposing warpgroup rewrites it [d][position]
//                    (ldmatrix.trans + stmatrix), zeroing positions at or past
//                    the tile's last needed position;
// and at the end O / l as bf16.
//
// Warps: 0 TMA (Q once, K and V double-buffered), 1 TMEM allocation and the
// MMA issuer (S two tiles ahead of P V, in two TMEM buffers, so the tensor
// cores compute the next scores while the softmax works), 2-5 softmax and
// output (TMEM lane quarter = warp % 4), 6-9 the V transpose.  Every
// mbarrier wait is bounded; one that runs out records error word 4 and the
// CTA winds down (the TMA thread lets its loads land, the TMEM owner frees its
// columns).  No TMA multicast.
#include "common.cuh"
#include "k_elem.cuh"
#include "k_tc.cuh"

namespace sb {

namespace {

using namespace tc;

constexpr int kQ = 128;    // query rows per CTA (TMEM lanes)
constexpr int kKV = 128;   // positions per KV tile
constexpr int kPfThreads = 320;
constexpr uint32_t kTmemColsPf = 512;  // two S buffers (128 columns each) and O (up to 128)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescale = 8.0f;  // log2 of the largest P before O is rescaled

template <int D>
struct PfLay {
  static constexpr int kKB = D / 64;                // 64-wide blocks of head_dim
  static constexpr int kQBytes = kQ * D * 2;        // Q: kKB blocks of [128 rows][128 B]
  static constexpr int kKBytes = kKV * D * 2;       // one K tile, same layout
  static constexpr int kVBytes = kKV * D * 2;       // the V tile as loaded
  static constexpr int kVtBytes = D * kKV * 2;      // V^T: 2 blocks (64 positions) of [D rows][128 B]
  static constexpr int kPBytes = kQ * kKV * 2;      // P: 2 blocks of [128 rows][128 B]
  static constexpr int kQOff = 0;
  static constexpr int kKOff = kQOff + kQBytes;     // 2 stages
  static constexpr int kVOff = kKOff + 2 * kKBytes;
  static constexpr int kVtOff = kVOff + 2 * kVBytes; // V: 2 stages
  static constexpr int kPOff = kVtOff + kVtBytes;
  static constexpr int kPosOff = kPOff + kPBytes;   // int [128] positions
  static constexpr int kBarOff = kPosOff + kQ * 4;  // mbarriers
  static constexpr int kBytes = kBarOff + 16 * 8 + 16 + 1024;
};

struct PfArgs {
  int tps, heads, kv_heads, max_len, qtiles;
  const int32_t* pos;
  uint16_t* out;
  int* err;
};

__device__ __forceinline__ void ldsm_x4_trans(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ void stsm_x4(uint32_t addr, const uint32_t (&r)[4]) {
  asm volatile("stmatrix.sync.aligned.m8n8.x4.shared.b16 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(r[0]), "r"(r[1]),
               "r"(r[2]), "r"(r[3])
               : "memory");
}

// 2^x by the hardware approximation (relative error about 2^-22).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ void sts128(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}

template <int D>
__global__ void __launch_bounds__(kPfThreads, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                           const __grid_constant__ CUtensorMap vmap, const PfArgs a) {
  using L = PfLay<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  int* s_pos = reinterpret_cast<int*>(smem + L::kPosOff);
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;   // [2]
  uint64_t* k_empty = bars + 3;  // [2]
  uint64_t* v_full = bars + 5;   // [2]
  uint64_t* v_empty = bars + 7;  // [2]
  uint64_t* s_full = bars + 9;   // [2]: S buffer b holds tile 2i + b
  uint64_t* s_used = bars + 11;  // [2]: the softmax has read S buffer b
  uint64_t* p_full = bars + 13;
  uint64_t* vt_full = bars + 14;
  uint64_t* pv_done = bars + 15;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 16);  // after 16 barriers
  __shared__ int s_len, s_fail;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int qt = a.qtiles - 1 - int(blockIdx.x);  // heaviest (latest) tiles first
  const int h = blockIdx.y, seq = blockIdx.z;
  const int kvh = h / (a.heads / a.kv_heads);
  const int t0 = qt * kQ;
  const int n_rows = min(kQ, a.tps - t0);
  const int64_t row0 = int64_t(seq) * a.tps + t0;
  const int kv_row0 = (seq * a.kv_heads + kvh) * a.max_len;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 4);
      mbar_init(&s_full[s], 1);
      mbar_init(&s_used[s], 4);
    }
    mbar_init(p_full, 4);
    mbar_init(vt_full, 4);
    mbar_init(pv_done, 1);
    s_len = 0;
    s_fail = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(tmem_slot)),
                 "r"(kTmemColsPf)
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  pdl_trigger();
  pdl_wait();  // q and the appended cache rows come from the previous kernels
  __syncthreads();
  if (threadIdx.x < kQ) {
    int p = -1;
    if (int(threadIdx.x) < n_rows) {
      p = a.pos[row0 + threadIdx.x];
      if (p < 0 || p >= a.max_len) {
        if (a.err) atomicExch(a.err, 2);
        p = -1;
      }
    }
    s_pos[threadIdx.x] = p;
    if (p >= 0) atomicMax(&s_len, p + 1);
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const int len = s_len;                       // positions any row needs
  const int nt = (len + kKV - 1) / kKV;        // KV tiles
  auto fail = [&]() { atomicExch(&s_fail, 1); };

  if (warp == 0) {
    // ---- TMA ------------------------------------------------------------------
    if (lane == 0 && nt > 0) {
      bool ok = true;
      mbar_expect_tx(q_full, L::kQBytes);
      for (int kb = 0; kb < L::kKB; ++kb)
        tma_load_2d(smem + L::kQOff + kb * 16384, &qmap, q_full, h * D + kb * 64, int(row0));
      int k_issued = 0, v_issued = 0;
      for (int j = 0; j < nt && ok; ++j) {
        const int s = j & 1;
        if (j >= 2 && !mbar_wait(&k_empty[s], ((j - 2) >> 1) & 1)) {
          ok = false;
          break;
        }
        mbar_expect_tx(&k_full[s], L::kKBytes);
        for (int kb = 0; kb < L::kKB; ++kb)
          tma_load_2d(smem + L::kKOff + s * L::kKBytes + kb * 16384, &kmap, &k_full[s], kb * 64, kv_row0 + j * kKV);
        k_issued = j + 1;
        if (j >= 2 && !mbar_wait(&v_empty[s], ((j - 2) >> 1) & 1)) {
          ok = false;
          break;
        }
        mbar_expect_tx(&v_full[s], L::kVBytes);
        for (int kb = 0; kb < L::kKB; ++kb)
          tma_load_2d(smem + L::kVOff + s * L::kVBytes + kb * 16384, &vmap, &v_full[s], kb * 64, kv_row0 + j * kKV);
        v_issued = j + 1;
      }
      if (!ok) fail();
      // Let the loads in flight land before the CTA can exit.
      mbar_wait(q_full, 0);
      for (int j = max(0, k_issued - 2); j < k_issued; ++j) mbar_wait(&k_full[j & 1], (j >> 1) & 1);
      for (int j = max(0, v_issued - 2); j < v_issued; ++j) mbar_wait(&v_full[j & 1], (j >> 1) & 1);
    }
  } else if (warp == 1) {
    // ---- MMA issuer -------------------------------------------------------------
    if (lane == 0 && nt > 0) {
      constexpr uint32_t kIdS = idesc_bf16(kQ, kKV), kIdO = idesc_bf16(kQ, D);
      const uint32_t tO = tmem + 256;
      bool ok = mbar_wait(q_full, 0);
      // S of tile j into TMEM buffer j % 2, once its K has landed and the
      // softmax has read that buffer's previous tile (j - 2).
      auto issue_s = [&](int j) {
        const int s = j & 1;
        if (!mbar_wait(&k_full[s], (j >> 1) & 1) || (j >= 2 && !mbar_wait(&s_used[s], ((j - 2) >> 1) & 1)))
          return false;
        tc_fence_after();
#pragma unroll
        for (int kb = 0; kb < L::kKB; ++kb) {
          const uint64_t da = sw128_desc(smem + L::kQOff + kb * 16384);
          const uint64_t db = sw128_desc(smem + L::kKOff + s * L::kKBytes + kb * 16384);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + uint32_t(s * 128), da + uint64_t(2 * kk), db + uint64_t(2 * kk), kIdS, (kb | kk) != 0);
        }
        umma_commit(&s_full[s]);
        umma_commit(&k_empty[s]);
        return true;
      };
      auto issue_pv = [&](int j) {
        if (!mbar_wait(p_full, j & 1) || !mbar_wait(vt_full, j & 1)) return false;
        tc_fence_after();
#pragma unroll
        for (int kb = 0; kb < 2; ++kb) {  // 64 positions per block
          const uint64_t da = sw128_desc(smem + L::kPOff + kb * 16384);
          const uint64_t db = sw128_desc(smem + L::kVtOff + kb * (D * 128));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tO, da + uint64_t(2 * kk), db + uint64_t(2 * kk), kIdO, (j | kb | kk) != 0);
        }
        umma_commit(pv_done);
        return true;
      };
      // S runs two tiles ahead of P V, so the scores of the next tile are
      // ready when the softmax finishes the current one.
      if (ok) ok = issue_s(0);
      if (ok && nt > 1) ok = issue_s(1);
      for (int j = 0; j < nt && ok; ++j) {
        ok = issue_pv(j);
        if (ok && j + 2 < nt) ok = issue_s(j + 2);
      }
      if (!ok) fail();
    }
  } else if (warp < 6) {
    // ---- softmax and output: thread = query row --------------------------------
    const int quarter = warp & 3, row = quarter * 32 + lane;
    const uint32_t lane_addr = uint32_t(quarter * 32) << 16;
    const uint32_t tO = tmem + lane_addr + 256;
    const int prow = s_pos[row];
    const float sl = kLog2e / sqrtf(float(D));
    float m_ref = -INFINITY, l = 0.0f;
    const uint32_t pbase = su32(smem + L::kPOff) + uint32_t(row) * 128;
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      if (ok && !mbar_wait(&s_full[j & 1], (j >> 1) & 1)) {
        fail();
        ok = false;
      }
      tc_fence_after();
      const uint32_t tS = tmem + lane_addr + uint32_t((j & 1) * 128);
      const int p0 = j * kKV;
      // The whole S row (128 columns) in two loads and one wait.
      uint32_t r[kKV];
      tmem_ld64_nowait(tS, r);
      tmem_ld64_nowait(tS + 64, r + 64);
      tmem_ld_wait();
      // The row maximum over this tile's valid positions (in base 2).
      const int nv = min(kKV, prow - p0 + 1);  // valid positions of this row in the tile (<= 0: none)
      float mt = -INFINITY;
#pragma unroll
      for (int e = 0; e < kKV; ++e) {
        const float x = __uint_as_float(r[e]) * sl;
        r[e] = __float_as_uint(x);
        if (e < nv) mt = fmaxf(mt, x);
      }
      bool rescale = false;
      float corr = 1.0f;
      if (mt > m_ref + kRescale) {  // also the first valid tile (m_ref = -inf)
        if (m_ref != -INFINITY) {
          corr = ex2(m_ref - mt);
          rescale = true;
        }
        l *= corr;
        m_ref = mt;
      }
      // P = 2^(s - m_ref) as bf16 pairs; masked positions are 0.
      uint32_t pk[kKV / 2];
      float ps = 0.0f;
#pragma unroll
      for (int e = 0; e < kKV; e += 2) {
        const float x0 = e < nv ? ex2(__uint_as_float(r[e]) - m_ref) : 0.0f;
        const float x1 = e + 1 < nv ? ex2(__uint_as_float(r[e + 1]) - m_ref) : 0.0f;
        ps += x0 + x1;
        pk[e / 2] = pack_bf2(x0, x1);
      }
      l += ps;
      // S has been read: the MMA may compute the next tile's scores.
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&s_used[j & 1]);
      // The previous tile's P V must be done before P and O are touched.
      if (j >= 1 && ok && !mbar_wait(pv_done, (j - 1) & 1)) {
        fail();
        ok = false;
      }
      tc_fence_after();
      if (j >= 1 && __any_sync(0xffffffffu, rescale)) {
#pragma unroll
        for (int c = 0; c < D / 32; ++c) {
          uint32_t o32[32];
          tmem_ld32(tO + uint32_t(c * 32), o32);
#pragma unroll
          for (int e = 0; e < 32; ++e) o32[e] = __float_as_uint(__uint_as_float(o32[e]) * corr);
          tmem_st32(tO + uint32_t(c * 32), o32);
        }
      }
      // P row into the two 64-position blocks (16-byte pieces swizzled by row & 7).
#pragma unroll
      for (int kb = 0; kb < 2; ++kb)
#pragma unroll
        for (int c8 = 0; c8 < 8; ++c8) {
          const int w0 = kb * 32 + c8 * 4;
          sts128(pbase + uint32_t(kb * 16384) + (uint32_t(c8 ^ (row & 7)) << 4), pk[w0], pk[w0 + 1], pk[w0 + 2],
                 pk[w0 + 3]);
        }
      fence_proxy_async();
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(p_full);
    }
    // ---- output: O / l ---------------------------------------------------------
    if (nt > 0 && ok && !mbar_wait(pv_done, (nt - 1) & 1)) {
      fail();
      ok = false;
    }
    tc_fence_after();
    const float inv = l > 0.0f ? 1.0f / l : 0.0f;
    uint16_t* orow = a.out + (row0 + row) * int64_t(a.heads) * D + int64_t(h) * D;
#pragma unroll
    for (int c = 0; c < D / 32; ++c) {
      uint32_t r[32];
      if (nt > 0) {
        tmem_ld32(tO + uint32_t(c * 32), r);
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) r[e] = 0u;
      }
      if (row < n_rows && ok) {
#pragma unroll
        for (int v = 0; v < 4; ++v) {
          uint32_t w[4];
#pragma unroll
          for (int e = 0; e < 4; ++e)
            w[e] = pack_bf2(__uint_as_float(r[8 * v + 2 * e]) * inv, __uint_as_float(r[8 * v + 2 * e + 1]) * inv);
          *reinterpret_cast<uint4*>(orow + c * 32 + 8 * v) = make_uint4(w[0], w[1], w[2], w[3]);
        }
      }
    }
  } else {
    // ---- V transpose: [position][d] -> [d][position], 8x8 blocks --------------
    const int tw = warp - 6;
    const int i = lane >> 3, jr = lane & 7;
    const uint32_t vdst = su32(smem + L::kVtOff);
    constexpr int kQuads = (D / 8) * 4;  // (d block, group of four position blocks)
    bool ok = true;
    for (int j = 0; j < nt; ++j) {
      if (ok && (!mbar_wait(&v_full[j & 1], (j >> 1) & 1) || (j >= 1 && !mbar_wait(pv_done, (j - 1) & 1)))) {
        fail();
        ok = false;
      }
      const uint32_t vsrc = su32(smem + L::kVOff + (j & 1) * L::kVBytes);
      const int p0 = j * kKV;
      for (int qi = tw; qi < kQuads; qi += 4) {
        const int db = qi >> 2, kq = qi & 3;
        const int kbk = 4 * kq + i;          // this lane's 8-position block
        const int r = 8 * kbk + jr;          // source row (position within the tile)
        const uint32_t src = vsrc + uint32_t((db >> 3) * 16384 + r * 128) + (uint32_t((db & 7) ^ (r & 7)) << 4);
        const int d = 8 * db + jr;           // destination row
        const uint32_t dst =
            vdst + uint32_t((kbk >> 3) * (D * 128) + d * 128) + (uint32_t((kbk & 7) ^ (d & 7)) << 4);
        uint32_t v[4];
        ldsm_x4_trans(v, src);
        // Thread (g, q) holds positions 8 (4 kq + b) + 2q and + 1 of block b.
        const int qq = lane & 3;
#pragma unroll
        for (int b = 0; b < 4; ++b) {
          const int pp = p0 + 8 * (4 * kq + b) + 2 * qq;
          if (pp >= len) v[b] &= 0u;
          else if (pp + 1 >= len) v[b] &= 0x0000FFFFu;
        }
        stsm_x4(dst, v);
      }
      fence_proxy_async();
      __syncwarp();
      if (lane == 0) {
        mbar_arrive(vt_full);
        mbar_arrive(&v_empty[j & 1]);
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemColsPf) : "memory");
  }
  if (threadIdx.x == 0 && s_fail && a.err) atomicExch(a.err, 4);
}

using EncodeTiled = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                 const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                 CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiled encode_fn() {
  static EncodeTiled fn = [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return EncodeTiled(nullptr);
    return reinterpret_cast<EncodeTiled>(p);
  }();
  return fn;
}

// bf16 [rows, cols] row-major as 64 x 128 tiles, 128-byte swizzled.
bool make_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols) {
  EncodeTiled enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {cols * 2};
  const cuuint32_t box[2] = {64, 128};
  const cuuint32_t estr[2] = {1, 1};
  return enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
             CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
             CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int D>
int launch_pf(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int32_t* pos, int64_t batch,
              int64_t tps, int64_t heads, int64_t kv_heads, int64_t max_len, uint16_t* out, int* err,
              cudaStream_t st) {
  using L = PfLay<D>;
  static PerDeviceOnce configured;
  if (!configured.run([] {
        return cudaFuncSetAttribute(attn_prefill_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    L::kBytes) == cudaSuccess;
      }))
    return SB_INTERNAL;
  CUtensorMap qm, km, vm;
  const uint64_t kv_rows = uint64_t(batch) * uint64_t(kv_heads) * uint64_t(max_len);
  if (!make_map(&qm, q, uint64_t(batch * tps), uint64_t(heads * D)) || !make_map(&km, kc, kv_rows, D) ||
      !make_map(&vm, vc, kv_rows, D))
    return SB_INTERNAL;
  PfArgs args{int(tps), int(heads), int(kv_heads), int(max_len), int((tps + kQ - 1) / kQ), pos, out, err};
  const dim3 grid{unsigned(args.qtiles), unsigned(heads), unsigned(batch)};
  if (launch_pdl(attn_prefill_tc_kernel<D>, grid, dim3(kPfThreads), size_t(L::kBytes), st, qm, km, vm, args) !=
      cudaSuccess)
    return SB_INTERNAL;
  count_launch();
  return SB_OK;
}

}  // namespace

bool attention_prefill_supported(int64_t rows, int64_t tokens_per_seq, int64_t heads, int64_t kv_heads,
                                 int64_t head_dim) {
  return tokens_per_seq >= 16 && rows % tokens_per_seq == 0 && attention_tc_supported(heads, kv_heads, head_dim) &&
         heads <= 65535 && rows / tokens_per_seq <= 65535 && encode_fn() != nullptr;
}

int launch_attention_prefill(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* pos,
                             int64_t rows, int64_t tokens_per_seq, int64_t heads, int64_t kv_heads, int64_t head_dim,
                             int64_t max_len, uint16_t* out, int* err, cudaStream_t st) {
  if (!attention_prefill_supported(rows, tokens_per_seq, heads, kv_heads, head_dim)) return SB_INVALID_ARGUMENT;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!a16(q) || !a16(k_cache) || !a16(v_cache)) return SB_INVALID_ARGUMENT;
  const int64_t batch = rows / tokens_per_seq;
  if (batch * kv_heads * max_len > int64_t(INT32_MAX)) return SB_INVALID_ARGUMENT;
  if (head_dim == 128)
    return launch_pf<128>(q, k_cache, v_cache, pos, batch, tokens_per_seq, heads, kv_heads, max_len, out, err, st);
  return launch_pf<64>(q, k_cache, v_cache, pos, batch, tokens_per_seq, heads, kv_heads, max_len, out, err, st);
}

}  // namespace sb
