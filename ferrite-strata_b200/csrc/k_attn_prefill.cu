// Prefill attention on the 5th-generation tensor cores (tcgen05, TMEM, TMA):
// bf16, head_dim 64 or 128, MHA and GQA.
//
// Same semantics as the decode kernels: query row r of sequence r / S
// (S = tokens per sequence) attends to cache positions 0..pos[r] of that
// sequence, after the step's KV append has written every row's k and v.
// With pos = 0..S-1 this is causal self-attention over the prompt.
//
// One CTA per (pair of 128-row query tiles, query head, sequence), heaviest
// pairs first; the two query tiles share every 128-position K/V tile, which
// is loaded once by TMA (double-buffered).  Per query tile t and KV tile j,
// FlashAttention-style, with both products on tcgen05.mma (kind::f16,
// M = 128, f32 accumulators in TMEM):
//   S_t = Q_t K^T    A = Q_t (shared memory, loaded once), B = the K tile;
//                    S_t in TMEM columns [128 t, 128 t + 128);
//   softmax          one thread per query row reads its S row from TMEM,
//                    masks positions past pos[r], and keeps a running row
//                    maximum in base 2.  O_t is rescaled in TMEM only when a
//                    row's maximum grows by more than 8 (a factor of 256), so
//                    the probabilities stay below 2^8; the row sum uses the
//                    same reference maximum, so the final O / l is exact.
//                    P goes back into the first 64 columns of S_t as bf16
//                    pairs;
//   O_t += P_t V     A = P_t from TMEM, B = the V tile exactly as loaded
//                    ([position][d] rows, read as an MN-major operand);
// and at the end O_t / l as bf16.
//
// The MMAs of one thread run in issue order, and each S_t is issued after
// the previous P_t V, so the commit that publishes S_t also says that O_t is
// settled and P_t's columns are free: the softmax never waits for the P V.
// While one softmax warpgroup works on its S, the tensor cores compute the
// other query tile's products.
//
// Positions at or past the last one any row needs hold whatever the cache
// holds there; P is zero for them, and the MMA warp zeroes the V rows of the
// last tile's 16-position group that contains the end (so 0 * NaN never
// reaches O) and stops the last P V at that group.
//
// Warps: 0 TMA, 1 TMEM allocation and the MMA issuer, 2-5 softmax and output
// for query tile 0, 6-9 for query tile 1 (TMEM lane quarter = warp % 4).
// Every mbarrier wait is bounded; one that runs out records error word 4 and
// the CTA winds down (the TMA thread lets its loads land, the MMA warp waits
// for its MMAs to finish, the TMEM owner frees its columns).  Every TMA load
// lands in the issuing CTA's own shared memory only.
#include "common.cuh"
#include "k_elem.cuh"
#include "k_tc.cuh"

namespace sb {

namespace {

using namespace tc;

constexpr int kQ = 128;    // query rows per tile (TMEM lanes); two tiles per CTA
constexpr int kKV = 128;   // positions per KV tile
constexpr int kPfThreads = 320;
constexpr uint32_t kTmemColsPf = 512;  // S_0, S_1 (128 columns each), O_0, O_1 (head_dim each)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescale = 8.0f;  // log2 of the largest P before O is rescaled

template <int D>
struct PfLay {
  static constexpr int kKB = D / 64;                 // 64-wide blocks of head_dim
  static constexpr int kTile = 128 * D * 2;          // a Q, K or V tile: kKB blocks of [128 rows][128 B]
  static constexpr int kQOff = 0;                    // two query tiles
  static constexpr int kKOff = kQOff + 2 * kTile;    // two K stages
  static constexpr int kVOff = kKOff + 2 * kTile;    // two V stages
  static constexpr int kBarOff = kVOff + 2 * kTile;  // mbarriers
  static constexpr int kBars = 17;
  static constexpr int kBytes = kBarOff + kBars * 8 + 16 + 1024;
  static constexpr uint32_t kOCol = 256;             // O_t at column 256 + t * D
};

struct PfArgs {
  int tps, heads, kv_heads, max_len, pairs, batch, items;
  const int32_t* pos;
  uint16_t* out;
  int* err;
  KvPages kp;     // paged caches: K/V tiles are loaded a page (or a 128-row part of one) at a time
  int pool_rows;  // rows of the K/V tensor maps
};

// One work item: a pair of query tiles of one head of one sequence.  Items
// are numbered heaviest first (latest query rows need the most KV tiles),
// heads fastest so that neighbouring items share a kv head's cache in L2.
struct PfItem {
  int t0, n_rows, h, seq, kvh;
  int64_t row0;
  int kv_row0;  // contiguous caches: the map row of position 0 of (seq, kvh)
};

__device__ __forceinline__ PfItem pf_item(const PfArgs& a, int w) {
  const int per = a.heads * a.batch;
  const int pair = a.pairs - 1 - w / per, rem = w % per;
  const int h = rem % a.heads, seq = rem / a.heads;
  PfItem it;
  it.t0 = pair * 2 * kQ;
  it.n_rows = min(2 * kQ, a.tps - it.t0);
  it.h = h;
  it.seq = seq;
  it.kvh = h / (a.heads / a.kv_heads);
  it.row0 = int64_t(seq) * a.tps + it.t0;
  it.kv_row0 = a.kp.paged() ? 0 : (seq * a.kv_heads + it.kvh) * a.max_len;
  return it;
}

// The k-th item of this CTA.  Items are numbered heaviest first and dealt to
// the CTAs in rounds of gridDim.x, in alternating direction (a "snake"), so
// every CTA's total work is within about one light item of the mean.
__device__ __forceinline__ int pf_work(int k) {
  return k * int(gridDim.x) + ((k & 1) ? int(gridDim.x) - 1 - int(blockIdx.x) : int(blockIdx.x));
}

// This lane's share of an item's positions: rows 32 i + lane of the 256
// (tile i / 4), -1 for rows past the item's end or outside [0, max_len).
// Loaded one item ahead, so the loads are in flight while the current item
// runs.
struct PfPos {
  int p[8];
};

__device__ __forceinline__ PfPos pf_pos_load(const PfArgs& a, int w, int lane) {
  PfPos q;
  const bool live = w < a.items;
  const PfItem it = pf_item(a, live ? w : 0);
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = i * 32 + lane;
    q.p[i] = live && r < it.n_rows ? a.pos[it.row0 + r] : -1;
  }
  return q;
}

// Positions query tile t needs: 1 + its largest valid position (0: none).
// Every lane of the warp gets the same answer.
__device__ __forceinline__ int pf_tile_len(const PfArgs& a, const PfPos& q, int t) {
  int m = 0;
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int p = q.p[4 * t + i];
    if (p >= 0 && p < a.max_len) m = max(m, p + 1);
  }
  return __reduce_max_sync(0xffffffffu, m);
}

// 2^x by the hardware approximation (relative error about 2^-22).
__device__ __forceinline__ float ex2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float m;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(m) : "f"(a), "f"(b), "f"(c));
  return m;
}

// Packed pairs of f32 (sm_100 f32x2 arithmetic).
__device__ __forceinline__ uint64_t pack_f2(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ void unpack_f2(uint64_t v, float& lo, float& hi) {
  asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v));
}
__device__ __forceinline__ uint64_t fma_f2(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.ftz.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
__device__ __forceinline__ uint64_t add_f2(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.ftz.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

__device__ __forceinline__ void sts128_zero(uint32_t addr) {
  asm volatile("st.shared.v4.u32 [%0], {%1,%1,%1,%1};" ::"r"(addr), "r"(0u) : "memory");
}

template <int D>
__global__ void __launch_bounds__(kPfThreads, 1)
    attn_prefill_tc_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                           const __grid_constant__ CUtensorMap vmap, const PfArgs a) {
  using L = PfLay<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + L::kBarOff);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;    // [2] per stage
  uint64_t* k_empty = bars + 3;   // [2]
  uint64_t* v_full = bars + 5;    // [2]
  uint64_t* v_empty = bars + 7;   // [2]
  uint64_t* s_full = bars + 9;    // [2] per query tile: S_t of the next KV tile is in TMEM
  uint64_t* p_full = bars + 11;   // [2] per query tile: P_t is in TMEM (4 warps arrive)
  uint64_t* o_done = bars + 13;   // [2] per query tile: the item's last P_t V has completed
  uint64_t* mma_done = bars + 15; // every MMA of the CTA has completed
  uint64_t* q_empty = bars + 16;  // the item's MMAs (all readers of Q) have completed
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + L::kBars);
  __shared__ int s_fail;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    mbar_init(q_empty, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&k_full[s], 1);
      mbar_init(&k_empty[s], 1);
      mbar_init(&v_full[s], 1);
      mbar_init(&v_empty[s], 1);
      mbar_init(&s_full[s], 1);
      mbar_init(&p_full[s], 4);
      mbar_init(&o_done[s], 1);
    }
    mbar_init(mma_done, 1);
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
  pdl_wait();  // q, pos and the appended cache rows come from the previous kernels
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  auto fail = [&]() { atomicExch(&s_fail, 1); };
  auto failed = [&]() { return *reinterpret_cast<volatile int*>(&s_fail) != 0; };

  // Every role walks the same items (pf_work(0), pf_work(1), ...) and counts
  // KV tiles, S/P tiles and items cumulatively, so each mbarrier phase is
  // known without any CTA-wide synchronisation between items.
  if (warp == 0) {
    // ---- TMA: Q of each item once it is free, then its K/V tiles ---------------
    // nk, nv: K and V tiles loaded so far (tile g uses stage g % 2); nq: items.
    int nk = 0, nv = 0, nq = 0;
    bool ok = true;
    PfPos nxt = pf_pos_load(a, pf_work(0), lane);
    for (int k = 0, w = pf_work(0); w < a.items && ok; w = pf_work(++k)) {
      if (__any_sync(0xffffffffu, failed())) break;
      const PfPos cur = nxt;
      nxt = pf_pos_load(a, pf_work(k + 1), lane);
      const PfItem it = pf_item(a, w);
      const int len = max(pf_tile_len(a, cur, 0), pf_tile_len(a, cur, 1));
      const int nt = (len + kKV - 1) / kKV;
      if (nt == 0) continue;
      // KV tile j of the item (positions [128 j, 128 j + 128)) into dst.  A
      // paged cache is read a page at a time (boxes of min(page_size, 128)
      // rows, each landing at its row offset: the 128-byte swizzle is a
      // function of the shared-memory address, which is 2048-byte aligned
      // for every box).  A page that is missing from the table or not in the
      // pool is read past the end of the map, which yields zeros; if the
      // item needs any of its positions, error word 6 is set.
      auto kv_tile = [&](const CUtensorMap* map, uint8_t* dst, uint64_t* bar, int j) {
        if (!a.kp.paged()) {
          for (int kb = 0; kb < L::kKB; ++kb)
            tma_load_2d(dst + kb * 16384, map, bar, kb * 64, it.kv_row0 + j * kKV);
          return;
        }
        const int br = min(a.kp.page_size, kKV);
        for (int r = 0; r < kKV; r += br) {
          const int p = j * kKV + r;
          const int64_t row = p < a.max_len ? kv_row(a.kp, it.seq, it.kvh, a.kv_heads, a.max_len, p) : -1;
          if (row < 0 && p < len && a.err) atomicExch(a.err, 6);
          const int y = row < 0 ? a.pool_rows : int(row);
          for (int kb = 0; kb < L::kKB; ++kb) tma_load_2d(dst + kb * 16384 + r * 128, map, bar, kb * 64, y);
        }
      };
      if (lane == 0) {
        if (nq >= 1 && !mbar_wait(q_empty, (nq - 1) & 1)) ok = false;
        if (ok) {
          mbar_expect_tx(q_full, 2 * L::kTile);
          for (int t = 0; t < 2; ++t)
            for (int kb = 0; kb < L::kKB; ++kb)
              tma_load_2d(smem + L::kQOff + t * L::kTile + kb * 16384, &qmap, q_full, it.h * D + kb * 64,
                          int(it.row0) + t * kQ);
          ++nq;
        }
        for (int j = 0; j < nt && ok; ++j) {
          const int g = nk, s = g & 1;
          if (g >= 2 && !mbar_wait(&k_empty[s], ((g - 2) >> 1) & 1)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&k_full[s], L::kTile);
          kv_tile(&kmap, smem + L::kKOff + s * L::kTile, &k_full[s], j);
          ++nk;
          if (g >= 2 && !mbar_wait(&v_empty[s], ((g - 2) >> 1) & 1)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&v_full[s], L::kTile);
          kv_tile(&vmap, smem + L::kVOff + s * L::kTile, &v_full[s], j);
          ++nv;
        }
      }
      ok = __shfl_sync(0xffffffffu, ok, 0);
    }
    if (!ok) fail();
    // Let the loads in flight land before the CTA can exit: the last Q, and
    // the last K and V tile of each stage (an earlier load into a stage was
    // waited for by the MMA warp before the stage was refilled).
    if (lane == 0) {
      if (nq > 0) mbar_wait(q_full, (nq - 1) & 1);
      for (int g = max(0, nk - 2); g < nk; ++g) mbar_wait(&k_full[g & 1], (g >> 1) & 1);
      for (int g = max(0, nv - 2); g < nv; ++g) mbar_wait(&v_full[g & 1], (g >> 1) & 1);
    }
  } else if (warp == 1) {
    // ---- MMA issuer (lane 0 issues; the warp waits and zeroes V) ----------------
    constexpr uint32_t kIdS = idesc_bf16(kQ, kKV), kIdO = idesc_bf16(kQ, D, true);
    int nk = 0, nq = 0;      // KV tiles and items consumed so far
    int ns[2] = {0, 0};      // S/P tiles of each query tile so far
    bool ok = true;
    // S_t of the KV tile in stage ks into TMEM columns [128 t, 128 t + 128).
    auto issue_s = [&](int t, int ks) {
      tc_fence_after();
      if (lane == 0) {
        const uint8_t* qs = smem + L::kQOff + t * L::kTile;
        const uint8_t* kst = smem + L::kKOff + ks * L::kTile;
#pragma unroll
        for (int kb = 0; kb < L::kKB; ++kb) {
          const uint64_t da = sw128_desc(qs + kb * 16384), db = sw128_desc(kst + kb * 16384);
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + uint32_t(t * 128), da + uint64_t(2 * kk), db + uint64_t(2 * kk), kIdS, (kb | kk) != 0);
        }
        umma_commit(&s_full[t]);
      }
      __syncwarp();
    };
    // Q may be replaced once the item's last S has been computed.
    auto release_q = [&]() {
      if (lane == 0) umma_commit(q_empty);
      __syncwarp();
    };
    PfPos nxt = pf_pos_load(a, pf_work(0), lane);
    for (int k = 0, w = pf_work(0); w < a.items && ok; w = pf_work(++k)) {
      if (__any_sync(0xffffffffu, failed())) break;
      const PfPos cur = nxt;
      nxt = pf_pos_load(a, pf_work(k + 1), lane);
      const int len0 = pf_tile_len(a, cur, 0), len1 = pf_tile_len(a, cur, 1);
      const int len = max(len0, len1);
      const int ntt[2] = {(len0 + kKV - 1) / kKV, (len1 + kKV - 1) / kKV};
      const int nt = max(ntt[0], ntt[1]);
      if (nt == 0) continue;
      if (!(ok = mbar_wait_warp(q_full, nq & 1) && mbar_wait_warp(&k_full[nk & 1], (nk >> 1) & 1))) break;
      for (int t = 0; t < 2; ++t)
        if (ntt[t] > 0) issue_s(t, nk & 1);
      if (lane == 0) umma_commit(&k_empty[nk & 1]);
      __syncwarp();
      if (nt == 1) release_q();
      for (int j = 0; j < nt && ok; ++j) {
        const int g = nk + j, s = g & 1;
        uint8_t* vs = smem + L::kVOff + s * L::kTile;
        if (!(ok = mbar_wait_warp(&v_full[s], (g >> 1) & 1))) break;
        int ksl = kKV / 16;  // 16-position K steps of the P V product
        if (j == nt - 1) {
          const int nv = len - j * kKV, nv16 = (nv + 15) & ~15, nz = nv16 - nv;
          for (int i = lane; i < nz * L::kKB * 8; i += 32) {
            const int piece = i & 7, rr = (i >> 3) % nz, kb = (i >> 3) / nz;
            sts128_zero(su32(vs + kb * 16384 + (nv + rr) * 128 + piece * 16));
          }
          fence_proxy_async();
          __syncwarp();
          ksl = nv16 / 16;
        }
        if (j + 1 < nt && !(ok = mbar_wait_warp(&k_full[(g + 1) & 1], ((g + 1) >> 1) & 1))) break;
        for (int t = 0; t < 2 && ok; ++t) {
          if (j >= ntt[t]) continue;
          if (!(ok = mbar_wait_warp(&p_full[t], ns[t] & 1))) break;
          ++ns[t];
          tc_fence_after();
          if (lane == 0) {
            const uint32_t tP = tmem + uint32_t(t * 128), tO = tmem + L::kOCol + uint32_t(t * D);
            const uint64_t vd = sw128_desc_mn(vs, 16384);
            for (int kk = 0; kk < ksl; ++kk)
              umma_bf16_ts(tO, tP + uint32_t(kk * 8), vd + uint64_t(kk * (2048 >> 4)), kIdO, (j | kk) != 0);
            if (j + 1 >= ntt[t]) umma_commit(&o_done[t]);
          }
          __syncwarp();
          if (j + 1 < ntt[t]) issue_s(t, (g + 1) & 1);
        }
        if (!ok) break;
        if (lane == 0) {
          umma_commit(&v_empty[s]);
          if (j + 1 < nt) umma_commit(&k_empty[(g + 1) & 1]);
        }
        __syncwarp();
        if (j == nt - 2) release_q();
      }
      if (!ok) break;
      nk += nt;
      ++nq;
    }
    if (!ok) fail();
    if (lane == 0) umma_commit(mma_done);
    __syncwarp();
    mbar_wait_warp(mma_done, 0);
  } else {
    // ---- softmax and output: thread = query row of tile t ------------------------
    const int t = (warp - 2) >> 2;
    const int quarter = warp & 3, row = quarter * 32 + lane;
    const uint32_t lane_addr = uint32_t(quarter * 32) << 16;
    const uint32_t tS = tmem + lane_addr + uint32_t(t * 128);
    const uint32_t tO = tmem + lane_addr + L::kOCol + uint32_t(t * D);
    const int qrow = t * kQ + row;
    const float sl = kLog2e / sqrtf(float(D));
    int nsp = 0, no = 0;  // S/P tiles and items with a P V of this query tile so far
    // This lane's positions of tile t, rows 32 i + lane (its own row is
    // i = quarter), -1 past the item's end; loaded one item ahead.
    int pp[4];
    auto load_pos = [&](int w) {
      const bool live = w < a.items;
      const PfItem it = pf_item(a, live ? w : 0);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int r = t * kQ + i * 32 + lane;
        pp[i] = live && r < it.n_rows ? a.pos[it.row0 + r] : -1;
      }
    };
    load_pos(pf_work(0));
    for (int k = 0, w = pf_work(0); w < a.items; w = pf_work(++k)) {
      if (__any_sync(0xffffffffu, failed())) break;
      const PfItem it = pf_item(a, w);
      int m = 0;
#pragma unroll
      for (int i = 0; i < 4; ++i)
        if (pp[i] >= 0 && pp[i] < a.max_len) m = max(m, pp[i] + 1);
      const int my_nt = (__reduce_max_sync(0xffffffffu, m) + kKV - 1) / kKV;
      const int own = quarter == 0 ? pp[0] : quarter == 1 ? pp[1] : quarter == 2 ? pp[2] : pp[3];
      const bool valid = own >= 0 && own < a.max_len;
      const int prow = valid ? own : -1;
      if (qrow < it.n_rows && !valid && a.err) atomicExch(a.err, 2);
      float m_ref = -INFINITY, l = 0.0f;
      bool ok = true;
      // The loop stays converged: a lane whose wait ran out stops waiting and
      // records the failure; no output is written then.
      for (int j = 0; j < my_nt; ++j) {
        if (ok && !mbar_wait(&s_full[t], nsp & 1)) ok = false;
        ++nsp;
        __syncwarp();  // the poll may have split the warp; tcgen05.ld needs it whole
        tc_fence_after();
        const int p0 = j * kKV;
        // The whole S row (128 columns).
        uint32_t r[kKV];
        tmem_ld64(tS, r);
        tmem_ld64(tS + 64, r + 64);
        // Positions past pos[r] become -inf (whatever the cache holds there), on
        // the diagonal tiles only: the others have no masked position in the warp.
        const int nv = min(kKV, prow - p0 + 1);  // valid positions of this row in the tile (<= 0: none)
        const bool full = __all_sync(0xffffffffu, nv >= kKV);
        if (!full) {
#pragma unroll
          for (int e = 0; e < kKV; ++e)
            if (e >= nv) r[e] = 0xFF800000u;
        }
        // Row maximum of the raw scores, four independent 3-input chains; the
        // scale is positive, so it is applied once to the maximum (base 2).
        float mc[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
#pragma unroll
        for (int e = 0; e < kKV; e += 8)
#pragma unroll
          for (int c = 0; c < 4; ++c) mc[c] = fmax3(mc[c], __uint_as_float(r[e + 2 * c]), __uint_as_float(r[e + 2 * c + 1]));
        const float mt = fmaxf(fmaxf(mc[0], mc[1]), fmaxf(mc[2], mc[3])) * sl;
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
        // P = 2^(s sl - m_ref) as bf16 pairs, packed in place; -inf gives 0.  A
        // row with no valid position yet has every score at -inf and uses 0 for
        // the maximum, so no inf - inf appears.
        const float mneg = m_ref == -INFINITY ? 0.0f : -m_ref;
        const uint64_t sl2 = pack_f2(sl, sl), mneg2 = pack_f2(mneg, mneg);
        uint64_t acc[4] = {0, 0, 0, 0};
#pragma unroll
        for (int e = 0; e < kKV; e += 2) {
          float x0, x1;
          unpack_f2(fma_f2(pack_f2(__uint_as_float(r[e]), __uint_as_float(r[e + 1])), sl2, mneg2), x0, x1);
          x0 = ex2(x0);
          x1 = ex2(x1);
          acc[(e >> 1) & 3] = add_f2(acc[(e >> 1) & 3], pack_f2(x0, x1));
          // bf16 by integer rounding (to nearest, ties away from zero): the
          // probabilities are finite and non-negative, and this keeps the
          // conversion off the pipe that computes the exponentials.
          r[e / 2] = __byte_perm(__float_as_uint(x0) + 0x8000u, __float_as_uint(x1) + 0x8000u, 0x7632);
        }
        float a0, a1, a2, a3;
        unpack_f2(add_f2(acc[0], acc[1]), a0, a1);
        unpack_f2(add_f2(acc[2], acc[3]), a2, a3);
        l += (a0 + a1) + (a2 + a3);
        // O_t is settled (its last P V completed before this S was published).
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll
          for (int c = 0; c < D / 32; ++c) {
            uint32_t o32[32];
            tmem_ld32(tO + uint32_t(c * 32), o32);
#pragma unroll
            for (int e = 0; e < 32; ++e) o32[e] = __float_as_uint(__uint_as_float(o32[e]) * corr);
            tmem_st32(tO + uint32_t(c * 32), o32);
          }
        }
        tmem_st64(tS, r);
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive(&p_full[t]);
      }
      // ---- output: O / l ---------------------------------------------------------
      if (my_nt > 0) {
        if (ok && !mbar_wait(&o_done[t], no & 1)) ok = false;
        ++no;
      }
      if (!__all_sync(0xffffffffu, ok)) {
        fail();
        break;
      }
      tc_fence_after();
      load_pos(pf_work(k + 1));  // in flight while O is written out
      const float inv = l > 0.0f ? 1.0f / l : 0.0f;
      uint16_t* orow = a.out + (it.row0 + qrow) * int64_t(a.heads) * D + int64_t(it.h) * D;
#pragma unroll
      for (int c = 0; c < D / 32; ++c) {
        uint32_t r[32];
        if (my_nt > 0) {
          tmem_ld32(tO + uint32_t(c * 32), r);
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) r[e] = 0u;
        }
        if (qrow < it.n_rows) {
#pragma unroll
          for (int v = 0; v < 4; ++v) {
            uint32_t w4[4];
#pragma unroll
            for (int e = 0; e < 4; ++e)
              w4[e] = pack_bf2(__uint_as_float(r[8 * v + 2 * e]) * inv, __uint_as_float(r[8 * v + 2 * e + 1]) * inv);
            *reinterpret_cast<uint4*>(orow + c * 32 + 8 * v) = make_uint4(w4[0], w4[1], w4[2], w4[3]);
          }
        }
      }
      // O_t has been read: the next item's first P V may overwrite it (the
      // p_full arrival that lets it start is ordered after this fence).
      tc_fence_before();
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


// bf16 [rows, cols] row-major as 64-column x box_rows tiles, 128-byte swizzled.
bool make_map(CUtensorMap* map, const void* base, uint64_t rows, uint64_t cols, uint32_t box_rows = 128) {
  return make_map_2d(map, base, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, rows, cols, 64, box_rows,
                     CU_TENSOR_MAP_SWIZZLE_128B);
}

template <int D>
int launch_pf(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int32_t* pos, int64_t batch,
              int64_t tps, int64_t heads, int64_t kv_heads, int64_t max_len, uint16_t* out, int* err,
              cudaStream_t st, const KvPages& kp) {
  using L = PfLay<D>;
  static PerDeviceOnce configured;
  if (!configured.run([] {
        return cudaFuncSetAttribute(attn_prefill_tc_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    L::kBytes) == cudaSuccess;
      }))
    return SB_INTERNAL;
  CUtensorMap qm, km, vm;
  const uint64_t kv_rows = kp.paged() ? uint64_t(kp.num_pages) * uint64_t(kv_heads) * uint64_t(kp.page_size)
                                      : uint64_t(batch) * uint64_t(kv_heads) * uint64_t(max_len);
  const uint32_t box = kp.paged() ? uint32_t(std::min(kp.page_size, kKV)) : 128u;
  if (!make_map(&qm, q, uint64_t(batch * tps), uint64_t(heads * D)) || !make_map(&km, kc, kv_rows, D, box) ||
      !make_map(&vm, vc, kv_rows, D, box))
    return SB_INTERNAL;
  const int pairs = int((tps + 2 * kQ - 1) / (2 * kQ));
  const int64_t items = int64_t(pairs) * heads * batch;
  if (items > int64_t(INT32_MAX)) return SB_INVALID_ARGUMENT;
  PfArgs args{int(tps), int(heads), int(kv_heads), int(max_len), pairs, int(batch), int(items), pos, out, err,
              kp, int(kv_rows)};
  const dim3 grid{unsigned(std::min<int64_t>(items, kNumSMs))};
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
         heads <= 65535 && rows / tokens_per_seq <= 65535 && encode_tiled_fn() != nullptr;
}

int launch_attention_prefill(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache, const int32_t* pos,
                             int64_t rows, int64_t tokens_per_seq, int64_t heads, int64_t kv_heads, int64_t head_dim,
                             int64_t max_len, uint16_t* out, int* err, cudaStream_t st, const KvPages& kp) {
  if (!attention_prefill_supported(rows, tokens_per_seq, heads, kv_heads, head_dim)) return SB_INVALID_ARGUMENT;
  if (kp.paged() && (!kv_page_size_ok(kp.page_size) || int64_t(kp.page_size) * kp.pages_per_seq != max_len ||
                     kp.num_pages <= 0 || int64_t(kp.num_pages) * kv_heads * kp.page_size >= int64_t(INT32_MAX)))
    return SB_INVALID_ARGUMENT;
  auto a16 = [](const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
  if (!a16(q) || !a16(k_cache) || !a16(v_cache)) return SB_INVALID_ARGUMENT;
  const int64_t batch = rows / tokens_per_seq;
  if (batch * kv_heads * max_len > int64_t(INT32_MAX) || rows + 2 * kQ > int64_t(INT32_MAX))
    return SB_INVALID_ARGUMENT;
  if (head_dim == 128)
    return launch_pf<128>(q, k_cache, v_cache, pos, batch, tokens_per_seq, heads, kv_heads, max_len, out, err, st,
                          kp);
  return launch_pf<64>(q, k_cache, v_cache, pos, batch, tokens_per_seq, heads, kv_heads, max_len, out, err, st, kp);
}

}  // namespace sb
