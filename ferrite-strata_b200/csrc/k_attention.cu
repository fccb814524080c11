// Causal / grouped-query attention over a KV cache.
//
// Cache layout in HBM: [batch, kv_heads, max_len, head_dim], so one
// (sequence, kv head) is a contiguous max_len x head_dim slab and a decode
// step streams it front to back.
//
// A query row r belongs to sequence r / tokens_per_seq and sits at position
// pos[r]; it attends to cache positions 0..pos[r] inclusive.  The new k/v rows
// are appended first (kv_append), then attention reads the cache.
//
// attn_kernel: one block per (split, kv head, query row).  The block loads the
// G = heads / kv_heads query heads that share the kv head, then walks its
// slice of positions in tiles of 128: one thread per position computes the G
// scores (k row read once for all G heads), the block keeps an online softmax
// (running max and sum per head), and the PV product reads each v row once,
// coalesced, for all G heads.  With one split the block normalises and writes
// the output; with several it writes (max, sum, unnormalised acc) partials
// and attn_merge_kernel combines them (flash-decoding).
#include <algorithm>
#include <cstdlib>
#include <string>

#include "common.cuh"
#include "k_elem.cuh"

namespace sb {

namespace {

template <typename T>
__device__ __forceinline__ float ld1(const T* p);
template <>
__device__ __forceinline__ float ld1<float>(const float* p) { return *p; }
template <>
__device__ __forceinline__ float ld1<uint16_t>(const uint16_t* p) { return bf2f(*p); }

template <typename T>
__device__ __forceinline__ void st1(T* p, float v);
template <>
__device__ __forceinline__ void st1<float>(float* p, float v) { *p = v; }
template <>
__device__ __forceinline__ void st1<uint16_t>(uint16_t* p, float v) { *p = f2bf(v); }

// Two consecutive elements as f32.
template <typename T>
__device__ __forceinline__ float2 ld2(const T* p);
template <>
__device__ __forceinline__ float2 ld2<float>(const float* p) {
  return *reinterpret_cast<const float2*>(p);
}
template <>
__device__ __forceinline__ float2 ld2<uint16_t>(const uint16_t* p) {
  const uint32_t v = *reinterpret_cast<const uint32_t*>(p);
  return make_float2(bf_lo(v), bf_hi(v));
}

// Eight consecutive elements as f32 (16-byte loads for bf16).
template <typename T>
__device__ __forceinline__ void ld8(const T* p, float (&v)[8]);
template <>
__device__ __forceinline__ void ld8<float>(const float* p, float (&v)[8]) {
  const float4 a = *reinterpret_cast<const float4*>(p);
  const float4 b = *reinterpret_cast<const float4*>(p + 4);
  v[0] = a.x, v[1] = a.y, v[2] = a.z, v[3] = a.w, v[4] = b.x, v[5] = b.y, v[6] = b.z, v[7] = b.w;
}
template <>
__device__ __forceinline__ void ld8<uint16_t>(const uint16_t* p, float (&v)[8]) {
  const uint4 a = *reinterpret_cast<const uint4*>(p);
  v[0] = bf_lo(a.x), v[1] = bf_hi(a.x), v[2] = bf_lo(a.y), v[3] = bf_hi(a.y);
  v[4] = bf_lo(a.z), v[5] = bf_hi(a.z), v[6] = bf_lo(a.w), v[7] = bf_hi(a.w);
}

template <typename T>
__global__ void kv_append_kernel(const T* __restrict__ k_new, const T* __restrict__ v_new,
                                 T* __restrict__ k_cache, T* __restrict__ v_cache,
                                 const int32_t* __restrict__ pos, int rows, int tokens_per_seq,
                                 int kv_heads, int head_dim, int max_len, KvPages kp, int* err) {
  pdl_trigger();
  pdl_wait();
  const int row = blockIdx.x;
  const int p = pos[row];
  const int seq = row / tokens_per_seq;
  // Row of kv head 0; head h is h * page_size (paged) or h * max_len rows on.
  const bool in_range = p >= 0 && p < max_len;
  const int64_t r0 = in_range ? kv_row(kp, seq, 0, kv_heads, max_len, p) : -1;
  if (r0 < 0) {  // error word 2: bad position; 6: its page is missing
    if (threadIdx.x == 0 && err) atomicExch(err, in_range ? 6 : 2);
    return;
  }
  const int64_t hstride = kp.paged() ? kp.page_size : max_len;
  const int width = kv_heads * head_dim;
  constexpr int kVec = 16 / int(sizeof(T));  // elements per 16-byte copy
  const bool vec = head_dim % kVec == 0 &&
                   ((reinterpret_cast<uintptr_t>(k_new) | reinterpret_cast<uintptr_t>(v_new) |
                     reinterpret_cast<uintptr_t>(k_cache) | reinterpret_cast<uintptr_t>(v_cache)) & 15) == 0;
  if (vec) {
    for (int c = threadIdx.x; c < width / kVec; c += blockDim.x) {
      const int i = c * kVec, h = i / head_dim, d = i - h * head_dim;
      const int64_t dst = (r0 + h * hstride) * head_dim + d;
      *reinterpret_cast<uint4*>(k_cache + dst) = *reinterpret_cast<const uint4*>(k_new + int64_t(row) * width + i);
      *reinterpret_cast<uint4*>(v_cache + dst) = *reinterpret_cast<const uint4*>(v_new + int64_t(row) * width + i);
    }
    return;
  }
  for (int i = threadIdx.x; i < width; i += blockDim.x) {
    const int h = i / head_dim, d = i % head_dim;
    const int64_t dst = (r0 + h * hstride) * head_dim + d;
    k_cache[dst] = k_new[int64_t(row) * width + i];
    v_cache[dst] = v_new[int64_t(row) * width + i];
  }
}

constexpr int kThreads = 128;
constexpr int kMaxGroup = 8;

template <typename T, int D>
__global__ void __launch_bounds__(kThreads)
    attn_kernel(const T* __restrict__ q, const T* __restrict__ kc, const T* __restrict__ vc,
                const int32_t* __restrict__ pos, int tokens_per_seq, int heads, int kv_heads,
                int max_len, int splits, float scale, float* __restrict__ partial,
                T* __restrict__ out, int* err) {
  pdl_trigger();
  pdl_wait();
  constexpr int kPairs = D / 2;              // d pairs per row
  constexpr int kPhases = kThreads / kPairs;  // position phases in the PV loop
  const int split = blockIdx.x, kvh = blockIdx.y, row = blockIdx.z;
  const int G = heads / kv_heads;
  const int tid = threadIdx.x;
  pdl_trigger();
  pdl_wait();

  __shared__ float qs[kMaxGroup][D];
  __shared__ float ps[kMaxGroup][kThreads];
  __shared__ float red[kThreads / 32][kMaxGroup];
  __shared__ float accs[kPhases][kMaxGroup][D];

  const int p = pos[row];
  const bool bad = p < 0 || p >= max_len;
  if (bad && tid == 0 && err) atomicExch(err, 2);
  const int len = bad ? 0 : p + 1;
  const int chunk = (len + splits - 1) / splits;
  const int t_begin = min(len, split * chunk);
  const int t_end = min(len, t_begin + chunk);

  for (int i = tid; i < G * D; i += kThreads) {
    const int g = i / D, d = i % D;
    qs[g][d] = ld1(q + int64_t(row) * heads * D + int64_t(kvh * G + g) * D + d);
  }
  __syncthreads();

  const int seq = row / tokens_per_seq;
  const T* kbase = kc + (int64_t(seq) * kv_heads + kvh) * int64_t(max_len) * D;
  const T* vbase = vc + (int64_t(seq) * kv_heads + kvh) * int64_t(max_len) * D;

  float m_run[kMaxGroup], l_run[kMaxGroup];
  float acc[kMaxGroup][2];
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    m_run[g] = -INFINITY;
    l_run[g] = 0.0f;
    acc[g][0] = acc[g][1] = 0.0f;
  }
  const int pair = tid % kPairs, phase = tid / kPairs;

  for (int t0 = t_begin; t0 < t_end; t0 += kThreads) {
    const int t = t0 + tid;
    const bool live = t < t_end;
    // Scores: one position per thread, all G heads from one k row.
    float sc[kMaxGroup];
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) sc[g] = 0.0f;
    if (live) {
      const T* kr = kbase + int64_t(t) * D;
#pragma unroll 2
      for (int d = 0; d < D; d += 8) {
        float kv[8];
        ld8(kr + d, kv);
#pragma unroll
        for (int g = 0; g < kMaxGroup; ++g) {
          if (g < G) {
#pragma unroll
            for (int e = 0; e < 8; ++e) sc[g] = fmaf(qs[g][d + e], kv[e], sc[g]);
          }
        }
      }
    }
    // Tile max per head.
    const int warp = tid >> 5, lane = tid & 31;
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) {
      sc[g] = live ? sc[g] * scale : -INFINITY;
      float v = g < G ? warp_max(sc[g]) : -INFINITY;
      if (lane == 0) red[warp][g] = v;
    }
    __syncthreads();
    float m_new[kMaxGroup], alpha[kMaxGroup];
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) {
      float tm = fmaxf(fmaxf(red[0][g], red[1][g]), fmaxf(red[2][g], red[3][g]));
      m_new[g] = fmaxf(m_run[g], tm);
      alpha[g] = m_run[g] == -INFINITY ? 0.0f : expf(m_run[g] - m_new[g]);
    }
    __syncthreads();
    // Probabilities and tile sums.
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) {
      const float pv = (live && g < G) ? expf(sc[g] - m_new[g]) : 0.0f;
      ps[g][tid] = pv;
      const float s = warp_sum(pv);
      if (lane == 0) red[warp][g] = s;
    }
    __syncthreads();
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) {
      l_run[g] = l_run[g] * alpha[g] + (red[0][g] + red[1][g] + red[2][g] + red[3][g]);
      m_run[g] = m_new[g];
      acc[g][0] *= alpha[g];
      acc[g][1] *= alpha[g];
    }
    // PV: each v row read once for all G heads.
    const int tn = min(kThreads, t_end - t0);
    for (int j = phase; j < tn; j += kPhases) {
      const float2 vv = ld2(vbase + int64_t(t0 + j) * D + 2 * pair);
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g) {
        if (g < G) {
          const float pj = ps[g][j];
          acc[g][0] = fmaf(pj, vv.x, acc[g][0]);
          acc[g][1] = fmaf(pj, vv.y, acc[g][1]);
        }
      }
    }
    __syncthreads();
  }

  // Combine the position phases.
#pragma unroll
  for (int g = 0; g < kMaxGroup; ++g) {
    if (g < G) {
      accs[phase][g][2 * pair] = acc[g][0];
      accs[phase][g][2 * pair + 1] = acc[g][1];
    }
  }
  __syncthreads();
  for (int i = tid; i < G * D; i += kThreads) {
    const int g = i / D, d = i % D;
    float a = 0.0f;
#pragma unroll
    for (int ph = 0; ph < kPhases; ++ph) a += accs[ph][g][d];
    const int h = kvh * G + g;
    if (splits == 1) {
      const float o = l_run[g] > 0.0f ? a / l_run[g] : 0.0f;
      st1(out + int64_t(row) * heads * D + int64_t(h) * D + d, o);
    } else {
      float* pp = partial + ((int64_t(row) * heads + h) * splits + split) * (D + 2);
      pp[2 + d] = a;
      if (d == 0) {
        pp[0] = m_run[g];
        pp[1] = l_run[g];
      }
    }
  }
}

template <typename T, int D>
__global__ void attn_merge_kernel(const float* __restrict__ partial, int heads, int splits,
                                  T* __restrict__ out) {
  pdl_trigger();
  pdl_wait();
  extern __shared__ float wts[];  // [splits] weight of each split
  __shared__ float inv_l;
  const int rh = blockIdx.x;  // row * heads + h
  const float* pp = partial + int64_t(rh) * splits * (D + 2);
  const int tid = threadIdx.x;
  // Per-split maxima, loaded in parallel.
  for (int s = tid; s < splits; s += blockDim.x) wts[s] = pp[s * (D + 2)];
  __syncthreads();
  if (tid < 32) {
    float mx = -INFINITY;
    for (int s = tid; s < splits; s += 32) mx = fmaxf(mx, wts[s]);
    mx = warp_max(mx);
    float l = 0.0f;
    for (int s = tid; s < splits; s += 32) {
      const float ms = wts[s];
      const float w = ms == -INFINITY ? 0.0f : expf(ms - mx);
      l += pp[s * (D + 2) + 1] * w;
      wts[s] = w;
    }
    l = warp_sum(l);
    if (tid == 0) inv_l = l > 0.0f ? 1.0f / l : 0.0f;
  }
  __syncthreads();
  for (int d = tid; d < D; d += blockDim.x) {
    float a0 = 0.0f, a1 = 0.0f, a2 = 0.0f, a3 = 0.0f;
    int s = 0;
    for (; s + 4 <= splits; s += 4) {  // four independent loads in flight
      a0 = fmaf(pp[(s + 0) * (D + 2) + 2 + d], wts[s + 0], a0);
      a1 = fmaf(pp[(s + 1) * (D + 2) + 2 + d], wts[s + 1], a1);
      a2 = fmaf(pp[(s + 2) * (D + 2) + 2 + d], wts[s + 2], a2);
      a3 = fmaf(pp[(s + 3) * (D + 2) + 2 + d], wts[s + 3], a3);
    }
    for (; s < splits; ++s) a0 = fmaf(pp[s * (D + 2) + 2 + d], wts[s], a0);
    st1(out + int64_t(rh) * D + d, ((a0 + a1) + (a2 + a3)) * inv_l);
  }
}

// ---------------------------------------------------------------------------
// bf16 decode attention, version 2: one block per (chunk of CH positions, kv
// head, query row).  Cache rows below the row's position never change during
// this step, so they are copied to shared memory with cp.async *before*
// griddepcontrol.wait -- under programmatic dependent launch the KV stream
// overlaps the previous kernel (the q/k/v projection).  The row at the
// position itself (just appended by that kernel) and q are read after the
// wait.  The block computes the G query heads' scores for its chunk from the
// staged k rows, a local softmax, and the unnormalised PV sum, and writes
// (max, sum, acc) partials for attn_merge_kernel.  A kv head shared by more
// than kMaxGroup query heads (wide GQA, MQA) is covered by several blocks,
// each taking kMaxGroup of its query heads: grid.y = kv head x head chunk.
// ---------------------------------------------------------------------------
template <int D, int CH>
struct AttnV2Smem {
  static constexpr int kRowK = D * 2 + 16;  // padded k row (bytes): conflict-free 16-byte reads
  static constexpr int kRowV = D * 2;
  static constexpr size_t bytes(int G) {
    return size_t(CH) * kRowK + size_t(CH) * kRowV + size_t(G) * D * 4 + size_t(G) * CH * 4 +
           size_t(kThreads / (D / 2)) * G * D * 4 + 2 * size_t(G) * 4;
  }
};

template <int D, int CH>
__global__ void __launch_bounds__(kThreads)
    attn_v2_kernel(const uint16_t* __restrict__ q, const uint16_t* __restrict__ kc,
                   const uint16_t* __restrict__ vc, const int32_t* __restrict__ pos,
                   int tokens_per_seq, int heads, int kv_heads, int max_len, int splits,
                   float scale, int pos_external, float* __restrict__ partial,
                   uint16_t* __restrict__ out, int* err) {
  using L = AttnV2Smem<D, CH>;
  constexpr int kPairs = D / 2;
  constexpr int kPhases = kThreads / kPairs;
  extern __shared__ __align__(128) uint8_t smem[];
  const int split = blockIdx.x, row = blockIdx.z;
  const int G_all = heads / kv_heads;                    // query heads per kv head
  const int nchunk = (G_all + kMaxGroup - 1) / kMaxGroup;
  const int kvh = blockIdx.y / nchunk;
  const int h0 = kvh * G_all + (blockIdx.y - kvh * nchunk) * kMaxGroup;  // first query head of this block
  const int G = min(kMaxGroup, kvh * G_all + G_all - h0);                // query heads of this block
  const int tid = threadIdx.x;
  uint8_t* sK = smem;
  uint8_t* sV = sK + CH * L::kRowK;
  float* sQ = reinterpret_cast<float*>(sV + CH * L::kRowV);  // [G][D]
  float* sS = sQ + G * D;                                    // [G][CH]
  float* sA = sS + G * CH;                                   // [kPhases][G][D]
  float* sM = sA + kPhases * G * D;                          // [G] max, [G] sum

  pdl_trigger();
  const int seq = row / tokens_per_seq;
  const uint8_t* kb = reinterpret_cast<const uint8_t*>(kc + (int64_t(seq) * kv_heads + kvh) * int64_t(max_len) * D);
  const uint8_t* vb = reinterpret_cast<const uint8_t*>(vc + (int64_t(seq) * kv_heads + kvh) * int64_t(max_len) * D);
  const int t_begin = split * CH;

  auto stage = [&](int r0, int r1) {  // rows [r0, r1) of this chunk, chunk-relative
    const int n = (r1 - r0) * (D / 8);
    for (int c = tid; c < 2 * n; c += kThreads) {
      const bool isv = c >= n;
      const int cc = isv ? c - n : c;
      const int r = r0 + cc / (D / 8), off = (cc % (D / 8)) * 16;
      const int64_t src = int64_t(t_begin + r) * D * 2 + off;
      if (isv) cp_async16(sV + r * L::kRowV + off, vb + src);
      else cp_async16(sK + r * L::kRowK + off, kb + src);
    }
  };

  int pre = 0;  // rows staged before the wait
  int p_early = -1;
  if (pos_external && tokens_per_seq == 1) {
    p_early = pos[row];
    if (p_early >= 0 && p_early < max_len) {
      pre = min(CH, max(0, p_early - t_begin));
      stage(0, pre);
    }
  }
  pdl_wait();
  const int p = pos_external && tokens_per_seq == 1 ? p_early : pos[row];
  const bool bad = p < 0 || p >= max_len;
  if (bad && tid == 0 && err) atomicExch(err, 2);
  const int len = bad ? 0 : p + 1;
  const int n_t = max(0, min(CH, len - t_begin));
  if (n_t > pre) stage(pre, n_t);
  for (int i = tid; i < G * D; i += kThreads) {
    const int g = i / D, d = i % D;
    sQ[i] = bf2f(q[int64_t(row) * heads * D + int64_t(h0 + g) * D + d]);
  }
  cp_async_commit_wait_all();
  __syncthreads();

  // Scores: position t = tid % CH, heads strided by kThreads / CH.
  for (int item = tid; item < CH * G; item += kThreads) {
    const int t = item % CH, g = item / CH;
    float acc = 0.0f;
    if (t < n_t) {
      const uint8_t* kr = sK + t * L::kRowK;
      const float* qg = sQ + g * D;
#pragma unroll 4
      for (int d = 0; d < D; d += 8) {
        const uint4 kv = *reinterpret_cast<const uint4*>(kr + d * 2);
        acc = fmaf(qg[d + 0], bf_lo(kv.x), acc);
        acc = fmaf(qg[d + 1], bf_hi(kv.x), acc);
        acc = fmaf(qg[d + 2], bf_lo(kv.y), acc);
        acc = fmaf(qg[d + 3], bf_hi(kv.y), acc);
        acc = fmaf(qg[d + 4], bf_lo(kv.z), acc);
        acc = fmaf(qg[d + 5], bf_hi(kv.z), acc);
        acc = fmaf(qg[d + 6], bf_lo(kv.w), acc);
        acc = fmaf(qg[d + 7], bf_hi(kv.w), acc);
      }
      acc *= scale;
    }
    sS[g * CH + t] = t < n_t ? acc : -INFINITY;
  }
  __syncthreads();
  // Softmax statistics: warp w handles heads w, w + 4, ...
  {
    const int warp = tid >> 5, lane = tid & 31;
    for (int g = warp; g < G; g += kThreads / 32) {
      float mx = -INFINITY;
      for (int t = lane; t < CH; t += 32) mx = fmaxf(mx, sS[g * CH + t]);
      mx = warp_max(mx);
      float sum = 0.0f;
      for (int t = lane; t < CH; t += 32) {
        const float e = t < n_t ? expf(sS[g * CH + t] - mx) : 0.0f;
        sS[g * CH + t] = e;
        sum += e;
      }
      sum = warp_sum(sum);
      if (lane == 0) {
        sM[g] = mx;
        sM[G + g] = sum;
      }
    }
  }
  __syncthreads();
  // PV: thread owns a d pair and one position phase; each v row read once.
  {
    const int pair = tid % kPairs, phase = tid / kPairs;
    float a[kMaxGroup][2];
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) a[g][0] = a[g][1] = 0.0f;
    for (int t = phase; t < n_t; t += kPhases) {
      const uint32_t vv = *reinterpret_cast<const uint32_t*>(sV + t * L::kRowV + pair * 4);
      const float v0 = bf_lo(vv), v1 = bf_hi(vv);
#pragma unroll
      for (int g = 0; g < kMaxGroup; ++g) {
        if (g < G) {
          const float pg = sS[g * CH + t];
          a[g][0] = fmaf(pg, v0, a[g][0]);
          a[g][1] = fmaf(pg, v1, a[g][1]);
        }
      }
    }
#pragma unroll
    for (int g = 0; g < kMaxGroup; ++g) {
      if (g < G) {
        sA[(phase * G + g) * D + 2 * pair] = a[g][0];
        sA[(phase * G + g) * D + 2 * pair + 1] = a[g][1];
      }
    }
  }
  __syncthreads();
  for (int i = tid; i < G * D; i += kThreads) {
    const int g = i / D, d = i % D;
    float acc = 0.0f;
#pragma unroll
    for (int ph = 0; ph < kPhases; ++ph) acc += sA[(ph * G + g) * D + d];
    const int h = h0 + g;
    const float mx = n_t > 0 ? sM[g] : -INFINITY, l = n_t > 0 ? sM[G + g] : 0.0f;
    if (splits == 1) {
      out[int64_t(row) * heads * D + int64_t(h) * D + d] = f2bf(l > 0.0f ? acc / l : 0.0f);
    } else {
      float* pp = partial + ((int64_t(row) * heads + h) * splits + split) * (D + 2);
      pp[2 + d] = acc;
      if (d == 0) {
        pp[0] = mx;
        pp[1] = l;
      }
    }
  }
}

}  // namespace

int attention_chunk(int64_t rows, int64_t kv_heads) {
  // Small grids (one or a few sequences) use shorter chunks for more blocks.
  return rows * kv_heads <= 64 ? 64 : 128;
}

int attention_v2_splits(int64_t rows, int64_t kv_heads, int64_t max_len) {
  const int ch = attention_chunk(rows, kv_heads);
  return int((max_len + ch - 1) / ch);
}

uint64_t attention_v2_scratch_bytes(int64_t rows, int64_t heads, int64_t kv_heads, int64_t head_dim,
                                    int64_t max_len) {
  // Only the CUDA-core kernel writes split partials; the tensor-core decode
  // kernel merges its splits on chip and the prefill kernel has none.  This
  // mirrors launch_attention_v2's choice of kernel.
  if (attention_tc_supported(heads, kv_heads, head_dim)) return 0;
  const int64_t s = attention_v2_splits(rows, kv_heads, max_len);
  if (s == 1) return 0;
  return uint64_t(rows) * heads * s * (head_dim + 2) * sizeof(float);
}

template <int D, int CH>
static int launch_v2(const uint16_t* q, const uint16_t* kc, const uint16_t* vc, const int32_t* pos,
                     int64_t rows, int64_t tps, int64_t heads, int64_t kv_heads, int64_t max_len,
                     int splits, bool pos_external, float* scratch, uint16_t* out, int* err,
                     cudaStream_t st) {
  const int G = int(heads / kv_heads);
  const int nchunk = (G + kMaxGroup - 1) / kMaxGroup;
  const size_t smem = AttnV2Smem<D, CH>::bytes(G < kMaxGroup ? G : kMaxGroup);
  static PerDeviceOnce configured;
  if (!configured.run([] {
        return cudaFuncSetAttribute(attn_v2_kernel<D, CH>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                    int(AttnV2Smem<D, CH>::bytes(kMaxGroup))) == cudaSuccess;
      }))
    return SB_INTERNAL;
  const float scale = 1.0f / sqrtf(float(D));
  const dim3 grid(splits, unsigned(kv_heads * nchunk), unsigned(rows));
  if (launch_pdl(attn_v2_kernel<D, CH>, grid, dim3(kThreads), smem, st, q, kc, vc, pos, int(tps), int(heads),
                 int(kv_heads), int(max_len), splits, scale, pos_external ? 1 : 0, scratch, out, err) !=
      cudaSuccess)
    return SB_INTERNAL;
  count_launch();
  if (splits > 1) {
    const unsigned nb = unsigned(rows * heads);
    if (launch_pdl(attn_merge_kernel<uint16_t, D>, dim3(nb), dim3(D), splits * sizeof(float), st, (const float*)scratch, int(heads),
                   splits, out) != cudaSuccess)
      return SB_INTERNAL;
    count_launch();
  }
  return SB_OK;
}

int launch_attention_merge_bf16(const float* scratch, int64_t rows, int64_t heads, int64_t head_dim, int splits,
                                uint16_t* out, cudaStream_t st) {
  const unsigned nb = unsigned(rows * heads);
  cudaError_t e;
  if (head_dim == 128)
    e = launch_pdl(attn_merge_kernel<uint16_t, 128>, dim3(nb), dim3(128), splits * sizeof(float), st, scratch,
                   int(heads), splits, out);
  else if (head_dim == 64)
    e = launch_pdl(attn_merge_kernel<uint16_t, 64>, dim3(nb), dim3(64), splits * sizeof(float), st, scratch,
                   int(heads), splits, out);
  else
    return SB_INVALID_ARGUMENT;
  if (e != cudaSuccess) return SB_INTERNAL;
  count_launch();
  return SB_OK;
}

// bf16 attention: the tensor-core prefill kernel for 16 or more tokens per
// sequence, the tensor-core decode kernel (k_attn_tc.cu) for up to 8 query
// heads per kv head, and the CUDA-core kernel above for wider groups (MQA,
// 16:1 GQA), which is the only one of the three that uses `scratch`.
int launch_attention_v2(const uint16_t* q, const uint16_t* k_cache, const uint16_t* v_cache,
                        const int32_t* pos, int64_t rows, int64_t tokens_per_seq, int64_t heads,
                        int64_t kv_heads, int64_t head_dim, int64_t max_len, bool pos_external,
                        float* scratch, uint16_t* out, int* err, cudaStream_t st, const KvPages& kp) {
  if (rows == 0) return SB_OK;
  if (attention_prefill_supported(rows, tokens_per_seq, heads, kv_heads, head_dim))
    return launch_attention_prefill(q, k_cache, v_cache, pos, rows, tokens_per_seq, heads, kv_heads, head_dim,
                                    max_len, out, err, st, kp);
  if (attention_tc_supported(heads, kv_heads, head_dim))
    return launch_attention_tc(q, k_cache, v_cache, pos, rows, tokens_per_seq, heads, kv_heads, head_dim, max_len,
                               pos_external, scratch, out, err, st, kp);
  if (kp.paged()) return SB_INVALID_ARGUMENT;
  if (kv_heads <= 0 || heads % kv_heads || rows > 65535) return SB_INVALID_ARGUMENT;
  if (kv_heads * ((heads / kv_heads + kMaxGroup - 1) / kMaxGroup) > 65535) return SB_INVALID_ARGUMENT;
  const int splits = attention_v2_splits(rows, kv_heads, max_len);
  if (splits > 1 && scratch == nullptr) return SB_INVALID_ARGUMENT;
  const int ch = attention_chunk(rows, kv_heads);
  if (head_dim == 128)
    return ch == 64 ? launch_v2<128, 64>(q, k_cache, v_cache, pos, rows, tokens_per_seq, heads, kv_heads, max_len,
                                         splits, pos_external, scratch, out, err, st)
                    : launch_v2<128, 128>(q, k_cache, v_cache, pos, rows, tokens_per_seq, heads, kv_heads,
                                          max_len, splits, pos_external, scratch, out, err, st);
  if (head_dim == 64)
    return ch == 64 ? launch_v2<64, 64>(q, k_cache, v_cache, pos, rows, tokens_per_seq, heads, kv_heads, max_len,
                                        splits, pos_external, scratch, out, err, st)
                    : launch_v2<64, 128>(q, k_cache, v_cache, pos, rows, tokens_per_seq, heads, kv_heads,
                                         max_len, splits, pos_external, scratch, out, err, st);
  return SB_INVALID_ARGUMENT;
}

namespace {
}  // namespace

// Splits so that the grid covers about two waves of the 148 SMs, with at
// least 256 positions per split.
int attention_splits(int64_t rows, int64_t kv_heads, int64_t max_len) {
  const int64_t blocks = rows * kv_heads;
  int64_t s = (2 * kNumSMs + blocks - 1) / blocks;
  const int64_t cap = (max_len + 255) / 256;
  if (s > cap) s = cap;
  if (s > 32) s = 32;
  return int(s < 1 ? 1 : s);
}

uint64_t attention_scratch_bytes(int64_t rows, int64_t heads, int64_t kv_heads, int64_t head_dim,
                                 int64_t max_len) {
  const int s = attention_splits(rows, kv_heads, max_len);
  if (s == 1) return 0;
  return uint64_t(rows) * heads * s * (head_dim + 2) * sizeof(float);
}

template <typename T>
int launch_kv_append(const T* k_new, const T* v_new, T* k_cache, T* v_cache, const int32_t* pos,
                     int64_t rows, int64_t tokens_per_seq, int64_t kv_heads, int64_t head_dim,
                     int64_t max_len, int* err, cudaStream_t st, const KvPages& kp) {
  if (rows == 0) return SB_OK;
  if (kp.paged() && (!kv_page_size_ok(kp.page_size) || int64_t(kp.page_size) * kp.pages_per_seq != max_len))
    return SB_INVALID_ARGUMENT;
  launch_pdl(kv_append_kernel<T>, dim3(unsigned(rows)), dim3(256), 0, st, k_new, v_new, k_cache, v_cache, pos,
             int(rows), int(tokens_per_seq), int(kv_heads), int(head_dim), int(max_len), kp, err);
  SB_LAUNCH_CHECK();
  return SB_OK;
}

template <typename T>
int launch_attention(const T* q, const T* k_cache, const T* v_cache, const int32_t* pos,
                     int64_t rows, int64_t tokens_per_seq, int64_t heads, int64_t kv_heads,
                     int64_t head_dim, int64_t max_len, float* scratch, T* out, int* err,
                     cudaStream_t st) {
  if (rows == 0) return SB_OK;
  if (kv_heads <= 0 || heads % kv_heads || heads / kv_heads > kMaxGroup)
    return SB_INVALID_ARGUMENT;
  if (head_dim != 64 && head_dim != 128) return SB_INVALID_ARGUMENT;
  const int splits = attention_splits(rows, kv_heads, max_len);
  if (splits > 1 && scratch == nullptr) return SB_INVALID_ARGUMENT;
  const float scale = 1.0f / sqrtf(float(head_dim));
  const dim3 grid(splits, unsigned(kv_heads), unsigned(rows));
  if (head_dim == 128) {
    launch_pdl(attn_kernel<T, 128>, dim3(grid), dim3(kThreads), 0, st, q, k_cache, v_cache, pos, int(tokens_per_seq),
                                                   int(heads), int(kv_heads), int(max_len),
                                                   splits, scale, scratch, out, err);
  } else {
    launch_pdl(attn_kernel<T, 64>, dim3(grid), dim3(kThreads), 0, st, q, k_cache, v_cache, pos, int(tokens_per_seq),
                                                  int(heads), int(kv_heads), int(max_len), splits,
                                                  scale, scratch, out, err);
  }
  SB_LAUNCH_CHECK();
  if (splits > 1) {
    const unsigned nb = unsigned(rows * heads);
    if (head_dim == 128)
      launch_pdl(attn_merge_kernel<T, 128>, dim3(nb), dim3(128), splits * sizeof(float), st, scratch, int(heads), splits, out);
    else
      launch_pdl(attn_merge_kernel<T, 64>, dim3(nb), dim3(64), splits * sizeof(float), st, scratch, int(heads), splits, out);
    SB_LAUNCH_CHECK();
  }
  return SB_OK;
}

template int launch_kv_append<uint16_t>(const uint16_t*, const uint16_t*, uint16_t*, uint16_t*,
                                        const int32_t*, int64_t, int64_t, int64_t, int64_t,
                                        int64_t, int*, cudaStream_t, const KvPages&);
template int launch_kv_append<float>(const float*, const float*, float*, float*, const int32_t*,
                                     int64_t, int64_t, int64_t, int64_t, int64_t, int*,
                                     cudaStream_t, const KvPages&);
template int launch_attention<uint16_t>(const uint16_t*, const uint16_t*, const uint16_t*,
                                        const int32_t*, int64_t, int64_t, int64_t, int64_t,
                                        int64_t, int64_t, float*, uint16_t*, int*, cudaStream_t);
template int launch_attention<float>(const float*, const float*, const float*, const int32_t*,
                                     int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                                     float*, float*, int*, cudaStream_t);

}  // namespace sb
