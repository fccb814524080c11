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
#include "common.cuh"

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
                                 int kv_heads, int head_dim, int max_len, int* err) {
  const int row = blockIdx.x;
  const int p = pos[row];
  if (p < 0 || p >= max_len) {
    if (threadIdx.x == 0 && err) atomicExch(err, 2);
    return;
  }
  const int seq = row / tokens_per_seq;
  const int width = kv_heads * head_dim;
  for (int i = threadIdx.x; i < width; i += blockDim.x) {
    const int h = i / head_dim, d = i % head_dim;
    const int64_t dst = ((int64_t(seq) * kv_heads + h) * max_len + p) * head_dim + d;
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
  constexpr int kPairs = D / 2;              // d pairs per row
  constexpr int kPhases = kThreads / kPairs;  // position phases in the PV loop
  const int split = blockIdx.x, kvh = blockIdx.y, row = blockIdx.z;
  const int G = heads / kv_heads;
  const int tid = threadIdx.x;

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
  const int rh = blockIdx.x;  // row * heads + h
  const float* pp = partial + int64_t(rh) * splits * (D + 2);
  float mx = -INFINITY;
  for (int s = 0; s < splits; ++s) mx = fmaxf(mx, pp[s * (D + 2)]);
  float l = 0.0f;
  for (int s = 0; s < splits; ++s) {
    const float ms = pp[s * (D + 2)];
    if (ms != -INFINITY) l += pp[s * (D + 2) + 1] * expf(ms - mx);
  }
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float a = 0.0f;
    for (int s = 0; s < splits; ++s) {
      const float ms = pp[s * (D + 2)];
      if (ms != -INFINITY) a += pp[s * (D + 2) + 2 + d] * expf(ms - mx);
    }
    st1(out + int64_t(rh) * D + d, l > 0.0f ? a / l : 0.0f);
  }
}

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
                     int64_t max_len, int* err, cudaStream_t st) {
  if (rows == 0) return SB_OK;
  kv_append_kernel<T><<<unsigned(rows), 256, 0, st>>>(k_new, v_new, k_cache, v_cache, pos,
                                                      int(rows), int(tokens_per_seq),
                                                      int(kv_heads), int(head_dim),
                                                      int(max_len), err);
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
    attn_kernel<T, 128><<<grid, kThreads, 0, st>>>(q, k_cache, v_cache, pos, int(tokens_per_seq),
                                                   int(heads), int(kv_heads), int(max_len),
                                                   splits, scale, scratch, out, err);
  } else {
    attn_kernel<T, 64><<<grid, kThreads, 0, st>>>(q, k_cache, v_cache, pos, int(tokens_per_seq),
                                                  int(heads), int(kv_heads), int(max_len), splits,
                                                  scale, scratch, out, err);
  }
  SB_LAUNCH_CHECK();
  if (splits > 1) {
    const unsigned nb = unsigned(rows * heads);
    if (head_dim == 128)
      attn_merge_kernel<T, 128><<<nb, 128, 0, st>>>(scratch, int(heads), splits, out);
    else
      attn_merge_kernel<T, 64><<<nb, 64, 0, st>>>(scratch, int(heads), splits, out);
    SB_LAUNCH_CHECK();
  }
  return SB_OK;
}

template int launch_kv_append<uint16_t>(const uint16_t*, const uint16_t*, uint16_t*, uint16_t*,
                                        const int32_t*, int64_t, int64_t, int64_t, int64_t,
                                        int64_t, int*, cudaStream_t);
template int launch_kv_append<float>(const float*, const float*, float*, float*, const int32_t*,
                                     int64_t, int64_t, int64_t, int64_t, int64_t, int*,
                                     cudaStream_t);
template int launch_attention<uint16_t>(const uint16_t*, const uint16_t*, const uint16_t*,
                                        const int32_t*, int64_t, int64_t, int64_t, int64_t,
                                        int64_t, int64_t, float*, uint16_t*, int*, cudaStream_t);
template int launch_attention<float>(const float*, const float*, const float*, const int32_t*,
                                     int64_t, int64_t, int64_t, int64_t, int64_t, int64_t,
                                     float*, float*, int*, cudaStream_t);

}  // namespace sb
