// Tensor-core GEMV for decode (M <= 16 rows of x per launch), int4 group-32,
// int8 per-channel and MX (MXFP8 / MXFP4, E8M0 scales per 32) weights, with
// fused epilogues.
//
// Work decomposition.  The output is cut into 16-row mma.m16n8k16 tiles.  The
// grid is persistent (at most one wave of resident blocks); block b computes
// tiles b, b + grid, b + 2 grid, ...  Within a tile the W warps (8, 12 or 16:
// choose_warps) split K into W slices of whole 32-code groups and the W
// partial fragments are summed through shared memory by finish_tile.  (Splitting a tile's K over the CTAs
// of a cluster, with the partial sums merged through distributed shared
// memory, measured slower on most 7B shapes and at best 9 % faster on one:
// the per-tile cluster barrier costs about what the shorter slices save.)
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
// int4 codes at k offsets 8q..8q+7.  Flipping each code's sign bit turns c
// into c + 8; placing nibble pairs (j, j+4) in the mantissa of bf16 128.0 and
// subtracting 136.0 gives the exact codes as bf16x2 pairs (int4_pair).  The MMA's k order
// inside a group is permuted to match (virtual k 2q,2q+1 <-> real 8q+2s,
// 8q+2s+4 for k16 step s) and the activations are permuted the same way with
// byte permutes, so the dot product is unchanged.  Each group's two MMAs
// accumulate into a fresh fragment that is scaled by the group's bf16 scale in
// f32: dequantisation is exactly code * scale, as in the oracle.
#include <cstdlib>
#include <string>

#include "k_gemv_mma.cuh"
#include "k_int4.cuh"

namespace sb {

namespace {

constexpr int kWarps = 8;      // K-slices per block (12 or 16 where choose_warps picks them)
constexpr int kTileRows = 16;  // output rows per block
constexpr int kChunk = 8;      // groups per pipeline stage
constexpr int kMaxRows = 64;  // x rows per launch

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
  int scale16;       // int4: slices are whole 8-group chunks, scales copied 16 B per row
  QkvExtra qkv;
};

// Tile y's matrix rows: tile row t < 8 is row row_lo + t of job job_lo, tile
// row t >= 8 is row row_hi + t - 8 of job job_hi.  Rows t and t + 8 form one
// epilogue pair (gate/up for SwiGLU, the two rotate-half partners for QkvRope).
struct TileRows {
  int job_lo, row_lo, job_hi, row_hi;
};

template <int MODE>
__device__ __forceinline__ TileRows tile_rows(const Params& p, int y) {
  TileRows tr;
  if constexpr (MODE == 0) {
    int r = y * kTileRows, job = 0;
    while (job + 1 < p.njobs && r >= p.n[job]) r -= p.n[job++];
    tr = {job, r, job, r + 8};
  } else if constexpr (MODE == 1) {
    tr = {0, y * 8, 1, y * 8};
  } else {
    const int hd = p.qkv.head_dim;
    const int bph = hd / 16;  // tiles per head: 8 rotate-half pairs per tile
    const int head = y / bph, j = y - head * bph;
    int job = 0, hb = head;
    if (head >= p.qkv.hq + p.qkv.hkv) {
      job = 2;
      hb = head - p.qkv.hq - p.qkv.hkv;
    } else if (head >= p.qkv.hq) {
      job = 1;
      hb = head - p.qkv.hq;
    }
    tr = {job, hb * hd + 8 * j, job, hb * hd + 8 * j + hd / 2};
  }
  return tr;
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], const void* smem) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(a));
}

__device__ __forceinline__ uint32_t lds32(const void* smem) {
  return *reinterpret_cast<const uint32_t*>(smem);
}

__device__ __forceinline__ void cp_async4(void* smem, const void* gmem) {
  const uint32_t a = static_cast<uint32_t>(__cvta_generic_to_shared(smem));
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(a), "l"(gmem) : "memory");
}

template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// The epilogue of output pair (tile row pp, pp + 8) for x row m: vlo / vhi are
// the finished dot products.
template <int FMT, int MODE>
__device__ __forceinline__ void tile_epilogue(const Params& p, const TileRows& tr, int pp, int m, float vlo,
                                              float vhi) {
  {
    const int jl = tr.job_lo, nlo = tr.row_lo + pp, jh = tr.job_hi, nhi = tr.row_hi + pp;
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
      // The projection output is a bf16 value: round before the rotation,
      // which runs in f32 as in rope_kernel.
      float xlo = bf2f(f2bf(vlo)), xhi = bf2f(f2bf(vhi));
      const int pos = e.pos[m];
      if (jl < 2) {
        const double inv = e.inv_freq ? e.inv_freq[i] : pow(e.theta, -2.0 * double(i) / double(hd));
        float sn, cs;
        rope_cos_sin(pos, inv, cs, sn);
        const float a = fmaf(xlo, cs, -xhi * sn), b = fmaf(xhi, cs, xlo * sn);
        xlo = a;
        xhi = b;
      }
      const uint16_t olo = f2bf(xlo), ohi = f2bf(xhi);
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
        const int seq = (p.m_base + m) / e.tokens_per_seq;
        const bool in_range = pos >= 0 && pos < e.max_len;
        const int64_t crow = in_range ? kv_row(e.kp, seq, head_in_job, e.hkv, e.max_len, pos) : -1;
        if (crow >= 0) {
          uint16_t* dst = (jl == 1 ? e.k_cache : e.v_cache) + crow * hd;
          dst[i] = olo;
          dst[i + half] = ohi;
        } else if (e.err) {
          atomicExch(e.err, in_range ? 6 : 2);  // 6: the position's page is missing
        }
      }
    }
  }
}

// Sum the 8 K-slice partials of one tile through shared memory and run the
// epilogue.  Every thread of the block calls this once per tile.
template <int FMT, int NT, int MODE, bool kTrailingSync, int W>
__device__ __forceinline__ void finish_tile(const Params& p, const TileRows& tr,
                                            float (&red)[W][kTileRows][8 * NT],
                                            const float (&acc)[NT][4], int warp, int g, int q, int tid) {
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    *reinterpret_cast<float2*>(&red[warp][g][t * 8 + 2 * q]) = make_float2(acc[t][0], acc[t][1]);
    *reinterpret_cast<float2*>(&red[warp][g + 8][t * 8 + 2 * q]) = make_float2(acc[t][2], acc[t][3]);
  }
  __syncthreads();
  const int items = 8 * p.m;
  for (int it = tid; it < items; it += W * 32) {
    const int pp = it / p.m, m = it - pp * p.m;
    float vlo = 0.0f, vhi = 0.0f;
#pragma unroll
    for (int w = 0; w < W; ++w) {
      vlo += red[w][pp][m];
      vhi += red[w][pp + 8][m];
    }
    tile_epilogue<FMT, MODE>(p, tr, pp, m, vlo, vhi);
  }
  // A single buffer is rewritten by the next tile; with two buffers the next
  // tile's barrier already orders this tile's reads before the reuse.
  if (kTrailingSync) __syncthreads();
}

// One pipeline stage of one warp: kChunk groups of the tile's 16 rows, stored
// row-major (16 rows x kChunk * bytes per group) with the 16-byte pieces of
// row r XOR-swizzled by r & 7: copies write whole rows and an ldmatrix 8x8
// matrix (8 rows of one piece) lands in 8 different bank groups.  int4
// stages also hold the bf16 scales [16 rows][kChunk].
// FMT: 0 int4 g32 (bf16 scales), 1 int8 per channel (f32 scale in the
// epilogue), 2 MXFP8 (E4M3 codes), 3 MXFP4 (E2M1 codes, two per byte); the
// MX formats have one E8M0 scale byte per row and group of 32.
template <int FMT>
struct Stage {
  static constexpr bool kNibbles = FMT == 0 || FMT == 3;             // two codes per byte
  static constexpr int kBPG = kNibbles ? 16 : 32;                    // bytes per row per group
  static constexpr int kRowBytes = kChunk * kBPG;                    // 128 / 256
  static constexpr int kPieces = kRowBytes / 16;                     // 8 / 16
  static constexpr int kW = kTileRows * kRowBytes;                   // weight bytes
  static constexpr int kS = FMT == 0 ? kTileRows * kChunk * 2 : FMT >= 2 ? kTileRows * kChunk : 0;  // scale bytes
  static constexpr int kBytes = kW + kS;
  static constexpr int kDepth = 2;                                   // stages per warp
};

// Byte offset of 16-byte piece `piece` of tile row `row` in a stage.
template <int FMT>
__device__ __forceinline__ int piece_off(int row, int piece) {
  return row * Stage<FMT>::kRowBytes + ((piece ^ (row & 7)) << 4);
}

__host__ __device__ constexpr size_t warp_smem_bytes(int fmt) {
  return fmt == 0   ? size_t(Stage<0>::kDepth) * Stage<0>::kBytes
         : fmt == 1 ? size_t(Stage<1>::kDepth) * Stage<1>::kBytes
         : fmt == 2 ? size_t(Stage<2>::kDepth) * Stage<2>::kBytes
                    : size_t(Stage<3>::kDepth) * Stage<3>::kBytes;
}

// One int4 group of the tile for every n-tile: dequantise the words of rows
// g (ul) and g + 8 (uh), two MMAs into a fresh fragment, scale by the group's
// bf16 scales (half `hi` of the scale pairs slo / shi), accumulate.
template <int NT, int J>
__device__ __forceinline__ void int4_group(float (&acc)[NT][4], uint32_t ul, uint32_t uh, uint32_t slo, uint32_t shi,
                                           int hi, const uint4 (&xv)[NT][J], int j) {
  const uint32_t p0 = int4_pair(ul, 0), p1 = int4_pair(ul, 1), p2 = int4_pair(ul, 2), p3 = int4_pair(ul, 3);
  const uint32_t h0 = int4_pair(uh, 0), h1 = int4_pair(uh, 1), h2 = int4_pair(uh, 2), h3 = int4_pair(uh, 3);
  const float sl = __uint_as_float(hi ? (slo & 0xFFFF0000u) : (slo << 16));
  const float sh = __uint_as_float(hi ? (shi & 0xFFFF0000u) : (shi << 16));
#pragma unroll
  for (int t = 0; t < NT; ++t) {
    const uint4 x = xv[t][j];
    float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
    mma_bf16(d, p0, h0, p1, h1, prmt(x.x, x.z, 0x5410), prmt(x.x, x.z, 0x7632));
    mma_bf16(d, p2, h2, p3, h3, prmt(x.y, x.w, 0x5410), prmt(x.y, x.w, 0x7632));
    acc[t][0] = fmaf(d[0], sl, acc[t][0]);
    acc[t][1] = fmaf(d[1], sl, acc[t][1]);
    acc[t][2] = fmaf(d[2], sh, acc[t][2]);
    acc[t][3] = fmaf(d[3], sh, acc[t][3]);
  }
}

// W warps per block: 8, or 12 / 16 for launches whose tiles fit one wave of
// 12-warp blocks (two per SM) / 16-warp blocks (one per SM), where every
// tile's K is split W ways.
template <int FMT, int NT, int MODE, int W>
__global__ void __launch_bounds__(W * 32, W == 16 ? 1 : W == 12 ? 2 : NT <= 2 ? 3 : 2)
    gemv_mma_kernel(const __grid_constant__ Params p) {
  using S = Stage<FMT>;
  constexpr int kRedBufs = NT <= 2 ? 2 : 1;  // partial-sum buffers (alternate tiles)
  __shared__ __align__(16) float red[kRedBufs][W][kTileRows][8 * NT];
  extern __shared__ __align__(128) uint8_t dsm[];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int g = lane >> 2, q = lane & 3;
  uint8_t* ring = dsm + size_t(warp) * warp_smem_bytes(FMT);

  const int64_t row_bytes = int64_t(p.k) * S::kBPG / 32;
  const int gb = warp * p.gpw;                               // first group of this warp's K-slice
  const int ng = max(0, min(p.groups, gb + p.gpw) - gb);     // groups in the slice
  const int nchunks = max(1, (ng + kChunk - 1) / kChunk);    // a warp with no groups still steps

  // Copy side.  Copy instruction i moves rows r = rs + R * i of the chunk
  // (rs = lane / kPieces, R = 32 / kPieces rows per instruction), lane piece
  // h = lane % kPieces: every instruction reads whole 128-byte lines.  The
  // copy runs kDepth items ahead of the math and crosses tile boundaries.
  constexpr int kRowsPerCopy = 32 / S::kPieces;                  // 4 (int4) or 2 (int8)
  const int h = lane % S::kPieces, rs = lane / S::kPieces;
  int i_tile = blockIdx.x, i_c = 0, i_slot = 0;
  const uint8_t* wlo = nullptr;  // row rs of the tile's low half, at this warp's slice
  const uint8_t* whi = nullptr;  // row rs of the high half
  const uint8_t* srow = nullptr; // int4 scales of row (lane & 15)
  auto set_rows = [&](int y) {
    const TileRows tr = tile_rows<MODE>(p, y);
    wlo = p.w[tr.job_lo] + int64_t(tr.row_lo + rs) * row_bytes + int64_t(gb) * S::kBPG;
    whi = p.w[tr.job_hi] + int64_t(tr.row_hi + rs) * row_bytes + int64_t(gb) * S::kBPG;
    if constexpr (FMT == 0 || FMT >= 2) {
      const int r = lane & 15;
      const int job = r < 8 ? tr.job_lo : tr.job_hi;
      const int row = r < 8 ? tr.row_lo + r : tr.row_hi + r - 8;
      srow = static_cast<const uint8_t*>(p.s[job]) + (int64_t(row) * p.groups + gb) * (FMT == 0 ? 2 : 1);
    }
  };
  if (i_tile < p.tiles) set_rows(i_tile);
  auto issue = [&]() {
    if (i_tile < p.tiles) {
      const int nj = min(kChunk, ng - i_c * kChunk);  // <= 0 for a warp with no groups
      uint8_t* dst = ring + i_slot * S::kBytes;
      const int64_t coff = int64_t(i_c) * S::kRowBytes + h * 16;
      if ((h * 16) / S::kBPG < nj) {
#pragma unroll
        for (int i = 0; i < kTileRows / kRowsPerCopy; ++i) {
          const int r = rs + kRowsPerCopy * i;
          const int rh = i < kTileRows / kRowsPerCopy / 2 ? kRowsPerCopy * i : kRowsPerCopy * i - 8;
          const uint8_t* base = i < kTileRows / kRowsPerCopy / 2 ? wlo : whi;
          cp_async16(dst + piece_off<FMT>(r, h), base + int64_t(rh) * row_bytes + coff);
        }
      }
      if constexpr (FMT == 0) {
        const uint8_t* ssrc = srow + i_c * (kChunk * 2);
        uint8_t* sdst = dst + S::kW + (lane & 15) * (kChunk * 2);
        if (p.scale16) {
          if (lane < 16 && nj > 0) cp_async16(sdst, ssrc);
        } else {
          // bf16 pairs: the group count and the slice start are even, so every
          // pair starts on a 4-byte boundary.
#pragma unroll
          for (int i = 0; i < kChunk / 4; ++i) {
            const int pr = (lane >> 4) + 2 * i;
            if (2 * pr < nj) cp_async4(sdst + pr * 4, ssrc + pr * 4);
          }
        }
      } else if constexpr (FMT >= 2) {
        // E8M0 bytes, 8 per row and chunk: lane copies 4 of row lane & 15
        // (group counts and slice starts are multiples of 4, so every copy
        // is whole and 4-byte aligned).
        const int half = lane >> 4;
        if (4 * half < nj)
          cp_async4(dst + S::kW + (lane & 15) * kChunk + half * 4, srow + i_c * kChunk + half * 4);
      }
      if (++i_c == nchunks) {
        i_c = 0;
        i_tile += gridDim.x;
        if (i_tile < p.tiles) set_rows(i_tile);
      }
    }
    asm volatile("cp.async.commit_group;" ::: "memory");
    i_slot = i_slot + 1 == S::kDepth ? 0 : i_slot + 1;
  };

  pdl_trigger();
#pragma unroll
  for (int i = 0; i < S::kDepth; ++i) issue();
  pdl_wait();  // activations come from the previous kernel

  // x row used by this thread's B fragment for n-tile t: rows past M repeat
  // the last row (their output columns are never written).
  const uint16_t* xbase[NT];
#pragma unroll
  for (int t = 0; t < NT; ++t)
    xbase[t] = p.x + int64_t(min(t * 8 + g, p.m - 1)) * p.k + int64_t(gb) * 32 + (S::kNibbles ? 8 * q : 4 * q);
  const int mi = lane >> 3, rr = lane & 7;  // ldmatrix: matrix mi, row rr
  int slot = 0, buf = 0;

  for (int y = blockIdx.x; y < p.tiles; y += gridDim.x) {
    float acc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;
    for (int c = 0; c < nchunks; ++c) {
      cp_async_wait<S::kDepth - 1>();
      __syncwarp();
      const uint8_t* st = ring + slot * S::kBytes;
      const int nj = min(kChunk, ng - c * kChunk);
      if constexpr (FMT == 0) {
        if (NT == 1 && nj == kChunk) {
          // Full chunk, two groups at a time: the pair's shared-memory and x
          // loads first, then its math with no branches.
#pragma unroll
          for (int hb = 0; hb < kChunk; hb += 2) {
            uint32_t f[4];
            uint4 xv[NT][2];
            ldsm_x4(f, st + piece_off<0>((mi & 1) * 8 + rr, hb + (mi >> 1)));
            const uint32_t slo = lds32(st + S::kW + g * (kChunk * 2) + hb * 2);
            const uint32_t shi = lds32(st + S::kW + (g + 8) * (kChunk * 2) + hb * 2);
#pragma unroll
            for (int t = 0; t < NT; ++t)
#pragma unroll
              for (int j = 0; j < 2; ++j) xv[t][j] = ldg16(xbase[t] + (c * kChunk + hb + j) * 32);
#pragma unroll
            for (int j = 0; j < 2; ++j) int4_group<NT>(acc, f[2 * j], f[2 * j + 1], slo, shi, j, xv, j);
          }
        } else {
#pragma unroll
          for (int j = 0; j < kChunk; j += 2) {
            if (j < nj) {  // nj is even
              uint32_t f[4];
              ldsm_x4(f, st + piece_off<0>((mi & 1) * 8 + rr, j + (mi >> 1)));
              const uint32_t slo = lds32(st + S::kW + g * (kChunk * 2) + j * 2);
              const uint32_t shi = lds32(st + S::kW + (g + 8) * (kChunk * 2) + j * 2);
#pragma unroll
              for (int jj = 0; jj < 2; ++jj) {
                uint4 xg[NT][1];
#pragma unroll
                for (int t = 0; t < NT; ++t) xg[t][0] = ldg16(xbase[t] + (c * kChunk + j + jj) * 32);
                int4_group<NT>(acc, f[2 * jj], f[2 * jj + 1], slo, shi, jj, xg, 0);
              }
            }
          }
        }
      } else if constexpr (FMT == 2) {
        // MXFP8: int8's layout (two 16 B halves per row and group, one k16
        // step each); each group's two MMAs go to a fresh fragment of values
        // times 2^-120, which is scaled by 2^120 and then by the group's
        // E8M0 scale, so every scale from 2^-126 to 2^127 is exact.
#pragma unroll
        for (int j = 0; j < kChunk; ++j) {
          if (j < nj) {
            const int gi = c * kChunk + j;
            uint32_t f[4];
            ldsm_x4(f, st + piece_off<2>((mi & 1) * 8 + rr, 2 * j + (mi >> 1)));
            const float sl = e8m0_scale(st[S::kW + g * kChunk + j], 0);
            const float sh = e8m0_scale(st[S::kW + (g + 8) * kChunk + j], 0);
            uint32_t a[2][4];
#pragma unroll
            for (int s2 = 0; s2 < 2; ++s2) {
              a[s2][0] = e4m3_pair02(f[2 * s2]);
              a[s2][1] = e4m3_pair02(f[2 * s2 + 1]);
              a[s2][2] = e4m3_pair13(f[2 * s2]);
              a[s2][3] = e4m3_pair13(f[2 * s2 + 1]);
            }
#pragma unroll
            for (int t = 0; t < NT; ++t) {
              float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
#pragma unroll
              for (int s2 = 0; s2 < 2; ++s2) {
                const uint2 xv = __ldg(reinterpret_cast<const uint2*>(xbase[t] + gi * 32 + 16 * s2));
                mma_bf16(d, a[s2][0], a[s2][1], a[s2][2], a[s2][3], prmt(xv.x, xv.y, 0x5410),
                         prmt(xv.x, xv.y, 0x7632));
              }
              acc[t][0] = fmaf(d[0] * 0x1p120f, sl, acc[t][0]);
              acc[t][1] = fmaf(d[1] * 0x1p120f, sl, acc[t][1]);
              acc[t][2] = fmaf(d[2] * 0x1p120f, sh, acc[t][2]);
              acc[t][3] = fmaf(d[3] * 0x1p120f, sh, acc[t][3]);
            }
          }
        }
      } else if constexpr (FMT == 3) {
        // MXFP4: int4's layout (thread (g, q) gets word q of a group: codes
        // 8q..8q+7); the pairs are adjacent codes, so the activations need
        // no permute.  Values come out doubled: the scale is 2^(e - 128).
#pragma unroll
        for (int j = 0; j < kChunk; j += 2) {
          if (j < nj) {  // nj is a multiple of 4
            uint32_t f[4];
            ldsm_x4(f, st + piece_off<3>((mi & 1) * 8 + rr, j + (mi >> 1)));
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
              const int gi = c * kChunk + j + jj;
              const float sl = e8m0_scale(st[S::kW + g * kChunk + j + jj], 1);
              const float sh = e8m0_scale(st[S::kW + (g + 8) * kChunk + j + jj], 1);
              uint32_t pl[4], ph[4];
              e2m1_pairs(f[2 * jj], pl);
              e2m1_pairs(f[2 * jj + 1], ph);
#pragma unroll
              for (int t = 0; t < NT; ++t) {
                const uint4 xv = ldg16(xbase[t] + gi * 32);
                float d[4] = {0.0f, 0.0f, 0.0f, 0.0f};
                mma_bf16(d, pl[0], ph[0], pl[1], ph[1], xv.x, xv.y);
                mma_bf16(d, pl[2], ph[2], pl[3], ph[3], xv.z, xv.w);
                acc[t][0] = fmaf(d[0], sl, acc[t][0]);
                acc[t][1] = fmaf(d[1], sl, acc[t][1]);
                acc[t][2] = fmaf(d[2], sh, acc[t][2]);
                acc[t][3] = fmaf(d[3], sh, acc[t][3]);
              }
            }
          }
        }
      } else {
#pragma unroll
        for (int j = 0; j < kChunk; ++j) {
          if (j < nj) {
            const int gi = c * kChunk + j;
            // int8: a group is 32 B per row = two 16 B halves, one k16 step each.
            uint32_t f[4];
            ldsm_x4(f, st + piece_off<1>((mi & 1) * 8 + rr, 2 * j + (mi >> 1)));
#pragma unroll
            for (int s2 = 0; s2 < 2; ++s2) {
              const uint32_t ul = f[2 * s2] ^ 0x80808080u, uh = f[2 * s2 + 1] ^ 0x80808080u;
              const uint32_t a0 = pack_bf16x2(int8_code(ul, 0), int8_code(ul, 2));
              const uint32_t a2 = pack_bf16x2(int8_code(ul, 1), int8_code(ul, 3));
              const uint32_t a1 = pack_bf16x2(int8_code(uh, 0), int8_code(uh, 2));
              const uint32_t a3 = pack_bf16x2(int8_code(uh, 1), int8_code(uh, 3));
#pragma unroll
              for (int t = 0; t < NT; ++t) {
                const uint2 xv = __ldg(reinterpret_cast<const uint2*>(xbase[t] + gi * 32 + 16 * s2));
                mma_bf16(acc[t], a0, a1, a2, a3, prmt(xv.x, xv.y, 0x5410), prmt(xv.x, xv.y, 0x7632));
              }
            }
          }
        }
      }
      __syncwarp();
      issue();  // refills the stage just read
      slot = slot + 1 == S::kDepth ? 0 : slot + 1;
    }
    finish_tile<FMT, NT, MODE, kRedBufs == 1, W>(p, tile_rows<MODE>(p, y), red[buf], acc, warp, g, q, tid);
    buf = kRedBufs == 1 ? 0 : buf ^ 1;
  }
  cp_async_wait<0>();
}

// Launch one x-row block with W warps per block: p holds everything but the
// K-slices and the grid.  scale16_ok: every job's int4 scale rows are 16-byte
// aligned.
template <int FMT, int NT, int MODE, int W>
int launch_w(Params p, bool scale16_ok, bool pdl, cudaStream_t st) {
  auto kern = gemv_mma_kernel<FMT, NT, MODE, W>;
  const size_t smem = W * warp_smem_bytes(FMT);
  // The shared-memory limit is a per-device setting: raise it on every
  // device that launches this instance.  Resident blocks per SM are the same
  // on every B200.
  static PerDeviceOnce configured;
  static std::atomic<int> resident{1};
  if (!configured.run([&] {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)) != cudaSuccess)
          return false;
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, W * 32, smem) != cudaSuccess || n < 1) {
          cudaGetLastError();
          n = 1;
        }
        resident.store(n, std::memory_order_relaxed);
        return true;
      }))
    return SB_INTERNAL;
  const int per_sm = resident.load(std::memory_order_relaxed);
  p.gpw = (p.groups + W - 1) / W;
  p.gpw += p.gpw & 1;  // even slice starts keep the bf16 scale pairs 4-byte aligned
  if (FMT >= 2) p.gpw = (p.gpw + 3) & ~3;  // E8M0 scales are copied 4 bytes (groups) at a time
  // Whole 8-group slices: each row's scales of a chunk are one aligned
  // 16-byte copy.
  p.scale16 = FMT == 0 && scale16_ok && p.groups % (8 * W) == 0 ? 1 : 0;
  // Persistent: at most one full wave of blocks, each walking tiles.
  const int slots = per_sm * kNumSMs;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(p.tiles < slots ? p.tiles : slots), 1, 1);
  cfg.blockDim = dim3(W * 32, 1, 1);
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

// Warps per block for an int4 launch of one n-tile.  Each warp walks its
// K-slice of one tile after another, so a launch takes about
// (tiles per block, rounded up) x (groups per slice + about four groups'
// worth of per-tile reduction and barrier) group steps: 8-warp blocks fit
// three per SM, 12-warp blocks two and 16-warp blocks one.  Few tiles with
// long K (o_proj and down_proj of a 7B layer: 256 tiles; most tensor-parallel
// shards) favour the wider blocks; the 7B gate/up (1376 tiles) measured
// slower with 12 warps (28.8 against 23.9 us cold) and keeps 8.  Every warp
// keeps at least two groups.  Ties keep the narrower block.
int choose_warps(int tiles, int groups) {
  int best = kWarps;
  long best_cost = -1;
  for (int w : {8, 12, 16}) {
    if (w > kWarps && groups < 2 * w) continue;
    const int blocks_per_sm = w == 8 ? 3 : w == 12 ? 2 : 1;
    const long slots = long(blocks_per_sm) * kNumSMs;
    int gpw = (groups + w - 1) / w;
    gpw += gpw & 1;
    const long cost = (tiles + slots - 1) / slots * (gpw + 4);
    if (best_cost < 0 || cost < best_cost) {
      best = w;
      best_cost = cost;
    }
  }
  return best;
}

template <int FMT, int NT, int MODE>
int launch_one(const Params& p, bool scale16_ok, bool pdl, cudaStream_t st) {
  if constexpr (FMT == 0 && NT == 1) {
    switch (choose_warps(p.tiles, p.groups)) {
      case 16: return launch_w<FMT, NT, MODE, 16>(p, scale16_ok, pdl, st);
      case 12: return launch_w<FMT, NT, MODE, 12>(p, scale16_ok, pdl, st);
      default: break;
    }
  }
  return launch_w<FMT, NT, MODE, kWarps>(p, scale16_ok, pdl, st);
}

template <int FMT, int NT>
int dispatch_mode(GemvMode mode, const Params& p, bool scale16_ok, bool pdl, cudaStream_t st) {
  switch (mode) {
    case GemvMode::Plain: return launch_one<FMT, NT, 0>(p, scale16_ok, pdl, st);
    case GemvMode::SwiGLU: return launch_one<FMT, NT, 1>(p, scale16_ok, pdl, st);
    case GemvMode::QkvRope: return launch_one<FMT, NT, 2>(p, scale16_ok, pdl, st);
  }
  return SB_INVALID_ARGUMENT;
}

// x rows per launch: n-tiles of 8 (1, 2, 4 or 8 of them).
template <int FMT>
int dispatch_nt(const Params& p, GemvMode mode, bool scale16_ok, bool pdl, cudaStream_t st) {
  if (p.m <= 8) return dispatch_mode<FMT, 1>(mode, p, scale16_ok, pdl, st);
  if (p.m <= 16) return dispatch_mode<FMT, 2>(mode, p, scale16_ok, pdl, st);
  if (p.m <= 32) return dispatch_mode<FMT, 4>(mode, p, scale16_ok, pdl, st);
  return dispatch_mode<FMT, 8>(mode, p, scale16_ok, pdl, st);
}

}  // namespace

bool gemv_mma_supported(const GemvMmaArgs& a) {
  const LinearBatch& b = a.lb;
  const bool mx = b.fmt == WFormat::MXFP8 || b.fmt == WFormat::MXFP4;
  if (b.fmt != WFormat::W4G32 && b.fmt != WFormat::W8PC && !mx) return false;
  if (b.k % 32 || b.m <= 0) return false;
  // MX scales are copied 4 groups at a time: whole multiples of 4 groups.
  if (mx && b.k % 128) return false;
  for (int j = 0; mx && j < b.njobs; ++j)
    if (reinterpret_cast<uintptr_t>(b.jobs[j].s) & 3) return false;
  // int4 scales are copied as 4-byte bf16 pairs: rows of an even number of
  // groups keep every pair aligned (an odd count goes to the CUDA-core GEMV).
  if (b.fmt == WFormat::W4G32 && (b.k / 32) % 2) return false;
  auto aligned = [](const void* q) { return (reinterpret_cast<uintptr_t>(q) & 15) == 0; };
  if (!aligned(b.x)) return false;
  for (int j = 0; j < b.njobs; ++j) {
    if (!aligned(b.jobs[j].w)) return false;
    if (b.fmt == WFormat::W4G32 && (reinterpret_cast<uintptr_t>(b.jobs[j].s) & 3)) return false;
  }
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
  const int fmt = b.fmt == WFormat::W4G32 ? 0 : b.fmt == WFormat::W8PC ? 1 : b.fmt == WFormat::MXFP8 ? 2 : 3;
  const int groups = b.k / 32;
  bool scale16_ok = fmt == 0;
  for (int j = 0; j < b.njobs && scale16_ok; ++j)
    scale16_ok = (reinterpret_cast<uintptr_t>(b.jobs[j].s) & 15) == 0 && (int64_t(groups) * 2) % 16 == 0;
  int rows = 0;
  switch (a.mode) {
    case GemvMode::Plain:
      for (int j = 0; j < b.njobs; ++j) rows += b.jobs[j].n;
      break;
    case GemvMode::SwiGLU: rows = 2 * b.jobs[0].n; break;
    case GemvMode::QkvRope: rows = b.jobs[0].n + b.jobs[1].n + b.jobs[2].n; break;
  }
  const int blocks = rows / kTileRows;

  for (int m0 = 0; m0 < b.m; m0 += kMaxRows) {
    Params p{};
    p.m = b.m - m0 < kMaxRows ? b.m - m0 : kMaxRows;
    p.x = b.x + int64_t(m0) * b.k;
    p.k = b.k;
    p.groups = groups;
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
    int rc;
    switch (fmt) {
      case 0: rc = dispatch_nt<0>(p, a.mode, scale16_ok, a.pdl, st); break;
      case 1: rc = dispatch_nt<1>(p, a.mode, scale16_ok, a.pdl, st); break;
      case 2: rc = dispatch_nt<2>(p, a.mode, false, a.pdl, st); break;
      default: rc = dispatch_nt<3>(p, a.mode, false, a.pdl, st); break;
    }
    if (rc) return rc;
  }
  return SB_OK;
}

}  // namespace sb
