// Decode GEMV (<= 32 rows of x per launch) for int4 group-32 and int8
// per-channel weights, with the fused epilogues of the decoder block: a
// TMA-fed weight stream split stream-K style over persistent CTAs.
//
//   y[m, n] = sum_k x[m, k] * deq(W)[n, k]        (then residual / SwiGLU /
//                                                   RoPE + KV append)
//
// Work.  The weight rows are cut into 128-row blocks (for a SwiGLU pair: 64
// gate rows over the 64 up rows of the same features) and K into chunks of
// 128 bytes per row (int4: 8 groups of 32 codes; int8: 4 groups).  A unit is
// one (block, chunk): 16 KB of codes.  The units, block-major, are split into
// one contiguous range per CTA, so every CTA streams the same number of bytes
// whatever the matrix shape.  A CTA whose range covers a block's whole K
// writes the block's outputs itself; a block shared by several CTAs is
// finished by the last of them to arrive: each writes its partial sums
// (128 rows x the x rows, f32) to a workspace slot and increments the block's
// counter; the one that completes the count sums every slot in K order (so the
// result does not depend on the arrival order), runs the epilogue and puts the
// counter back to zero for the next launch.  No CTA ever waits on another.
//
// Roles in a CTA (9 warps):
//   warp 8   producer: per unit one TMA load (128-byte swizzle, no
//            multicast) of the 128 x 128 B of codes (two 64-row loads for a
//            SwiGLU pair), for int4 the rows' bf16 scales of those groups
//            (a TMA box when the scale rows allow one, else cp.async), and
//            the chunk's x rows, into a D-deep ring that runs across the
//            CTA's units.  Weights are requested before the programmatic
//            dependency wait (they never depend on the previous kernel), x
//            only after it.
//   warps 0-7  16 weight rows each: ldmatrix of the swizzled codes, dequant
//            in registers, mma.sync m16n8k16 with f32 accumulators.  Each
//            unit's x fragments (the k order permuted to match the int4
//            pairs below), the int4 scales as f32 and, for int4, each group's
//            -136 * sum(x) are prepared by the 8 warps together one unit
//            ahead (warp w: group w), published by a named barrier.
//
// int4 dequantisation without a subtraction: one lop3 turns a code word's
// nibbles j and j + 4 into the bf16 pair (136 + c_j, 136 + c_j+4) (the sign
// bit flipped, the nibble in the mantissa of bf16 128).  The group's MMA
// starts from C = -136 * sum_k x[k] instead of zero, so its result is exactly
// sum_k c_k x[k]; each group's result is then scaled by its bf16 scale in
// f32, as the oracle's code * scale.  int8 codes convert exactly to bf16 and
// accumulate over all of K; the per-channel scale is applied in the epilogue.
//
// Every mbarrier wait is bounded; a wait that runs out records error word 4
// and the CTA winds down (the producer lets its copies in flight land first).
#include <cuda.h>

#include "k_gemv_mma.cuh"
#include "k_int4.cuh"

namespace sb {

namespace {

constexpr int kRows = 128;                 // weight rows per block
constexpr int kCons = 8;                   // consumer warps, 16 rows each
constexpr int kProducerWarp = kCons;       // warp 8
constexpr int kThreads = (kCons + 1) * 32;
constexpr int kCodeBytes = kRows * 128;    // 16 KB of codes per stage
constexpr int kPrepDepth = 2;
constexpr uint32_t kWaitLimit = 1u << 22;  // bounded mbarrier polls
constexpr uint32_t kOnes = 0x3F803F80u;    // bf16x2 (1, 1)
constexpr int kMaxRowsTma = 32;            // x rows per launch
constexpr int kMinUnits = 4;               // units per CTA at least (fewer partial sums on small matrices)

template <int FMT>
struct Fmt {
  static constexpr int kGroups = FMT == 0 ? 8 : 4;            // 32-code groups per stage
  static constexpr int kK = kGroups * 32;                      // k values per stage
  static constexpr int kScaleRaw = FMT == 0 ? kRows * 16 : 0;  // raw bf16 scales per stage
};

template <int FMT, int NT, int D>
struct Layout {
  static constexpr int kG = Fmt<FMT>::kGroups;
  static constexpr int kXRows = 8 * NT;                               // x rows of the launch, padded
  static constexpr int kXBytes = kXRows * Fmt<FMT>::kK * 2;           // the chunk's x, [row][k] bf16
  static constexpr int kXOff = kCodeBytes + Fmt<FMT>::kScaleRaw;
  static constexpr int kTmaStage = kXOff + kXBytes;                   // multiple of 1024
  static constexpr int kScaleF32 = FMT == 0 ? kRows * 8 * 4 : 0;      // [row][8 groups] f32
  static constexpr int kXf = kG * NT * 32 * 16;                       // B fragments [group][n-tile][lane]
  static constexpr int kCinit = FMT == 0 ? kG * NT * 4 * 8 : 0;       // [group][n-tile][q] float2
  static constexpr int kPrepStage = kScaleF32 + kXf + kCinit;
  static constexpr int kRing = D * kTmaStage;
  static constexpr int kBarOff = kRing + kPrepDepth * kPrepStage;
  static constexpr int kBarBytes = 2 * D * 8 + 16;
  static constexpr int kBytes = kBarOff + kBarBytes + 1024;  // + alignment slack
};

struct SkParams {
  CUtensorMap wmap[3];      // codes of each job: [rows, row bytes] u8, box 128 B x (128 or 64) rows
  CUtensorMap smap[3];      // int4 scales of each job: [rows, groups] bf16, box 8 x (128 or 64) rows
  CUtensorMap xmap;         // x: [m, k] bf16, box (k per stage) x (8 NT) rows; rows past m read as zero
  const uint16_t* x;        // [m, k] bf16
  int m, k, groups, chunks;
  int njobs;
  const void* s[3];         // int4: bf16 scales [n, groups]; int8: f32 [n]
  int n[3];
  uint16_t* y[3];
  const uint16_t* res[3];
  int jb[4];                // first block of each job; jb[njobs] = blocks
  int blocks;
  int scale_tma;            // int4: 1 when the scales come by TMA (smap valid), else cp.async
  int m_base;
  QkvExtra qkv;
  int* counters;            // [blocks], zero between launches
  float* partials;          // [2 * gridDim.x][kRows * 8 * NT]
  int* err;
};

__device__ __forceinline__ uint32_t su32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(su32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(su32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(su32(bar)) : "memory");
}

// cp.async completion of this thread's earlier copies arrives on `bar`
// (without adding to its expected count: the count includes it).
__device__ __forceinline__ void cp_async_arrive_noinc(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(su32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  const uint32_t a = su32(bar);
  for (uint32_t i = 0; i < kWaitLimit; ++i) {
    uint32_t done;
    asm volatile(
        "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}"
        : "=r"(done)
        : "r"(a), "r"(parity)
        : "memory");
    if (done) return true;
  }
  return false;
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(su32(bar))
      : "memory");
}

__device__ __forceinline__ void cp_async4(uint32_t dst, const void* gmem) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(dst), "l"(gmem) : "memory");
}

__device__ __forceinline__ void cp_async16s(uint32_t dst, const void* gmem) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(dst), "l"(gmem) : "memory");
}

__device__ __forceinline__ void ldsm_x4(uint32_t (&r)[4], uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
               : "r"(addr));
}

__device__ __forceinline__ uint4 lds128(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

__device__ __forceinline__ uint2 lds64(uint32_t addr) {
  uint2 v;
  asm volatile("ld.shared.v2.u32 {%0,%1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(addr));
  return v;
}

__device__ __forceinline__ float4 lds128f(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0,%1,%2,%3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

__device__ __forceinline__ float2 lds64f(uint32_t addr) {
  float2 v;
  asm volatile("ld.shared.v2.f32 {%0,%1}, [%2];" : "=f"(v.x), "=f"(v.y) : "r"(addr));
  return v;
}

// D = A * B + C with C given separately from D.
__device__ __forceinline__ void mma_c(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                      uint32_t b0, uint32_t b1, float c0, float c1, float c2, float c3) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%10,%11,%12,%13};"
      : "=f"(d[0]), "=f"(d[1]), "=f"(d[2]), "=f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "f"(c0), "f"(c1), "f"(c2), "f"(c3));
}

// Nibbles j and j + 4 of the code word u as the bf16 pair (136 + c_j,
// 136 + c_j+4): lop3 computes (a & 0x000F000F) ^ 0x43084308 (keep the two
// nibbles, flip their sign bits, set the exponent of bf16 128).  The right
// shift is a high multiply, which issues on the FMA pipe.
__device__ __forceinline__ uint32_t pair136(uint32_t u, int j) {
  uint32_t a = u, v;
  if (j) asm("mul.hi.u32 %0, %1, %2;" : "=r"(a) : "r"(u), "r"(1u << (32 - 4 * j)));
  asm("lop3.b32 %0, %1, %2, %3, 0x6A;" : "=r"(v) : "r"(a), "r"(0x000F000Fu), "r"(0x43084308u));
  return v;
}

// Shared-memory row of weight row (warp w, half h, pair row g) of a block.
// Rows g of half 0 and half 1 form an epilogue pair: the gate and up rows of
// one feature (SwiGLU), or the two rotate-half partners of one head (q/k/v).
template <int MODE>
__device__ __forceinline__ int smem_row(const SkParams& p, int w, int h, int g) {
  if constexpr (MODE == 0) return 16 * w + 8 * h + g;
  if constexpr (MODE == 1) return 64 * h + 8 * w + g;
  if (p.qkv.head_dim == 128) return 64 * h + 8 * w + g;
  return 64 * (w >> 2) + 32 * h + 8 * (w & 3) + g;  // head_dim 64: two heads per block
}

struct RowRef {
  int job, row;  // row < 0: no such row (past the matrix)
};

// The (job, matrix row) of shared-memory row r of block rb.
template <int MODE>
__device__ __forceinline__ RowRef block_row(const SkParams& p, int rb, int r) {
  if constexpr (MODE == 1) {
    const int j = r < 64 ? 0 : 1;
    const int row = rb * 64 + (r & 63);
    return {j, row < p.n[j] ? row : -1};
  }
  int j = 0;
  while (j + 1 < p.njobs && rb >= p.jb[j + 1]) ++j;
  const int row = (rb - p.jb[j]) * kRows + r;
  return {j, row < p.n[j] ? row : -1};
}

// The epilogue of one output pair: vlo / vhi are the finished dot products
// of rows lo and hi for x row m.
template <int FMT, int MODE>
__device__ __forceinline__ void pair_epilogue(const SkParams& p, RowRef lo, RowRef hi, int m, float vlo, float vhi) {
  if (FMT == 1) {
    if (lo.row >= 0) vlo *= static_cast<const float*>(p.s[lo.job])[lo.row];
    if (hi.row >= 0) vhi *= static_cast<const float*>(p.s[hi.job])[hi.row];
  }
  if constexpr (MODE == 0) {
    if (lo.row >= 0) {
      if (p.res[lo.job]) vlo += bf2f(p.res[lo.job][int64_t(m) * p.n[lo.job] + lo.row]);
      p.y[lo.job][int64_t(m) * p.n[lo.job] + lo.row] = f2bf(vlo);
    }
    if (hi.row >= 0) {
      if (p.res[hi.job]) vhi += bf2f(p.res[hi.job][int64_t(m) * p.n[hi.job] + hi.row]);
      p.y[hi.job][int64_t(m) * p.n[hi.job] + hi.row] = f2bf(vhi);
    }
  } else if constexpr (MODE == 1) {
    if (lo.row < 0) return;
    const float silu = vlo / (1.0f + expf(-vlo));
    p.y[0][int64_t(m) * p.n[0] + lo.row] = f2bf(silu * vhi);
  } else {
    if (lo.row < 0) return;
    const QkvExtra& e = p.qkv;
    const int hd = e.head_dim, half = hd / 2;
    const int jl = lo.job;
    const int head_in_job = lo.row / hd, i = lo.row % hd;  // i < half: the pair's first row
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

// A unit's (block, chunk), advanced one unit at a time.
struct Cursor {
  int rb, c;
  __device__ __forceinline__ void next(int chunks) {
    if (++c == chunks) {
      c = 0;
      ++rb;
    }
  }
};

// Stream-K bookkeeping: CTA i owns units [lo(i), lo(i + 1)).
__device__ __forceinline__ int64_t unit_lo(int64_t i, int64_t units, int64_t ctas) { return i * units / ctas; }
__device__ __forceinline__ int unit_owner(int64_t u, int64_t units, int64_t ctas) {
  return int(((u + 1) * ctas - 1) / units);
}

__device__ __forceinline__ void named_bar(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

template <int FMT, int NT, int MODE, int D>
__global__ void __launch_bounds__(kThreads, NT <= 2 ? 2 : 1) gemv_tma_kernel(const __grid_constant__ SkParams p) {
  using L = Layout<FMT, NT, D>;
  constexpr int G = L::kG;
  extern __shared__ uint8_t dsm_raw[];
  uint8_t* dsm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(dsm_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(dsm + L::kBarOff);
  uint64_t* empty = full + D;
  volatile int* flags = reinterpret_cast<volatile int*>(empty + D);  // [0] abort, [1] last arriver
  const uint32_t ring = su32(dsm);

  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int64_t units = int64_t(p.blocks) * p.chunks, ctas = gridDim.x;
  const int64_t u_lo = unit_lo(blockIdx.x, units, ctas), u_hi = unit_lo(blockIdx.x + 1, units, ctas);
  const int nunits = int(u_hi - u_lo);
  const Cursor first_unit{int(u_lo / p.chunks), int(u_lo % p.chunks)};
  // int4 scales by cp.async: one arrival per producer lane joins the TMA's.
  const bool scale_copies = FMT == 0 && !p.scale_tma;

  if (tid == 0) {
    for (int s = 0; s < D; ++s) {
      mbar_init(&full[s], scale_copies ? 1 + 32 : 1);
      mbar_init(&empty[s], kCons);
    }
    flags[0] = 0;
    flags[1] = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  pdl_trigger();

  auto abort = [&]() {
    flags[0] = 1;
    if (p.err) atomicExch(p.err, 4);
  };

  if (warp == kProducerWarp) {
    // ---- producer ------------------------------------------------------------
    if (lane == 0) {
      for (int i = 0; i < p.njobs; ++i) {
        asm volatile("prefetch.tensormap [%0];" ::"l"(&p.wmap[i]) : "memory");
        if (FMT == 0 && p.scale_tma) asm volatile("prefetch.tensormap [%0];" ::"l"(&p.smap[i]) : "memory");
      }
      asm volatile("prefetch.tensormap [%0];" ::"l"(&p.xmap) : "memory");
    }
    Cursor wcur = first_unit, xcur = first_unit;
    // Weights of stage j: codes by TMA and (int4) scales.
    auto issue_weights = [&](int j) {
      const int s = j % D;
      const int rb = wcur.rb, c = wcur.c;
      wcur.next(p.chunks);
      const uint32_t st = ring + s * L::kTmaStage;
      if (lane == 0) {
        const uint32_t sbytes = FMT == 0 && p.scale_tma ? uint32_t(Fmt<FMT>::kScaleRaw) : 0u;
        mbar_expect_tx(&full[s], kCodeBytes + sbytes + L::kXBytes);
        if constexpr (MODE == 1) {
          tma_load_2d(st, &p.wmap[0], &full[s], c * 128, rb * 64);
          tma_load_2d(st + 64 * 128, &p.wmap[1], &full[s], c * 128, rb * 64);
          if (sbytes) {
            tma_load_2d(st + kCodeBytes, &p.smap[0], &full[s], c * G, rb * 64);
            tma_load_2d(st + kCodeBytes + 64 * 16, &p.smap[1], &full[s], c * G, rb * 64);
          }
        } else {
          int jj = 0;
          while (jj + 1 < p.njobs && rb >= p.jb[jj + 1]) ++jj;
          tma_load_2d(st, &p.wmap[jj], &full[s], c * 128, (rb - p.jb[jj]) * kRows);
          if (sbytes) tma_load_2d(st + kCodeBytes, &p.smap[jj], &full[s], c * G, (rb - p.jb[jj]) * kRows);
        }
      }
      if (FMT == 0 && scale_copies) {
        // Scales of the chunk's groups for the block's 128 rows: lane l takes
        // rows l, l + 32, l + 64, l + 96.
        const int g0 = c * G, ng = min(G, p.groups - g0);
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int r = lane + 32 * i;
          const RowRef rr = block_row<MODE>(p, rb, r);
          if (rr.row < 0) continue;
          const uint8_t* src =
              static_cast<const uint8_t*>(p.s[rr.job]) + (int64_t(rr.row) * p.groups + g0) * 2;
          for (int pr = 0; 2 * pr < ng; ++pr) cp_async4(st + kCodeBytes + r * 16 + 4 * pr, src + 4 * pr);
        }
        cp_async_arrive_noinc(&full[s]);
      }
    };
    // x of stage j, which the previous kernel may still be writing: only
    // after the dependency wait.
    auto issue_x = [&](int j) {
      const int c = xcur.c;
      xcur.next(p.chunks);
      if (lane == 0) tma_load_2d(ring + (j % D) * L::kTmaStage + L::kXOff, &p.xmap, &full[j % D], c * Fmt<FMT>::kK, 0);
    };
    const int pro = min(D, nunits);
    for (int j = 0; j < pro; ++j) issue_weights(j);
    pdl_wait();
    for (int j = 0; j < pro; ++j) issue_x(j);
    int issued = pro;
    for (int j = pro; j < nunits; ++j) {
      const int s = j % D;
      if (!mbar_wait(&empty[s], ((j / D) - 1) & 1)) {
        abort();
        break;
      }
      if (flags[0]) break;
      issue_weights(j);
      issue_x(j);
      issued = j + 1;
    }
    if (scale_copies) asm volatile("cp.async.wait_all;" ::: "memory");
    // Let every copy this CTA requested land before it exits.
    if (lane == 0)
      for (int j = max(0, issued - D); j < issued; ++j) mbar_wait(&full[j % D], (j / D) & 1);
  } else {
    // ---- consumers -------------------------------------------------------------
    pdl_wait();
    const int w = warp, g = lane >> 2, q = lane & 3;
    const int mi = lane >> 3, rr = lane & 7;
    const int lrow = smem_row<MODE>(p, w, mi & 1, rr);  // this lane's ldmatrix row
    const uint32_t lrow_off = uint32_t(lrow) * 128, lkey = uint32_t(lrow & 7);
    const int row_lo = smem_row<MODE>(p, w, 0, g), row_hi = smem_row<MODE>(p, w, 1, g);

    // Preparation of unit j (cursor pc) into prep slot j % 2 by warp w: group
    // w's x fragments and bias, scale rows 16w..16w+15 as f32.
    auto prep = [&](int j, Cursor pc) {
      const int s = j % D;
      if (flags[0]) return;
      if (!mbar_wait(&full[s], (j / D) & 1)) {
        abort();
        return;
      }
      const uint32_t st = ring + s * L::kTmaStage;
      const uint32_t pst = ring + L::kRing + (j % kPrepDepth) * L::kPrepStage;
      const int g0 = pc.c * G;
      if constexpr (FMT == 0) {
        // f32 scales of rows 16w + lane / 2, groups 4 (lane & 1) .. + 3.
        const int r = 16 * w + (lane >> 1), e0 = 4 * (lane & 1);
        const bool ok = block_row<MODE>(p, pc.rb, r).row >= 0;
        const uint2 v = lds64(st + kCodeBytes + r * 16 + e0 * 2);
        const int ng = p.groups - g0;
        float4 f;
        f.x = ok && e0 + 0 < ng ? __uint_as_float(v.x << 16) : 0.0f;
        f.y = ok && e0 + 1 < ng ? __uint_as_float(v.x & 0xFFFF0000u) : 0.0f;
        f.z = ok && e0 + 2 < ng ? __uint_as_float(v.y << 16) : 0.0f;
        f.w = ok && e0 + 3 < ng ? __uint_as_float(v.y & 0xFFFF0000u) : 0.0f;
        asm volatile("st.shared.v4.f32 [%0], {%1,%2,%3,%4};" ::"r"(pst + r * 32 + e0 * 4), "f"(f.x), "f"(f.y),
                     "f"(f.z), "f"(f.w)
                     : "memory");
      }
      if (w < G) {
        const int gi = w;
        const uint32_t xs = st + L::kXOff;
#pragma unroll
        for (int t = 0; t < NT; ++t) {
          const uint32_t xrow = xs + uint32_t(8 * t + g) * (Fmt<FMT>::kK * 2);
          uint4 b;
          if constexpr (FMT == 0) {
            // k16 step 0 pairs (8q, 8q + 4) and (8q + 1, 8q + 5); step 1 the next two.
            const uint4 v = lds128(xrow + gi * 64 + q * 16);
            b = make_uint4(prmt(v.x, v.z, 0x5410), prmt(v.x, v.z, 0x7632), prmt(v.y, v.w, 0x5410),
                           prmt(v.y, v.w, 0x7632));
          } else {
            // int8: step s pairs (4q, 4q + 2) and (4q + 1, 4q + 3) of its 16 k.
            const uint2 v0 = lds64(xrow + gi * 64 + q * 8);
            const uint2 v1 = lds64(xrow + gi * 64 + 32 + q * 8);
            b = make_uint4(prmt(v0.x, v0.y, 0x5410), prmt(v0.x, v0.y, 0x7632), prmt(v1.x, v1.y, 0x5410),
                           prmt(v1.x, v1.y, 0x7632));
          }
          asm volatile("st.shared.v4.u32 [%0], {%1,%2,%3,%4};" ::"r"(pst + L::kScaleF32 +
                                                                     uint32_t((gi * NT + t) * 32 + lane) * 16),
                       "r"(b.x), "r"(b.y), "r"(b.z), "r"(b.w)
                       : "memory");
          if constexpr (FMT == 0) {
            // sum of the group's x over its 32 k for x rows 8t + 2q, 8t + 2q + 1.
            float d[4];
            mma_c(d, kOnes, kOnes, kOnes, kOnes, b.x, b.y, 0.0f, 0.0f, 0.0f, 0.0f);
            mma_c(d, kOnes, kOnes, kOnes, kOnes, b.z, b.w, d[0], d[1], d[2], d[3]);
            if (g == 0)
              asm volatile("st.shared.v2.f32 [%0], {%1,%2};" ::"r"(pst + L::kScaleF32 + L::kXf +
                                                                   uint32_t((gi * NT + t) * 4 + q) * 8),
                           "f"(-136.0f * d[0]), "f"(-136.0f * d[1])
                           : "memory");
          }
        }
      }
    };

    float acc[NT][4];
#pragma unroll
    for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;
    int seg_c0 = first_unit.c;
    Cursor cur = first_unit, nxt = first_unit;
    prep(0, cur);
    nxt.next(p.chunks);
    named_bar(1, kCons * 32);
    // Every consumer warp walks every unit and reaches every barrier, also
    // after a wait has run out (it then skips the waits and the math), so no
    // warp is left at a barrier the others never reach.
    for (int j = 0; j < nunits; ++j, cur = nxt, nxt.next(p.chunks)) {
      const int s = j % D, ps = j % kPrepDepth;
      const int rb = cur.rb, c = cur.c;
      if (!flags[0]) {
        const uint32_t codes = ring + s * L::kTmaStage + lrow_off;
        const uint32_t pst = ring + L::kRing + ps * L::kPrepStage;
        const uint32_t xf = pst + L::kScaleF32 + uint32_t(lane) * 16;
        if constexpr (FMT == 0) {
          const uint32_t ci = pst + L::kScaleF32 + L::kXf + uint32_t(q) * 8;
          const float4 sl0 = lds128f(pst + row_lo * 32), sl1 = lds128f(pst + row_lo * 32 + 16);
          const float4 sh0 = lds128f(pst + row_hi * 32), sh1 = lds128f(pst + row_hi * 32 + 16);
          const float sl[8] = {sl0.x, sl0.y, sl0.z, sl0.w, sl1.x, sl1.y, sl1.z, sl1.w};
          const float sh[8] = {sh0.x, sh0.y, sh0.z, sh0.w, sh1.x, sh1.y, sh1.z, sh1.w};
#pragma unroll
          for (int hb = 0; hb < G; hb += 2) {
            uint32_t f[4];
            ldsm_x4(f, codes + ((uint32_t(hb + (mi >> 1)) ^ lkey) << 4));
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
              const int gi = hb + jj;
              const uint32_t ul = f[2 * jj], uh = f[2 * jj + 1];
              const uint32_t p0 = pair136(ul, 0), p1 = pair136(ul, 1), p2 = pair136(ul, 2), p3 = pair136(ul, 3);
              const uint32_t h0 = pair136(uh, 0), h1 = pair136(uh, 1), h2 = pair136(uh, 2), h3 = pair136(uh, 3);
#pragma unroll
              for (int t = 0; t < NT; ++t) {
                const uint4 b = lds128(xf + uint32_t(gi * NT + t) * 512);
                const float2 c2 = lds64f(ci + uint32_t(gi * NT + t) * 32);
                float d[4];
                mma_c(d, p0, h0, p1, h1, b.x, b.y, c2.x, c2.y, c2.x, c2.y);
                mma_c(d, p2, h2, p3, h3, b.z, b.w, d[0], d[1], d[2], d[3]);
                acc[t][0] = fmaf(d[0], sl[gi], acc[t][0]);
                acc[t][1] = fmaf(d[1], sl[gi], acc[t][1]);
                acc[t][2] = fmaf(d[2], sh[gi], acc[t][2]);
                acc[t][3] = fmaf(d[3], sh[gi], acc[t][3]);
              }
            }
          }
        } else {
#pragma unroll
          for (int gi = 0; gi < G; ++gi) {
            uint32_t f[4];
            ldsm_x4(f, codes + ((uint32_t(2 * gi + (mi >> 1)) ^ lkey) << 4));
#pragma unroll
            for (int s2 = 0; s2 < 2; ++s2) {
              const uint32_t ul = f[2 * s2] ^ 0x80808080u, uh = f[2 * s2 + 1] ^ 0x80808080u;
              const uint32_t a0 = pack_bf16x2(int8_code(ul, 0), int8_code(ul, 2));
              const uint32_t a2 = pack_bf16x2(int8_code(ul, 1), int8_code(ul, 3));
              const uint32_t a1 = pack_bf16x2(int8_code(uh, 0), int8_code(uh, 2));
              const uint32_t a3 = pack_bf16x2(int8_code(uh, 1), int8_code(uh, 3));
#pragma unroll
              for (int t = 0; t < NT; ++t) {
                const uint4 b = lds128(xf + uint32_t(gi * NT + t) * 512);
                const uint32_t b0 = s2 ? b.z : b.x, b1 = s2 ? b.w : b.y;
                mma_c(acc[t], a0, a1, a2, a3, b0, b1, acc[t][0], acc[t][1], acc[t][2], acc[t][3]);
              }
            }
          }
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);  // the codes of unit j are read
      if (j + 1 < nunits) prep(j + 1, nxt);
      // Publishes unit j + 1's preparation; every warp is done with slot j % 2.
      named_bar(1, kCons * 32);
      // ---- end of a block's segment: write the outputs or a partial ---------
      if (c + 1 < p.chunks && j + 1 < nunits) continue;
      const bool whole = seg_c0 == 0 && c + 1 == p.chunks;
      bool finish = whole && !flags[0];
      if (!whole) {
        const int64_t bu0 = int64_t(rb) * p.chunks;
        const int first = unit_owner(bu0, units, ctas), last = unit_owner(bu0 + p.chunks - 1, units, ctas);
        auto slot = [&](int cta) {
          const int rbf = int(unit_lo(cta, units, ctas) / p.chunks);
          return int64_t(2 * cta + (rb == rbf ? 0 : 1)) * (kRows * 8 * NT);
        };
        float4* mine = reinterpret_cast<float4*>(p.partials + slot(blockIdx.x)) + (w * 32 + lane) * NT;
#pragma unroll
        for (int t = 0; t < NT; ++t) __stcg(mine + t, make_float4(acc[t][0], acc[t][1], acc[t][2], acc[t][3]));
        // The barrier orders every thread's partial before thread 0's release
        // (a gpu-scope fence, then the counter); the last arriver acquires the
        // same way before its threads read the other partials.
        named_bar(1, kCons * 32);
        if (tid == 0) {
          int last_one = 0;
          if (!flags[0]) {
            __threadfence();
            last_one = atomicAdd(p.counters + rb, 1) == last - first;
            if (last_one) __threadfence();
          }
          flags[1] = last_one;
        }
        named_bar(1, kCons * 32);
        finish = flags[1] != 0;
        if (finish) {
          float sum[NT][4];
#pragma unroll
          for (int t = 0; t < NT; ++t) sum[t][0] = sum[t][1] = sum[t][2] = sum[t][3] = 0.0f;
          for (int cta = first; cta <= last; ++cta) {
            float v[NT][4];
            if (cta == int(blockIdx.x)) {
#pragma unroll
              for (int t = 0; t < NT; ++t) v[t][0] = acc[t][0], v[t][1] = acc[t][1], v[t][2] = acc[t][2], v[t][3] = acc[t][3];
            } else {
              const float4* other = reinterpret_cast<const float4*>(p.partials + slot(cta)) + (w * 32 + lane) * NT;
#pragma unroll
              for (int t = 0; t < NT; ++t) {
                const float4 o = __ldcg(other + t);
                v[t][0] = o.x, v[t][1] = o.y, v[t][2] = o.z, v[t][3] = o.w;
              }
            }
#pragma unroll
            for (int t = 0; t < NT; ++t)
#pragma unroll
              for (int e = 0; e < 4; ++e) sum[t][e] += v[t][e];
          }
#pragma unroll
          for (int t = 0; t < NT; ++t)
#pragma unroll
            for (int e = 0; e < 4; ++e) acc[t][e] = sum[t][e];
          if (tid == 0) p.counters[rb] = 0;  // ready for the next launch
        }
      }
      if (finish) {
        const RowRef lo = block_row<MODE>(p, rb, row_lo), hi = block_row<MODE>(p, rb, row_hi);
#pragma unroll
        for (int t = 0; t < NT; ++t)
#pragma unroll
          for (int e = 0; e < 2; ++e) {
            const int m = 8 * t + 2 * q + e;
            if (m < p.m) pair_epilogue<FMT, MODE>(p, lo, hi, m, acc[t][e], acc[t][2 + e]);
          }
      }
#pragma unroll
      for (int t = 0; t < NT; ++t) acc[t][0] = acc[t][1] = acc[t][2] = acc[t][3] = 0.0f;
      seg_c0 = 0;
    }
  }
  __syncthreads();
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

// A 2-D tensor [rows, inner] of elements of `type` (`esize` bytes), box
// box_inner x box_rows; elements past either end read as zero.
bool make_map(CUtensorMap* m, CUtensorMapDataType type, uint32_t esize, const void* base, uint64_t inner,
              uint64_t rows, uint32_t box_inner, uint32_t box_rows, CUtensorMapSwizzle swz) {
  EncodeTiled enc = encode_fn();
  if (!enc) return false;
  const cuuint64_t dims[2] = {inner, rows};
  const cuuint64_t strides[1] = {inner * esize};
  const cuuint32_t box[2] = {box_inner, box_rows};
  const cuuint32_t estr[2] = {1, 1};
  return enc(m, type, 2, const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
             CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

template <int NT>
constexpr int depth_for() {
  // Weight stages in flight: as many as shared memory allows at two CTAs per
  // SM (up to 16 x rows) or one (17 to 32).
  return NT == 1 ? 4 : NT == 2 ? 3 : 4;
}

// Blocks of 128 rows (SwiGLU: 64 feature pairs) of a launch.
int block_count(GemvMode mode, const int* n, int njobs, int* jb) {
  if (mode == GemvMode::SwiGLU) {
    jb[0] = 0;
    jb[1] = (n[0] + 63) / 64;
    return jb[1];
  }
  int total = 0;
  for (int j = 0; j < njobs; ++j) {
    jb[j] = total;
    total += (n[j] + kRows - 1) / kRows;
  }
  jb[njobs] = total;
  return total;
}

int nt_of(int m) { return m <= 8 ? 1 : m <= 16 ? 2 : 4; }

int ctas_per_sm(int nt) { return nt <= 2 ? 2 : 1; }

struct Occupancy {
  PerDeviceOnce once;
  int per_sm = 1;
};

template <int FMT, int NT, int MODE>
int launch_t(const SkParams& p0, bool pdl, cudaStream_t st) {
  constexpr int D = depth_for<NT>();
  using L = Layout<FMT, NT, D>;
  auto kern = gemv_tma_kernel<FMT, NT, MODE, D>;
  static Occupancy occ;
  if (!occ.once.run([&] {
        if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kBytes) != cudaSuccess)
          return false;
        int n = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kThreads, L::kBytes) != cudaSuccess || n < 1)
          n = 1;
        occ.per_sm = n;
        return true;
      }))
    return SB_INTERNAL;
  SkParams p = p0;
  const int64_t units = int64_t(p.blocks) * p.chunks;
  // The partial slots are sized for ctas_per_sm(NT) CTAs per SM.
  const int per_sm = occ.per_sm < ctas_per_sm(NT) ? occ.per_sm : ctas_per_sm(NT);
  const int64_t slots = int64_t(per_sm) * kNumSMs;
  const int64_t want = (units + kMinUnits - 1) / kMinUnits;
  const int grid = int(want < slots ? want : slots);
  if (grid <= 0) return SB_OK;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid), 1, 1);
  cfg.blockDim = dim3(kThreads, 1, 1);
  cfg.dynamicSmemBytes = L::kBytes;
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
int dispatch_mode(GemvMode mode, const SkParams& p, bool pdl, cudaStream_t st) {
  switch (mode) {
    case GemvMode::Plain: return launch_t<FMT, NT, 0>(p, pdl, st);
    case GemvMode::SwiGLU: return launch_t<FMT, NT, 1>(p, pdl, st);
    case GemvMode::QkvRope: return launch_t<FMT, NT, 2>(p, pdl, st);
  }
  return SB_INVALID_ARGUMENT;
}

template <int FMT>
int dispatch_nt(const SkParams& p, GemvMode mode, bool pdl, cudaStream_t st) {
  switch (nt_of(p.m)) {
    case 1: return dispatch_mode<FMT, 1>(mode, p, pdl, st);
    case 2: return dispatch_mode<FMT, 2>(mode, p, pdl, st);
    default: return dispatch_mode<FMT, 4>(mode, p, pdl, st);
  }
}

}  // namespace

bool gemv_tma_supported(const GemvMmaArgs& a) {
  const LinearBatch& b = a.lb;
  if (b.fmt != WFormat::W4G32 && b.fmt != WFormat::W8PC) return false;
  // Up to 32 x rows per launch (more rows stay on the register-staged GEMV).
  if (b.k % 32 || b.m <= 0 || b.m > kMaxRowsTma || b.k <= 0) return false;
  const int groups = b.k / 32;
  if (b.fmt == WFormat::W4G32 && groups % 2) return false;  // scales copied as 4-byte bf16 pairs
  auto al = [](const void* q, uintptr_t n) { return (reinterpret_cast<uintptr_t>(q) & (n - 1)) == 0; };
  if (!al(b.x, 16)) return false;
  for (int j = 0; j < b.njobs; ++j) {
    if (!b.jobs[j].w || !al(b.jobs[j].w, 16) || b.jobs[j].n <= 0) return false;
    if (b.fmt == WFormat::W4G32 && !al(b.jobs[j].s, 4)) return false;
  }
  if (!encode_fn()) return false;
  switch (a.mode) {
    case GemvMode::Plain:
      return b.epi != Epilogue::SwiGLU && b.njobs >= 1 && b.njobs <= 3;
    case GemvMode::SwiGLU:
      return b.njobs == 2 && b.jobs[0].n == b.jobs[1].n;
    case GemvMode::QkvRope: {
      const QkvExtra& e = a.qkv;
      if (b.njobs != 3 || (e.head_dim != 64 && e.head_dim != 128)) return false;
      return b.jobs[0].n == e.hq * e.head_dim && b.jobs[1].n == e.hkv * e.head_dim &&
             b.jobs[2].n == e.hkv * e.head_dim && e.tokens_per_seq > 0;
    }
  }
  return false;
}

int gemv_tma_counters(GemvMode mode, const int* n, int njobs) {
  int jb[4];
  return block_count(mode, n, njobs, jb);
}

uint64_t gemv_tma_partial_bytes(int m) {
  const int nt = nt_of(m < kMaxRowsTma ? m : kMaxRowsTma);
  return uint64_t(2) * ctas_per_sm(nt) * kNumSMs * kRows * 8 * nt * sizeof(float);
}

int launch_gemv_tma(const GemvMmaArgs& a, int* counters, int counter_capacity, float* partials,
                    uint64_t partial_bytes, int* err, cudaStream_t st) {
  if (!gemv_tma_supported(a)) return SB_INVALID_ARGUMENT;
  const LinearBatch& b = a.lb;
  SkParams p{};
  int ns[3] = {0, 0, 0};
  for (int j = 0; j < b.njobs; ++j) ns[j] = b.jobs[j].n;
  p.blocks = block_count(a.mode, ns, b.njobs, p.jb);
  if (p.blocks > counter_capacity || !counters || !partials) return SB_INVALID_ARGUMENT;
  const int fmt = b.fmt == WFormat::W4G32 ? 0 : 1;
  p.k = b.k;
  p.groups = b.k / 32;
  p.chunks = fmt == 0 ? (p.groups + 7) / 8 : (p.groups + 3) / 4;
  p.njobs = b.njobs;
  p.counters = counters;
  p.partials = partials;
  p.err = err;
  p.qkv = a.qkv;
  const uint64_t row_bytes = fmt == 0 ? uint64_t(b.k) / 2 : uint64_t(b.k);
  const uint32_t box_rows = a.mode == GemvMode::SwiGLU ? 64 : kRows;
  // int4 scales by TMA when every scale row starts on a 16-byte boundary.
  p.scale_tma = fmt == 0 && (p.groups * 2) % 16 == 0 ? 1 : 0;
  for (int j = 0; j < b.njobs; ++j) {
    if (!make_map(&p.wmap[j], CU_TENSOR_MAP_DATA_TYPE_UINT8, 1, b.jobs[j].w, row_bytes, uint64_t(b.jobs[j].n), 128,
                  box_rows, CU_TENSOR_MAP_SWIZZLE_128B))
      return SB_INTERNAL;
    p.s[j] = b.jobs[j].s;
    p.n[j] = b.jobs[j].n;
    if (p.scale_tma && (reinterpret_cast<uintptr_t>(b.jobs[j].s) & 15)) p.scale_tma = 0;
  }
  if (p.scale_tma)
    for (int j = 0; j < b.njobs; ++j)
      if (!make_map(&p.smap[j], CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, b.jobs[j].s, uint64_t(p.groups),
                    uint64_t(b.jobs[j].n), 8, box_rows, CU_TENSOR_MAP_SWIZZLE_NONE))
        return SB_INTERNAL;
  for (int m0 = 0; m0 < b.m; m0 += kMaxRowsTma) {
    p.m = b.m - m0 < kMaxRowsTma ? b.m - m0 : kMaxRowsTma;
    if (gemv_tma_partial_bytes(p.m) > partial_bytes) return SB_INVALID_ARGUMENT;
    p.x = b.x + int64_t(m0) * b.k;
    p.m_base = m0;
    if (!make_map(&p.xmap, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, p.x, uint64_t(b.k), uint64_t(p.m),
                  fmt == 0 ? 256 : 128, uint32_t(8 * nt_of(p.m)), CU_TENSOR_MAP_SWIZZLE_NONE))
      return SB_INTERNAL;
    for (int j = 0; j < b.njobs; ++j) {
      const LinearJob& J = b.jobs[j];
      p.y[j] = J.y ? J.y + int64_t(m0) * J.ldy : nullptr;
      p.res[j] = J.residual ? J.residual + int64_t(m0) * J.ldr : nullptr;
    }
    if (a.mode == GemvMode::QkvRope) {
      const QkvExtra& e = a.qkv;
      p.qkv.pos = e.pos + m0;
      p.qkv.q_out = e.q_out + int64_t(m0) * e.hq * e.head_dim;
      p.qkv.k_out = e.k_out ? e.k_out + int64_t(m0) * e.hkv * e.head_dim : nullptr;
      p.qkv.v_out = e.v_out ? e.v_out + int64_t(m0) * e.hkv * e.head_dim : nullptr;
    }
    const int rc = fmt == 0 ? dispatch_nt<0>(p, a.mode, a.pdl, st) : dispatch_nt<1>(p, a.mode, a.pdl, st);
    if (rc) return rc;
  }
  return SB_OK;
}

}  // namespace sb
