// TMA-pipelined fused dequant-GEMV for the INT formats (N <= 16 tokens).
//
// CTA = 4 consumer warps + 1 producer warp.  The producer streams
// (64*TR)-row x S-group tiles of packed codes with 2-D TMA copies, the
// matching x' records with 1-D bulk copies, and (with its other lanes) the
// tiles' fp16 scales and zero points into a 2-4 stage shared-memory ring
// guarded by mbarriers; the weights of the first stages are requested before
// the kernel waits for the x-prep grid (programmatic dependent launch), so
// weight streaming overlaps the preceding kernel.  Consumers never touch
// global memory until they write y: they read their rows' words from shared
// memory (128B-swizzled tiles, row order permuted so the reads are
// bank-conflict free) with 32-bit shared addresses, keep a few registers per
// row from which every code pair is one AND (codes already below mantissa
// bit 10 are not shifted; the per-position power of two lives in x'), and
// multiply on the tensor cores (mma.sync m16n8k16, register A) for TR
// independent 16-row tiles per warp.
//
// Codes become exact subnormal fp16 values  h = q 2^(p-24)  and x' was scaled
// by 2^(14-p-E), so  sum h B = 2^-10 sum q x'/2^E  with no bias term.  Per
// 128-column group:   sum w x' = s 2^E Q + m Sx,   Q = sum q x'/2^E.
// Work is split stream-K style: the (row block, stage) units are dealt out
// evenly to the CTAs; row blocks split between CTAs are combined through
// per-warp partial slots and arrival counters in chunk order (deterministic).
// Every wait is bounded (2 s, %globaltimer); on expiry the kernel records
// PF_ERR_TIMEOUT in the workspace status word and returns.
#include <cuda.h>
#include <cudaTypedefs.h>

#include <mutex>

#include "common.cuh"
#include "gemv.cuh"

namespace pfb {

namespace {

constexpr int kCWarps = 8;                     // consumer warps per CTA
constexpr int kThreadsT = (kCWarps + 1) * 32;  // + 1 producer warp
constexpr int kMaxCtasPerSm = 4;
constexpr unsigned long long kWaitNs = 2000000000ull;

template <int FMT>
struct TmaFmt;
template <>
struct TmaFmt<PF_FMT_INT4_G128> {
  static constexpr int S = 2, WPG = 16;
  static constexpr bool SW128 = true;
};
template <>
struct TmaFmt<PF_FMT_INT4> : TmaFmt<PF_FMT_INT4_G128> {};
template <>
struct TmaFmt<PF_FMT_INT2_G128> {
  static constexpr int S = 4, WPG = 8;
  static constexpr bool SW128 = true;
};
template <>
struct TmaFmt<PF_FMT_INT2> : TmaFmt<PF_FMT_INT2_G128> {};
template <>
struct TmaFmt<PF_FMT_INT3_G128> {
  static constexpr int S = 4, WPG = 13;
  static constexpr bool SW128 = false;
};

constexpr bool is_int4(int f) { return f == PF_FMT_INT4_G128 || f == PF_FMT_INT4; }
constexpr bool is_int2(int f) { return f == PF_FMT_INT2_G128 || f == PF_FMT_INT2; }

// Box row of quad-row rq: under the 128B swizzle a warp's smem reads are
// split into 8-lane (128-bit) or 16-lane (64-bit) phases; these orders put
// rows whose swizzle masks differ in the right bits into one phase.
template <int FMT>
__device__ __forceinline__ int row_perm(int rq) {
  if constexpr (is_int4(FMT))
    return ((rq & 1) << 2) | (rq >> 1);
  else if constexpr (is_int2(FMT))
    return ((rq & 3) << 1) | (rq >> 2);
  else
    return rq;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}
__device__ __forceinline__ uint32_t lds32(uint32_t a) {
  uint32_t v;
  asm volatile("ld.shared.b32 %0, [%1];" : "=r"(v) : "r"(a));
  return v;
}
__device__ __forceinline__ uint2 lds64(uint32_t a) {
  uint2 v;
  asm volatile("ld.shared.v2.b32 {%0, %1}, [%2];" : "=r"(v.x), "=r"(v.y) : "r"(a));
  return v;
}
__device__ __forceinline__ uint4 lds128(uint32_t a) {
  uint4 v;
  asm volatile("ld.shared.v4.b32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(a));
  return v;
}
__device__ __forceinline__ float4 lds128f(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
  return v;
}

__device__ __forceinline__ unsigned long long now_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity) {
  unsigned long long t0 = 0;
  for (unsigned it = 0;; ++it) {
    uint32_t done;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if ((it & 63) == 63) {
      unsigned long long t = now_ns();
      if (t0 == 0)
        t0 = t;
      else if (t - t0 > kWaitNs)
        return false;
    }
  }
}

__device__ __forceinline__ void mbar_expect(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes) : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
__device__ __forceinline__ void tma_2d(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
__device__ __forceinline__ void bulk_1d(uint32_t dst, const void* src, uint32_t bytes, uint32_t bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(dst),
               "l"(src), "r"(bytes), "r"(bar)
               : "memory");
}
__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---- per-row decode state: the few registers from which every code pair of
// a group is one AND (codes land as exact subnormal fp16 q * 2^(p-24)).
template <int FMT>
struct RowCodes;

template <>
struct RowCodes<PF_FMT_INT4_G128> {
  uint32_t w[4], v[4];
  __device__ __forceinline__ void load(uint32_t addr_j) {  // 16 bytes of the row's group
    const uint4 q = lds128(addr_j);
    w[0] = q.x; w[1] = q.y; w[2] = q.z; w[3] = q.w;
#pragma unroll
    for (int t = 0; t < 4; ++t) v[t] = w[t] >> 8;
  }
  // half2 i (frag_cols2): word i/4; sub 0,1 from w, 2,3 from w >> 8
  __device__ __forceinline__ uint32_t h(int i) const {
    const int t = i >> 2, sub = i & 3;
    const uint32_t src = sub < 2 ? w[t] : v[t];
    return src & ((sub & 1) ? 0x00F000F0u : 0x000F000Fu);
  }
};
template <>
struct RowCodes<PF_FMT_INT4> : RowCodes<PF_FMT_INT4_G128> {};

template <>
struct RowCodes<PF_FMT_INT2_G128> {
  uint32_t w[2], v[2];
  __device__ __forceinline__ void load(uint32_t addr_j) {
    const uint2 q = lds64(addr_j);
    w[0] = q.x; w[1] = q.y;
    v[0] = w[0] >> 10;
    v[1] = w[1] >> 10;
  }
  __device__ __forceinline__ uint32_t h(int i) const {
    const int t = i >> 3, sub = i & 7;
    return sub < 5 ? (w[t] & (0x00030003u << (2 * sub))) : (v[t] & (0x00030003u << (2 * (sub - 5))));
  }
};
template <>
struct RowCodes<PF_FMT_INT2> : RowCodes<PF_FMT_INT2_G128> {};

template <>
struct RowCodes<PF_FMT_INT3_G128> {
  uint32_t g[3], v[3], h15;
  __device__ __forceinline__ void load3(uint32_t a0, uint32_t a12, int c) {  // words c, c+4, c+8 and 12
    uint32_t w[3];
    w[0] = lds32(a0);
    w[1] = lds32(a0 + 16);
    w[2] = lds32(a0 + 32);
    const uint32_t w12 = lds32(a12);
#pragma unroll
    for (int t = 0; t < 3; ++t) {
      g[t] = (w[t] & 0x0000FFFFu) | ((w[t] << 1) & 0xFFFF0000u);
      v[t] = g[t] >> 9;
    }
    const uint32_t t12 = w12 >> (6 * c);
    h15 = (t12 & 7u) | ((t12 << 13) & 0x00070000u);
  }
  __device__ __forceinline__ uint32_t h(int i) const {
    if (i == 15) return h15;
    const int t = i / 5, sub = i % 5;
    switch (sub) {
      case 0: return g[t] & 0x00070007u;
      case 1: return g[t] & 0x00380038u;
      case 2: return g[t] & 0x01C001C0u;
      case 3: return v[t] & 0x00070007u;
      default: return v[t] & 0x00380038u;
    }
  }
};

__device__ __forceinline__ long long cta_of(long long u, long long U, long long P) {
  return ((u + 1) * P + U - 1) / U - 1;
}

// Compile-time layout of one pipeline stage.
template <int FMT, int NT, int LP, int TR, int SMODE>
struct Stage {
  static constexpr int S = TmaFmt<FMT>::S;
  static constexpr int kRowsBlk = 16 * kCWarps * TR;
  static constexpr uint32_t W = kRowsBlk * S * TmaFmt<FMT>::WPG * 4;
  static constexpr uint32_t R = NT * 8 * LP * 8 + 64 * NT;  // x' record per group
  static constexpr uint32_t X = S * R;
  static constexpr uint32_t SC = SMODE == kScaleGroup ? kRowsBlk * S * 4 : (SMODE == kScaleRow ? kRowsBlk * 4 : 0);
  static constexpr uint32_t XOFF = W;
  static constexpr uint32_t SOFF = (XOFF + X + 127u) & ~127u;
  static constexpr uint32_t BYTES = ((SOFF + SC + 1023u) & ~1023u);
  static constexpr int NS = BYTES * 4 <= 112 * 1024 ? 4 : (BYTES * 3 <= 112 * 1024 ? 3 : 2);
  static constexpr size_t SMEM = 1024 + (size_t)NS * BYTES + 2 * NS * 8;
};

template <int FMT, int NT, int LP, int TR, int SMODE>
__global__ void __launch_bounds__(kThreadsT, 2)
    gemv_tma_kernel(const __grid_constant__ CUtensorMap tmap, const TmaArgs a) {
  using F = TmaFmt<FMT>;
  using L = Stage<FMT, NT, LP, TR, SMODE>;
  constexpr int S = F::S;
  constexpr int NS = L::NS;
  constexpr int kRowsBlk = L::kRowsBlk;
  constexpr int kOffset = IntFmt<FMT>::kOffset;

  asm volatile("griddepcontrol.launch_dependents;");

  extern __shared__ unsigned char smem_raw[];
  const uint32_t base = (smem_u32(smem_raw) + 1023u) & ~1023u;
  const uint32_t full0 = base + NS * L::BYTES, empty0 = full0 + 8 * NS;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < NS; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(full0 + 8 * s), "r"(33));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(empty0 + 8 * s), "r"(kCWarps));
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  const long long U = a.n_units, P = gridDim.x, cta = blockIdx.x;
  const int u0 = (int)(cta * U / P), u1 = (int)((cta + 1) * U / P);
  const int nunits = u1 - u0;
  const int spb = a.spb, M = a.M, G = a.G, N = a.N;

  if (warp == kCWarps) {
    // ------------------------------------------------------------ producer
    // lane 0 issues the copies; all lanes stage the units' scales in smem
    int rb = u0 / spb, st = u0 % spb;
    const int first = nunits < NS ? nunits : NS;
    for (int it = 0; it < nunits; ++it) {
      const int slot = it % NS;
      const uint32_t sb = base + slot * L::BYTES;
      if (it >= NS) {
        bool ok = true;
        if (lane == 0) ok = mbar_wait(empty0 + 8 * slot, ((it / NS) & 1) ^ 1);
        ok = __shfl_sync(0xffffffffu, ok, 0);
        if (!ok) {
          if (lane == 0) atomicExch(a.counters + kWsStatusSlot, (unsigned)PF_ERR_TIMEOUT);
          return;
        }
      }
      if (lane == 0) {
        mbar_expect(full0 + 8 * slot, L::W + L::X);
        tma_2d(sb, &tmap, st * S * F::WPG, rb * kRowsBlk, full0 + 8 * slot);
        if (it >= first) bulk_1d(sb + L::XOFF, a.rec + (size_t)st * L::X, L::X, full0 + 8 * slot);
      }
      if constexpr (SMODE == kScaleGroup) {
        const uint32_t* sc = static_cast<const uint32_t*>(a.scales);
        const uint32_t* mn = reinterpret_cast<const uint32_t*>(a.mins);
#pragma unroll
        for (int k = 0; k < kRowsBlk / 32; ++k) {
          const int row = lane + 32 * k, grow = rb * kRowsBlk + row;
          const size_t o = ((size_t)grow * G + (size_t)st * S) / 2;
          uint32_t sv[S / 2], mv[S / 2];
#pragma unroll
          for (int q = 0; q < S / 2; ++q) {
            sv[q] = grow < M ? __ldg(sc + o + q) : 0u;
            mv[q] = grow < M ? __ldg(mn + o + q) : 0u;
          }
          const uint32_t d = sb + L::SOFF + row * (S * 4);
#pragma unroll
          for (int q = 0; q < S / 2; ++q) {
            asm volatile("st.shared.b32 [%0], %1;" ::"r"(d + 4 * q), "r"(sv[q]));
            asm volatile("st.shared.b32 [%0], %1;" ::"r"(d + 2 * S + 4 * q), "r"(mv[q]));
          }
        }
      } else if constexpr (SMODE == kScaleRow) {
        const float* sc = static_cast<const float*>(a.scales);
#pragma unroll
        for (int k = 0; k < kRowsBlk / 32; ++k) {
          const int row = lane + 32 * k, grow = rb * kRowsBlk + row;
          const float v = grow < M ? __ldg(sc + grow) : 0.f;
          asm volatile("st.shared.f32 [%0], %1;" ::"r"(sb + L::SOFF + row * 4), "f"(v));
        }
      }
      mbar_arrive(full0 + 8 * slot);
      if (it == first - 1) {
        // x' comes from the x-prep grid: wait for it, then fetch the records
        // of the stages already in flight
        asm volatile("griddepcontrol.wait;" ::: "memory");
        if (lane == 0) {
          int rb2 = u0 / spb, st2 = u0 % spb;
          for (int k = 0; k < first; ++k) {
            bulk_1d(base + k * L::BYTES + L::XOFF, a.rec + (size_t)st2 * L::X, L::X, full0 + 8 * k);
            if (++st2 == spb) { st2 = 0; ++rb2; }
          }
        }
      }
      if (++st == spb) { st = 0; ++rb; }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int c = lane & 3, rq = lane >> 2;
  int rowb[TR][2];  // box rows of the thread
#pragma unroll
  for (int tr = 0; tr < TR; ++tr) {
    rowb[tr][0] = warp * 16 * TR + tr * 16 + row_perm<FMT>(rq);
    rowb[tr][1] = rowb[tr][0] + 8;
  }
  // per-row smem byte offsets of the thread's words (group 0), relative to the stage
  uint32_t woff[TR][2], woff12[TR][2];
#pragma unroll
  for (int tr = 0; tr < TR; ++tr)
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int r = rowb[tr][hh];
      if constexpr (FMT == PF_FMT_INT3_G128) {
        woff[tr][hh] = r * (S * 52) + 4 * c;
        woff12[tr][hh] = r * (S * 52) + 48;
      } else {
        woff[tr][hh] = r * 128;
        woff12[tr][hh] = r & 7;
      }
    }
  const uint32_t blane = (uint32_t)(lane & (LP - 1)) * 8;  // B fragment byte offset within a k-step row

  float y[TR][NT][2];
  int seg_st0 = 0;
  int rb = u0 / spb, st = u0 % spb;
  for (int it = 0; it < nunits; ++it) {
    const int slot = it % NS;
    const uint32_t sb = base + slot * L::BYTES;
    if (it == 0 || st == 0) {
      seg_st0 = st;
#pragma unroll
      for (int tr = 0; tr < TR; ++tr)
#pragma unroll
        for (int i = 0; i < NT; ++i) y[tr][i][0] = y[tr][i][1] = 0.f;
    }
    if (!mbar_wait(full0 + 8 * slot, (it / NS) & 1)) {
      atomicExch(a.counters + kWsStatusSlot, (unsigned)PF_ERR_TIMEOUT);
      return;
    }
    // scales / zero points of the thread's rows (fp32 row scale: per row)
    uint32_t srow[TR][2][S / 2], mrow[TR][2][S / 2];
    float frow[TR][2];
#pragma unroll
    for (int tr = 0; tr < TR; ++tr)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        const int r = rowb[tr][hh];
        if constexpr (SMODE == kScaleGroup) {
          const uint32_t d = sb + L::SOFF + r * (S * 4);
#pragma unroll
          for (int q = 0; q < S / 2; ++q) {
            srow[tr][hh][q] = lds32(d + 4 * q);
            mrow[tr][hh][q] = lds32(d + 2 * S + 4 * q);
          }
        } else if constexpr (SMODE == kScaleRow) {
          frow[tr][hh] = __uint_as_float(lds32(sb + L::SOFF + r * 4));
        } else {
          frow[tr][hh] = a.tensor_scale;
        }
      }
#pragma unroll
    for (int j = 0; j < S; ++j) {
      RowCodes<FMT> rc[TR][2];
#pragma unroll
      for (int tr = 0; tr < TR; ++tr)
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          if constexpr (FMT == PF_FMT_INT3_G128) {
            rc[tr][hh].load3(sb + woff[tr][hh] + 52 * j, sb + woff12[tr][hh] + 52 * j, c);
          } else if constexpr (is_int4(FMT)) {
            const uint32_t chunk = (uint32_t)((4 * j + c) ^ woff12[tr][hh]);
            rc[tr][hh].load(sb + woff[tr][hh] + (chunk << 4));
          } else {
            const uint32_t chunk = (uint32_t)((2 * j + (c >> 1)) ^ woff12[tr][hh]);
            rc[tr][hh].load(sb + woff[tr][hh] + (chunk << 4) + ((c & 1) << 3));
          }
        }
      const uint32_t rec = sb + L::XOFF + j * L::R;
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        // two independent accumulator chains per tile (even / odd k-steps);
        // lanes whose B columns carry no token read a valid finite value
        // (columns of an MMA are independent, the extra outputs are unused)
        float acc[TR][2][4];
#pragma unroll
        for (int tr = 0; tr < TR; ++tr)
#pragma unroll
          for (int e = 0; e < 2; ++e) acc[tr][e][0] = acc[tr][e][1] = acc[tr][e][2] = acc[tr][e][3] = 0.f;
#pragma unroll
        for (int j8 = 0; j8 < 8; ++j8) {
          const uint2 b = lds64(rec + (uint32_t)((i * 8 + j8) * LP * 8) + blane);
#pragma unroll
          for (int tr = 0; tr < TR; ++tr)
            mma16816(acc[tr][j8 & 1], rc[tr][0].h(2 * j8), rc[tr][1].h(2 * j8), rc[tr][0].h(2 * j8 + 1),
                     rc[tr][1].h(2 * j8 + 1), b.x, b.y);
        }
        const int t = 4 * i + c;
        const float4 g4 = lds128f(rec + NT * 8 * LP * 8 + (t < N ? t : 0) * 16);
#pragma unroll
        for (int tr = 0; tr < TR; ++tr)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            float sv, mv;
            if constexpr (SMODE == kScaleGroup) {
              const float2 s2 = __half22float2(*reinterpret_cast<const __half2*>(&srow[tr][hh][j >> 1]));
              const float2 m2 = __half22float2(*reinterpret_cast<const __half2*>(&mrow[tr][hh][j >> 1]));
              sv = (j & 1) ? s2.y : s2.x;
              mv = (j & 1) ? m2.y : m2.x;
            } else {
              sv = frow[tr][hh];
              mv = -(float)kOffset * sv;
            }
            const float q = 1024.f * ((acc[tr][0][2 * hh] + acc[tr][1][2 * hh]) +
                                      (acc[tr][0][2 * hh + 1] + acc[tr][1][2 * hh + 1]));
            y[tr][i][hh] += (sv * g4.y) * q + mv * g4.x;
          }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8 * slot);

    // -------------------------------------------------- end of a row-block segment
    const bool seg_end = (st == spb - 1 || it == nunits - 1);
    if (seg_end) {
      const bool whole = (seg_st0 == 0 && st == spb - 1);
      if (whole) {
#pragma unroll
        for (int tr = 0; tr < TR; ++tr)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            const int grow = rb * kRowsBlk + rowb[tr][hh];
            if (grow >= M) continue;
            const float bv = a.bias ? a.bias[grow] : 0.f;
#pragma unroll
            for (int i = 0; i < NT; ++i) {
              const int t = 4 * i + c;
              if (t < N) a.y[(size_t)t * M + grow] = y[tr][i][hh] + bv;
            }
          }
      } else {
        const int my_slot = (rb == u0 / spb) ? (int)(2 * cta) : (int)(2 * cta + 1);
        float* part = a.partials + (size_t)my_slot * kRowsBlk * N;
#pragma unroll
        for (int tr = 0; tr < TR; ++tr)
#pragma unroll
          for (int hh = 0; hh < 2; ++hh)
#pragma unroll
            for (int i = 0; i < NT; ++i) {
              const int t = 4 * i + c;
              if (t < N) part[(size_t)rowb[tr][hh] * N + t] = y[tr][i][hh];
            }
        __threadfence();
        __syncwarp();
        const long long first = cta_of((long long)rb * spb, U, P);
        const long long last = cta_of((long long)(rb + 1) * spb - 1, U, P);
        const unsigned n_share = (unsigned)(last - first + 1);
        unsigned* ctr = a.counters + (size_t)rb * kCWarps + warp;
        unsigned prev = 0;
        if (lane == 0) prev = atomicAdd(ctr, 1u);
        prev = __shfl_sync(0xffffffffu, prev, 0);
        if (prev == n_share - 1) {
          __threadfence();
#pragma unroll
          for (int tr = 0; tr < TR; ++tr)
#pragma unroll
            for (int hh = 0; hh < 2; ++hh) {
              const int r = rowb[tr][hh], grow = rb * kRowsBlk + r;
#pragma unroll
              for (int i = 0; i < NT; ++i) {
                const int t = 4 * i + c;
                if (t >= N) continue;
                float accv = 0.f;
                for (long long k = first; k <= last; ++k) {
                  const long long ku0 = k * U / P;
                  const int ks = (rb == (int)(ku0 / spb)) ? (int)(2 * k) : (int)(2 * k + 1);
                  accv += __ldcg(a.partials + ((size_t)ks * kRowsBlk + r) * N + t);
                }
                if (grow < M) a.y[(size_t)t * M + grow] = accv + (a.bias ? a.bias[grow] : 0.f);
              }
            }
          if (lane == 0) *ctr = 0u;
        }
      }
    }
    if (++st == spb) { st = 0; ++rb; }
  }
}

// ------------------------------------------------------------------ host side
int sm_count() {
  static int n = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  });
  return n;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

constexpr int kTR = 1;  // 16-row MMA tiles per consumer warp (rows per block = 16 * kCWarps * kTR)

template <int FMT, int NT, int LP, int SMODE>
cudaError_t launch_one(const TmaArgs& a, cudaStream_t s) {
  using F = TmaFmt<FMT>;
  using L = Stage<FMT, NT, LP, kTR, SMODE>;
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)a.row_words, (cuuint64_t)a.M};
  cuuint64_t strides[1] = {(cuuint64_t)a.row_words * 4};
  cuuint32_t box[2] = {(cuuint32_t)(F::S * F::WPG), (cuuint32_t)L::kRowsBlk};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(a.codes), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  F::SW128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  const size_t smem = L::SMEM;
  auto kern = gemv_tma_kernel<FMT, NT, LP, kTR, SMODE>;
  static int occ = 0;
  if (occ == 0) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kThreadsT, smem) != cudaSuccess || n < 1) n = 1;
    occ = n < kMaxCtasPerSm ? n : kMaxCtasPerSm;
  }
  int grid = sm_count() * occ;
  if (grid > a.n_units) grid = a.n_units;
  if (grid < 1) grid = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(kThreadsT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kern, map, a);
}

template <int FMT, int NT, int LP>
cudaError_t launch_sm(const TmaArgs& a, int smode, cudaStream_t s) {
  if constexpr (FMT == PF_FMT_INT4 || FMT == PF_FMT_INT2) {
    if (smode == kScaleRow) return launch_one<FMT, NT, LP, kScaleRow>(a, s);
    return launch_one<FMT, NT, LP, kScaleTensor>(a, s);
  } else {
    return launch_one<FMT, NT, LP, kScaleGroup>(a, s);
  }
}

template <int FMT>
cudaError_t launch_fmt(const TmaArgs& a, int smode, cudaStream_t s) {
  if (a.NT == 1) return a.N == 1 ? launch_sm<FMT, 1, 8>(a, smode, s) : launch_sm<FMT, 1, 32>(a, smode, s);
  if (a.NT == 2) return launch_sm<FMT, 2, 32>(a, smode, s);
  return launch_sm<FMT, 4, 32>(a, smode, s);
}

}  // namespace

int tma_stage_groups(int fmt) {
  switch (fmt) {
    case PF_FMT_INT4_G128:
    case PF_FMT_INT4: return TmaFmt<PF_FMT_INT4_G128>::S;
    case PF_FMT_INT2_G128:
    case PF_FMT_INT2: return TmaFmt<PF_FMT_INT2_G128>::S;
    default: return TmaFmt<PF_FMT_INT3_G128>::S;
  }
}

bool tma_eligible(int fmt, int M, int K, const void* codes) {
  if (!(fmt == PF_FMT_INT4_G128 || fmt == PF_FMT_INT3_G128 || fmt == PF_FMT_INT2_G128 || fmt == PF_FMT_INT4 ||
        fmt == PF_FMT_INT2))
    return false;
  if (K % 512 != 0) return false;
  if (reinterpret_cast<uintptr_t>(codes) % 16) return false;
  const long long n_rb = (M + 16 * kCWarps * kTR - 1) / (16 * kCWarps * kTR);
  if (n_rb * kCWarps >= (long long)kWsStatusSlot) return false;
  return encode_fn() != nullptr;
}

// CTAs of one launch: never more than the units, at most kMaxCtasPerSm per SM
// (shared memory bounds the real residency; the partial-slot area is sized
// for this count).
int tma_block_rows() { return 16 * kCWarps * kTR; }

int tma_grid(int fmt, int NT, int n_units) {
  (void)fmt;
  (void)NT;
  long long g = (long long)sm_count() * kMaxCtasPerSm;
  if (g > n_units) g = n_units;
  return (int)(g < 1 ? 1 : g);
}

cudaError_t launch_gemv_tma(int fmt, const TmaArgs& a, int smode, int subnormal, cudaStream_t s) {
  (void)subnormal;
  switch (fmt) {
    case PF_FMT_INT4_G128: return launch_fmt<PF_FMT_INT4_G128>(a, smode, s);
    case PF_FMT_INT3_G128: return launch_fmt<PF_FMT_INT3_G128>(a, smode, s);
    case PF_FMT_INT2_G128: return launch_fmt<PF_FMT_INT2_G128>(a, smode, s);
    case PF_FMT_INT4: return launch_fmt<PF_FMT_INT4>(a, smode, s);
    case PF_FMT_INT2: return launch_fmt<PF_FMT_INT2>(a, smode, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace pfb
