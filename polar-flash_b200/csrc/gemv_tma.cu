// Streaming fused dequant-GEMV for the INT formats (N <= 16 tokens): one
// launch computes y_j = x_j W_j^T for up to sixteen weights ("jobs") of one
// format, each with its own input, e.g. every linear of a model layer.
//
// x' (the forward block RWHT of x, scaled and split into the tensor cores'
// B fragments) is made once per input by xprep_frag_kernel into the
// workspace: one 576-byte record per 128-column group at N = 1.
//
// GEMV work unit = (job, 128-row block, stage of S groups of 128 columns).
// The units are dealt to the CTAs stream-K style, each CTA taking an equal
// contiguous range in row-block-major order, so a CTA walks all stages of
// its row blocks and keeps their sums in registers: only the (at most two)
// row blocks a CTA shares with its neighbours are reduced through memory,
// by the last of their warps to arrive (arrival counter per 16 rows, parts
// added in stage order, so the result does not depend on timing).  There is
// no separate combine launch.
//
// CTA = 8 warps, two CTAs per SM.  Every warp owns 16 rows of each unit and
// streams them itself through a private ring of shared-memory slots: lane 0
// issues the 2-D TMA copy of its 16 x (S groups) tile of packed codes (L2
// evict-first), all lanes copy the tile's fp16 scales / zero points with
// cp.async, and the copies themselves arrive on the slot's mbarrier.  The
// x' records of each unit's stage come from the workspace (L2) into a small
// CTA-wide ring by one bulk copy; the last warp done with a stage's records
// refills that slot.  Weights are requested before the kernel waits for the
// preceding grid (programmatic dependent launch: packed weights and scales
// are never written by a kernel that precedes a GEMV in this library).
//
// Compute: the unit's code words are read into registers, every code pair
// becomes one AND (exact subnormal fp16 q 2^(p-24)), and mma.sync m16n8k16
// multiplies two groups at a time against the B fragments of x' (fp16 hi / lo
// halves of x' in the two columns of each token).
// Per 128-column group:  sum w x' = s 2^E Q + m Sx  with  Q = sum q x'/2^E.
// Every wait is bounded (%globaltimer): on expiry the kernel records
// PF_ERR_TIMEOUT in the workspace status word, skips every later wait and
// finishes.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <stdlib.h>
#include <string.h>

#include <mutex>

#include "common.cuh"
#include "gemv.cuh"
#include "tma.cuh"

namespace pfb {

namespace {

constexpr int kWarps = 8;                  // warps per CTA
constexpr int kThreadsT = kWarps * 32;
constexpr int kWarpRows = 16;              // rows per warp and unit (one MMA row tile)
constexpr int kRowsBlk = kWarpRows * kWarps;  // rows per unit
constexpr int kMaxStages = 8;

// Dynamic shared memory per CTA: two CTAs share an SM's 228 KB.
int smem_budget(int ctas_per_sm) { return ctas_per_sm >= 2 ? 110 * 1024 : 200 * 1024; }

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

// One slot of a warp's ring: the 16-row code tile, then its scales.  Tiles
// under the 128B swizzle start on a 1024-byte boundary.
template <int FMT, int SMODE>
struct WarpSlot {
  static constexpr int S = TmaFmt<FMT>::S;
  static constexpr uint32_t W = kWarpRows * S * TmaFmt<FMT>::WPG * 4;
  static constexpr uint32_t SROW = SMODE == kScaleGroup ? S * 4 : (SMODE == kScaleRow ? 4 : 0);  // bytes per row
  static constexpr uint32_t ALIGN = TmaFmt<FMT>::SW128 ? 1024u : 128u;
  static constexpr uint32_t BYTES = (W + kWarpRows * SROW + ALIGN - 1) & ~(ALIGN - 1);
};

// x' record of one 128-column group: [NT tiles][4 k-step pairs][LP lanes]
// uint4 (the B fragments of two k-steps), then float4 {Sx, 1024 2^E, -, -}
// per token slot.  A tile's 8 B columns hold TPT tokens: 4 tokens as fp16
// hi / lo pairs (N <= 4), or 8 tokens as one fp16 each (N > 4).
template <int NT, int LP, int TPT = 4>
struct XRec {
  static constexpr uint32_t FRAG = NT * 4 * LP * 16;
  static constexpr uint32_t R = FRAG + 16 * TPT * NT;
};

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

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm("mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// ---- per-row decode state: the few registers from which every code pair of
// a group is one AND (codes land as exact subnormal fp16 q * 2^(p-24)); the
// pair -> column map is frag_cols2 (common.cuh).
template <int FMT>
struct RowCodes;

template <>
struct RowCodes<PF_FMT_INT4_G128> {
  uint32_t w[4], v[4];
  __device__ __forceinline__ void set(const uint32_t (&raw)[4], int) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      w[t] = raw[t];
      v[t] = raw[t] >> 8;
    }
  }
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
  __device__ __forceinline__ void set(const uint32_t (&raw)[4], int) {
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      w[t] = raw[t];
      v[t] = raw[t] >> 10;
    }
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
  __device__ __forceinline__ void set(const uint32_t (&raw)[4], int c) {
#pragma unroll
    for (int t = 0; t < 3; ++t) {
      g[t] = (raw[t] & 0x0000FFFFu) | ((raw[t] << 1) & 0xFFFF0000u);
      v[t] = g[t] >> 9;
    }
    const uint32_t t12 = raw[3] >> (6 * c);
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

// Raw words of row r, group j of a ring stage: INT3 words c, c+4, c+8 and 12;
// INT4 words 4c..4c+3; INT2 words 2c, 2c+1 (128B-swizzled rows for INT4/INT2).
template <int FMT>
__device__ __forceinline__ void load_words(const unsigned char* stg, int r, int j, int c, uint32_t (&raw)[4]) {
  constexpr int S = TmaFmt<FMT>::S;
  if constexpr (FMT == PF_FMT_INT3_G128) {
    const unsigned char* p = stg + r * (S * 52) + 52 * j;
    raw[0] = lds<uint32_t>(p + 4 * c);
    raw[1] = lds<uint32_t>(p + 16 + 4 * c);
    raw[2] = lds<uint32_t>(p + 32 + 4 * c);
    raw[3] = lds<uint32_t>(p + 48);
  } else if constexpr (is_int4(FMT)) {
    const uint32_t chunk = (uint32_t)((4 * j + c) ^ (r & 7));
    const uint4 q = lds<uint4>(stg + r * 128 + (chunk << 4));
    raw[0] = q.x; raw[1] = q.y; raw[2] = q.z; raw[3] = q.w;
  } else {
    const uint32_t chunk = (uint32_t)((2 * j + (c >> 1)) ^ (r & 7));
    const uint2 q = lds<uint2>(stg + r * 128 + (chunk << 4) + ((c & 1) << 3));
    raw[0] = q.x; raw[1] = q.y; raw[2] = 0u; raw[3] = 0u;
  }
}


// Group-relative columns (lo0, hi0, lo1, hi1) of a lane's B fragment and the
// mantissa positions of its two code pairs.
struct LaneCols {
  int col[4];
  int p[2];
};

// 2^e as a float for an unbiased exponent e clamped to the normal range.
__device__ __forceinline__ float pow2f(int e) {
  e = e < -126 ? -126 : (e > 127 ? 127 : e);
  return __int_as_float((e + 127) << 23);
}

// ---- x' of one prep chunk (C = 32 E columns of token t, one warp): forward
// block RWHT of x (signs, Walsh-Hadamard butterflies in registers and across
// lanes, 1/sqrt(b)), then for every group of the chunk inside [g_lo, g_hi):
// the group's power-of-two normaliser E (|x'| < 2^E), the tensor-core B
// fragments of x' 2^(14 - p - E) split into fp16 hi + lo, and {Sx, 1024 2^E},
// written to the records at `recs` (the record of group g_lo first).
// Tokens t >= N write zeros.  Every global load is issued before any is used.
template <int NT, int LP, int E, int TPT>
__device__ __forceinline__ void prep_chunk(const XPrepJob& jb, int N, int x_dtype, int col0, int g_lo, int g_hi,
                                           int t, unsigned char* recs, float* scratch, int lane,
                                           const LaneCols& lc) {
  constexpr int C = 32 * E;
  constexpr int LG = 128 / E;  // lanes per 128-column group
  const int b = jb.had_block;
  float v[E];
  if (t < N) {
    const size_t base = (size_t)t * jb.K + col0 + E * lane;
    int s4[E / 4];
    const int* sp = reinterpret_cast<const int*>((b > 0 ? jb.signs : static_cast<const int8_t*>(jb.x)) + col0 +
                                                 E * lane);
#pragma unroll
    for (int q = 0; q < E / 4; ++q) s4[q] = __ldg(sp + q);
    if (x_dtype == PF_DTYPE_F32) {
      const float4* xp = reinterpret_cast<const float4*>(static_cast<const float*>(jb.x) + base);
      float4 f[E / 4];
#pragma unroll
      for (int q = 0; q < E / 4; ++q) f[q] = __ldg(xp + q);
#pragma unroll
      for (int q = 0; q < E / 4; ++q) {
        v[4 * q] = f[q].x; v[4 * q + 1] = f[q].y; v[4 * q + 2] = f[q].z; v[4 * q + 3] = f[q].w;
      }
    } else {
      const uint2* xp = reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(jb.x) + base);
      uint2 r[E / 4];
#pragma unroll
      for (int q = 0; q < E / 4; ++q) r[q] = __ldg(xp + q);
#pragma unroll
      for (int q = 0; q < E / 4; ++q) {
        if (x_dtype == PF_DTYPE_F16) {
          const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&r[q].x));
          const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&r[q].y));
          v[4 * q] = f0.x; v[4 * q + 1] = f0.y; v[4 * q + 2] = f1.x; v[4 * q + 3] = f1.y;
        } else {  // bf16: the upper half of an fp32
          v[4 * q] = __uint_as_float(r[q].x << 16);
          v[4 * q + 1] = __uint_as_float(r[q].x & 0xFFFF0000u);
          v[4 * q + 2] = __uint_as_float(r[q].y << 16);
          v[4 * q + 3] = __uint_as_float(r[q].y & 0xFFFF0000u);
        }
      }
    }
    if (b > 0) {
#pragma unroll
      for (int q = 0; q < E / 4; ++q)
#pragma unroll
        for (int e = 0; e < 4; ++e)  // sign bit of the int8 column sign
          v[4 * q + e] = __uint_as_float(__float_as_uint(v[4 * q + e]) ^ (((uint32_t)s4[q] << (24 - 8 * e)) & 0x80000000u));
#pragma unroll
      for (int h = 1; h < E; h *= 2) {
        if (h < b) {
#pragma unroll
          for (int e = 0; e < E; ++e)
            if (!(e & h)) {
              const float u = v[e], w = v[e + h];
              v[e] = u + w;
              v[e + h] = u - w;
            }
        }
      }
#pragma unroll
      for (int m = 1; m < 32; m *= 2) {
        if (m * E < b) {
          const float sg = (lane & m) ? -1.f : 1.f;
#pragma unroll
          for (int e = 0; e < E; ++e) {
            const float p = __shfl_xor_sync(0xffffffffu, v[e], m);
            v[e] = fmaf(sg, v[e], p);
          }
        }
      }
      const float rs = jb.had_rscale;
#pragma unroll
      for (int e = 0; e < E; ++e) v[e] *= rs;
    }
  } else {
#pragma unroll
    for (int e = 0; e < E; ++e) v[e] = 0.f;
  }
  // group statistics: max |x'| (as ordered bit patterns of non-negative floats) and sum
  uint32_t amax = 0u;
  float sx = 0.f;
#pragma unroll
  for (int e = 0; e < E; ++e) {
    amax = max(amax, __float_as_uint(v[e]) & 0x7FFFFFFFu);
    sx += v[e];
  }
  if constexpr (LG == 32) {
    amax = __reduce_max_sync(0xffffffffu, amax);
  } else {
#pragma unroll
    for (int o = 1; o < LG; o *= 2) amax = max(amax, __shfl_xor_sync(0xffffffffu, amax, o));
  }
#pragma unroll
  for (int o = 1; o < LG; o *= 2) sx += __shfl_xor_sync(0xffffffffu, sx, o);
  // |x'| < 2^ex: one more than the exponent of amax (any value for amax = 0)
  const int ex = amax == 0u ? 0 : (amax < 0x00800000u ? -125 : (int)(amax >> 23) - 126);
#pragma unroll
  for (int q = 0; q < E / 4; ++q)
    *reinterpret_cast<float4*>(scratch + E * lane + 4 * q) =
        make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  __syncwarp();
  const int j8 = lane >> 2;
  // B-fragment lane of the token's column: hi at column 2 (t % 4), lo next to
  // it, or the token's own column t % 8
  const int fl = TPT == 4 ? 8 * (t & 3) + (lane & 3) : 4 * (t & 7) + (lane & 3);
  const int tile = TPT == 4 ? t >> 2 : t >> 3;
#pragma unroll
  for (int gi = 0; gi < C / 128; ++gi) {
    const int g = col0 / 128 + gi;
    const int eg = __shfl_sync(0xffffffffu, ex, gi * LG);
    const float sg = __shfl_sync(0xffffffffu, sx, gi * LG);
    if (g < g_lo || g >= g_hi) continue;
    const float f0 = pow2f(14 - lc.p[0] - eg), f1 = pow2f(14 - lc.p[1] - eg);
    const float* xs = scratch + gi * 128;
    const float xv[4] = {xs[lc.col[0]] * f0, xs[lc.col[1]] * f0, xs[lc.col[2]] * f1, xs[lc.col[3]] * f1};
    uint32_t hw[2], lw[2];
#pragma unroll
    for (int k = 0; k < 2; ++k) {
      const __half h0 = __float2half_rn(xv[2 * k]), h1 = __float2half_rn(xv[2 * k + 1]);
      const __half l0 = __float2half_rn(xv[2 * k] - __half2float(h0));
      const __half l1 = __float2half_rn(xv[2 * k + 1] - __half2float(h1));
      hw[k] = (uint32_t)__half_as_ushort(h0) | ((uint32_t)__half_as_ushort(h1) << 16);
      lw[k] = (uint32_t)__half_as_ushort(l0) | ((uint32_t)__half_as_ushort(l1) << 16);
    }
    using XR = XRec<NT, LP, TPT>;
    unsigned char* rec = recs + (size_t)(g - g_lo) * XR::R;
    unsigned char* fr = rec + (tile * 4 + (j8 >> 1)) * LP * 16 + (j8 & 1) * 8;
    *reinterpret_cast<uint2*>(fr + fl * 16) = make_uint2(hw[0], hw[1]);
    if (TPT == 4) *reinterpret_cast<uint2*>(fr + (fl + 4) * 16) = make_uint2(lw[0], lw[1]);
    if (lane == 0) *reinterpret_cast<float2*>(rec + XR::FRAG + t * 16) = make_float2(sg, 1024.f * pow2f(eg));
  }
  __syncwarp();
}

// Inputs of one x' preparation launch.
struct XPrepArgs {
  XPrepJob xj[kXPrepMaxJobs];
  int n_xj, N, x_dtype;
};
constexpr int kPrepCols = 512;  // columns of one prep block

// One block per (input, 512 columns): the four groups' records of every
// token slot.  Launched as a programmatic dependent (x may come from the
// preceding grid).
template <int NT, int LP, int TPT>
__global__ void __launch_bounds__(kThreadsT) xprep_frag_kernel(const __grid_constant__ XPrepArgs a) {
  asm volatile("griddepcontrol.launch_dependents;");
  __shared__ __align__(16) float scratch[kWarps][kPrepCols];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  int k = 0;
  for (int i = 1; i < a.n_xj; ++i)
    if ((int)blockIdx.x >= a.xj[i].blk0) k = i;
  const XPrepJob& jb = a.xj[k];
  const int region = (int)blockIdx.x - jb.blk0;
  const int g_lo = region * (kPrepCols / 128), g_hi = g_lo + kPrepCols / 128;
  LaneCols lc;
  {
    const int c = lane & 3, rq = lane >> 2;
    int lo, hi, p;
    frag_cols2(jb.fmt, c, 2 * rq, lo, hi, p);
    lc.col[0] = lo; lc.col[1] = hi; lc.p[0] = p;
    frag_cols2(jb.fmt, c, 2 * rq + 1, lo, hi, p);
    lc.col[2] = lo; lc.col[3] = hi; lc.p[1] = p;
  }
  using XR = XRec<NT, LP, TPT>;
  unsigned char* recs = jb.xq + (size_t)g_lo * XR::R;
  const int b = jb.had_block;
  const int E = b > 256 ? 16 : (b > 128 ? 8 : 4);
  const int Cc = 32 * E;
  const int tslots = LP == 8 ? 1 : TPT * NT;
  asm volatile("griddepcontrol.wait;" ::: "memory");
  int task = 0;
  for (int ci = 0; ci < kPrepCols / Cc; ++ci)
    for (int t = 0; t < tslots; ++t, ++task) {
      if (task % kWarps != warp) continue;
      const int col0 = region * kPrepCols + ci * Cc;
      if (E == 4)
        prep_chunk<NT, LP, 4, TPT>(jb, a.N, a.x_dtype, col0, g_lo, g_hi, t, recs, scratch[warp], lane, lc);
      else if (E == 8)
        prep_chunk<NT, LP, 8, TPT>(jb, a.N, a.x_dtype, col0, g_lo, g_hi, t, recs, scratch[warp], lane, lc);
      else
        prep_chunk<NT, LP, 16, TPT>(jb, a.N, a.x_dtype, col0, g_lo, g_hi, t, recs, scratch[warp], lane, lc);
    }
}

struct TmaMaps {
  CUtensorMap m[kTmaMaxJobs];
};

// Job holding global unit u.
__device__ __forceinline__ int job_of(const TmaArgs& a, int u) {
  int j = 0;
#pragma unroll
  for (int k = 1; k < kTmaMaxJobs; ++k)
    if (k < a.n_jobs && u >= a.job[k].unit0) j = k;
  return j;
}

// Stream-K partition: CTA c of P takes units [c U / P, (c + 1) U / P).
__device__ __forceinline__ int cta_first_unit(unsigned c, unsigned U, unsigned P) {
  return (int)(((unsigned long long)c * U) / P);
}
__device__ __forceinline__ int cta_of_unit(unsigned u, unsigned U, unsigned P) {
  return (int)((((unsigned long long)u + 1) * P - 1) / U);
}

// One stage of a CTA's ring for format FMT: the 128-row code tile (one TMA
// box), the rows' scales / zero points, then the stage's x' records.  Tiles
// under the 128B swizzle start on a 1024-byte boundary.
template <int FMT, int SMODE, int XB>
struct CtaSlot {
  static constexpr int S = TmaFmt<FMT>::S;
  static constexpr uint32_t ROW = S * TmaFmt<FMT>::WPG * 4;  // code bytes per row
  static constexpr uint32_t CW = kRowsBlk * ROW;
  static constexpr uint32_t SROW = SMODE == kScaleGroup ? S * 4 : (SMODE == kScaleRow ? 4 : 0);
  static constexpr uint32_t XOFF = (CW + kRowsBlk * SROW + 127) & ~127u;
  static constexpr uint32_t ALIGN = TmaFmt<FMT>::SW128 ? 1024u : 128u;
  static constexpr uint32_t BYTES = (XOFF + XB + ALIGN - 1) & ~(ALIGN - 1);
};
template <int FA, int FB, int SMODE, int XB>
struct MixSlot {
  using A = CtaSlot<FA, SMODE, XB>;
  using B = CtaSlot<FB, SMODE, XB>;
  static constexpr uint32_t ALIGN = A::ALIGN > B::ALIGN ? A::ALIGN : B::ALIGN;
  static constexpr uint32_t RAW = A::BYTES > B::BYTES ? A::BYTES : B::BYTES;
  static constexpr uint32_t BYTES = (RAW + ALIGN - 1) & ~(ALIGN - 1);
};

// One unit of format FMT (this warp's 16 rows x S groups) accumulated into
// y: code words read into registers, decoded by one AND per code pair,
// mma.sync against the x' B fragments, per-group scale and zero point.
// codes: the warp's 16-row code tile; sc: its rows' scales; xs: the x' records.
template <int FMT, int NT, int LP, int SMODE, int TPT>
__device__ __forceinline__ void unit_body(const unsigned char* codes, const unsigned char* sc, const unsigned char* xs,
                                          const int (&rl)[2], int c, uint32_t blane, float jts,
                                          float (&y)[NT][2][TPT / 4]) {
  using XR = XRec<NT, LP, TPT>;
  constexpr int S = TmaFmt<FMT>::S;
  constexpr int kOffset = IntFmt<FMT>::kOffset;
  constexpr int YT = TPT / 4;
  constexpr uint32_t SROW = SMODE == kScaleGroup ? S * 4 : (SMODE == kScaleRow ? 4 : 0);
#pragma unroll
  for (int pp = 0; pp < S / 2; ++pp) {
    // scales / zero points of the pair's two groups, then their code words
    uint32_t sv2[2], mv2[2];
    float frow[2];
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const unsigned char* sp = sc + rl[hh] * SROW;
      if constexpr (SMODE == kScaleGroup) {
        sv2[hh] = lds<uint32_t>(sp + 4 * pp);
        mv2[hh] = lds<uint32_t>(sp + 2 * S + 4 * pp);
        frow[hh] = 0.f;
      } else if constexpr (SMODE == kScaleRow) {
        frow[hh] = lds<float>(sp);
        sv2[hh] = mv2[hh] = 0u;
      } else {
        frow[hh] = jts;
        sv2[hh] = mv2[hh] = 0u;
      }
    }
    RowCodes<FMT> rc[2][2];
#pragma unroll
    for (int gg = 0; gg < 2; ++gg)
#pragma unroll
      for (int hh = 0; hh < 2; ++hh) {
        uint32_t raw[4];
        load_words<FMT>(codes, rl[hh], 2 * pp + gg, c, raw);
        rc[gg][hh].set(raw, c);
      }
    float acc[2][NT][4];
#pragma unroll
    for (int gg = 0; gg < 2; ++gg)
#pragma unroll
      for (int i = 0; i < NT; ++i) acc[gg][i][0] = acc[gg][i][1] = acc[gg][i][2] = acc[gg][i][3] = 0.f;
#pragma unroll
    for (int jp = 0; jp < 4; ++jp)
#pragma unroll
      for (int i = 0; i < NT; ++i)
#pragma unroll
        for (int gg = 0; gg < 2; ++gg) {
          const uint4 bq = lds<uint4>(xs + (2 * pp + gg) * XR::R + (i * 4 + jp) * LP * 16 + blane);
          const RowCodes<FMT>& r0 = rc[gg][0];
          const RowCodes<FMT>& r1 = rc[gg][1];
          mma16816(acc[gg][i], r0.h(4 * jp), r1.h(4 * jp), r0.h(4 * jp + 1), r1.h(4 * jp + 1), bq.x, bq.y);
          mma16816(acc[gg][i], r0.h(4 * jp + 2), r1.h(4 * jp + 2), r0.h(4 * jp + 3), r1.h(4 * jp + 3), bq.z, bq.w);
        }
#pragma unroll
    for (int gg = 0; gg < 2; ++gg) {
      const int g = 2 * pp + gg;
#pragma unroll
      for (int i = 0; i < NT; ++i) {
#pragma unroll
        for (int u = 0; u < YT; ++u) {
          // token of accumulator columns 2c, 2c + 1: one token as hi + lo, or two tokens
          const int t = LP == 8 ? 0 : (TPT == 4 ? 4 * i + c : 8 * i + 2 * c + u);
          const float2 gs = lds<float2>(xs + g * XR::R + XR::FRAG + t * 16);
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            float sv, mv;
            if constexpr (SMODE == kScaleGroup) {
              sv = __half2float(__ushort_as_half((unsigned short)(gg ? (sv2[hh] >> 16) : (sv2[hh] & 0xFFFFu))));
              mv = __half2float(__ushort_as_half((unsigned short)(gg ? (mv2[hh] >> 16) : (mv2[hh] & 0xFFFFu))));
            } else {
              sv = frow[hh];
              mv = -(float)kOffset * sv;
            }
            const float q = TPT == 4 ? acc[gg][i][2 * hh] + acc[gg][i][2 * hh + 1] : acc[gg][i][2 * hh + u];
            y[i][hh][u] += (sv * gs.y) * q + mv * gs.x;
          }
        }
      }
    }
  }
}

template <int FA, int FB, int NT, int LP, int SMODE, int TPT>
__global__ void __launch_bounds__(kThreadsT, 2)
    gemv_tma_kernel(const __grid_constant__ TmaMaps maps, const __grid_constant__ TmaArgs a) {
  using XR = XRec<NT, LP, TPT>;
  constexpr int S = TmaFmt<FA>::S;
  static_assert(TmaFmt<FB>::S == S, "formats of one launch share the stage width");
  constexpr int XB = S * XR::R;  // x' bytes of one stage (a multiple of 128)
  using SA = CtaSlot<FA, SMODE, XB>;
  using SB = CtaSlot<FB, SMODE, XB>;
  constexpr uint32_t SLOT = MixSlot<FA, FB, SMODE, XB>::BYTES;
  constexpr int YT = TPT / 4;  // tokens of a thread per tile

  asm volatile("griddepcontrol.launch_dependents;");
  // the launch's parameters are cold in every SM's constant cache: touch each
  // 64-byte line once, in parallel, before the dependent reads that follow
  if (threadIdx.x < (sizeof(TmaArgs) + 63) / 64) {
    constexpr unsigned kLast = sizeof(TmaArgs) / 4 - 1;
    const unsigned i = threadIdx.x * 16 < kLast ? threadIdx.x * 16 : kLast;
    const uint32_t w = reinterpret_cast<const uint32_t*>(&a)[i];
    asm volatile("" ::"r"(w));
  }

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ int abort_flag;
  __shared__ unsigned scnt[kMaxStages];  // warps done with each ring stage
  __shared__ int flast;                  // CTA unit ordinal of the last stage fill issued
  unsigned char* const base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int NS = a.NS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t ring_s = smem_u32(base);
  const uint32_t full0 = ring_s + NS * SLOT;  // NS mbarriers after the stages

  const unsigned U = (unsigned)a.n_units, P = gridDim.x, cta = blockIdx.x;
  const int u0 = cta_first_unit(cta, U, P), u1 = cta_first_unit(cta + 1, U, P);  // U * P < 2^32 (host-checked)
  const int nunits = u1 - u0;

  if (threadIdx.x >= 32 && threadIdx.x < 32 + kTmaMaxJobs && nunits > 0) {
    const int k = threadIdx.x - 32;
    if (k >= job_of(a, u0) && k <= job_of(a, u1 - 1))
      asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&maps.m[k])) : "memory");
  }
  if (threadIdx.x == 0) {
    abort_flag = 0;
    flast = -1;
    for (int s = 0; s < NS; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(full0 + 8 * s), "r"(33));
  }
  if (threadIdx.x < kMaxStages) scnt[threadIdx.x] = 0u;
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  __syncthreads();
  // Gathering launches: once every CTA's rows are stored (in every rank's
  // buffer), the last CTA to finish raises this rank's flag in every buffer
  // to the rank's next epoch (system-scope release), then waits (bounded)
  // until every rank's flag in the local buffer has reached that epoch
  // (acquire): when the launch completes, all ranks' rows are here.  Every
  // rank raises its flag before it waits, and each rank runs on its own GPU.
  auto signal_done = [&]() {
    if (a.world <= 0) return;
    __syncthreads();  // the block's peer stores come before thread 0's fence (cumulative)
    if (threadIdx.x != 0) return;
    __threadfence_system();
    if (atomicAdd(a.done, 1u) == gridDim.x - 1) {
      atomicExch(a.done, 0u);
      __threadfence_system();
      volatile unsigned* ep = reinterpret_cast<volatile unsigned*>(a.peer[a.rank]);
      const unsigned e = *ep + 1u;
      *ep = e;
      for (int pr = 0; pr < a.world; ++pr) {
        unsigned* flag = reinterpret_cast<unsigned*>(a.peer[pr] + 16 + 4 * a.rank);
        asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(e) : "memory");
      }
      const unsigned long long t0 = now_ns();
      for (int q = 0; q < a.world; ++q) {
        const unsigned* flag = reinterpret_cast<const unsigned*>(a.peer[a.rank] + 16 + 4 * q);
        for (;;) {
          unsigned f;
          asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(f) : "l"(flag) : "memory");
          if ((int)(f - e) >= 0) break;
          if (now_ns() - t0 > kWaitNs) {
            atomicExch(a.status, (unsigned)PF_ERR_TIMEOUT);
            q = a.world;
            break;
          }
          __nanosleep(64);
        }
      }
    }
  };
  if (nunits <= 0) {
    signal_done();
    return;
  }
  const int N = a.N;
  const int c = lane & 3, rq = lane >> 2;
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));

  // Fill ring stage `slot` with the CTA's unit ordinal `i` (called by a whole
  // warp): lane 0 announces the bytes and issues the TMA of the 128-row code
  // tile (and, unless `weights_only`, the bulk copy of the stage's x'
  // records), every lane copies its share of the rows' scales / zero points
  // with cp.async and arrives on the stage's barrier when they land.
  auto fill = [&](int slot, int i, bool weights_only) {
    const int u = u0 + i;
    const int jj = job_of(a, u);
    const TmaJob& jb = a.job[jj];
    const int v = u - jb.unit0, rb = v / jb.spb, st = v - rb * jb.spb;
    const bool fs = FA != FB && jb.fsel;
    const uint32_t sb = ring_s + slot * SLOT, bar = full0 + 8 * slot;
    const uint32_t cw = fs ? SB::CW : SA::CW, xoff = fs ? SB::XOFF : SA::XOFF;
    const int wpg = fs ? TmaFmt<FB>::WPG : TmaFmt<FA>::WPG;
    __syncwarp();
    if (lane == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_expect(bar, cw + XB);
      tma_2d(sb, &maps.m[jj], st * S * wpg, rb * kRowsBlk, bar, policy);
      if (!weights_only) bulk_g2s(sb + xoff, jb.xq + (size_t)st * XB, XB, bar);
    }
    if constexpr (SMODE == kScaleGroup) {
      const __half* const sc0 = static_cast<const __half*>(jb.scales);
      const __half* const mn0 = jb.mins;
      const int M = jb.M, G = jb.G;
#pragma unroll
      for (int q = 0; q < 2 * kRowsBlk / 32; ++q) {
        const int idx = q * 32 + lane, row = idx & (kRowsBlk - 1), which = idx / kRowsBlk;
        const int grow = rb * kRowsBlk + row;
        const bool ok = grow < M;
        const __half* src = (which ? mn0 : sc0) + (ok ? (size_t)grow * G + (size_t)st * S : 0);
        const uint32_t d = sb + cw + row * SA::SROW + which * (S * 2);
        if constexpr (S == 4)
          cp_async8(d, src, ok ? 8u : 0u);
        else
          cp_async4(d, src, ok ? 4u : 0u);
      }
    } else if constexpr (SMODE == kScaleRow) {
#pragma unroll
      for (int q = 0; q < kRowsBlk / 32; ++q) {
        const int row = q * 32 + lane, grow = rb * kRowsBlk + row;
        const bool ok = grow < jb.M;
        cp_async4(sb + cw + row * 4, static_cast<const float*>(jb.scales) + (ok ? grow : 0), ok ? 4u : 0u);
      }
    }
    cp_async_arrive(bar);
  };
  // x' records of the CTA's unit ordinal i into stage `slot` (after the
  // preceding grid: they come from the x' preparation launch)
  auto fill_x = [&](int slot, int i) {
    const int u = u0 + i;
    const TmaJob& jb = a.job[job_of(a, u)];
    const int st = (u - jb.unit0) % jb.spb;
    const bool fs = FA != FB && jb.fsel;
    bulk_g2s(ring_s + slot * SLOT + (fs ? SB::XOFF : SA::XOFF), jb.xq + (size_t)st * XB, XB, full0 + 8 * slot);
  };

  // the first stages' weights (never written by the preceding grid), one warp per stage
  const int first = nunits < NS ? nunits : NS;
  if (warp < first) fill(warp, warp, true);
  // x' records, y, partial sums and counters may be written by the preceding grid
  asm volatile("griddepcontrol.wait;" ::: "memory");
  if (warp < first && lane == 0) fill_x(warp, warp);
  if (threadIdx.x == 0) flast = first - 1;

  // ---- unit walk (job, row block, stage)
  int j = job_of(a, u0), rb, st;
  {
    const TmaJob& jb = a.job[j];
    const int v = u0 - jb.unit0;
    rb = v / jb.spb;
    st = v - rb * jb.spb;
  }
  int seg0 = st;  // first stage of this CTA's part of the current row block
  int rl[2];      // the thread's two rows within the warp's 16 (the order depends on the format)
  const uint32_t blane = (uint32_t)(lane & (LP - 1)) * 16;
  float jts = 0.f;
  int jM = 0, jnrb = 1, jspb = 1;
  bool jfs = false;
  auto load_job = [&]() {
    const TmaJob& jb = a.job[j];
    jts = jb.tensor_scale;
    jM = jb.M;
    jnrb = jb.n_rb;
    jspb = jb.spb;
    jfs = FA != FB && jb.fsel;
    rl[0] = jfs ? row_perm<FB>(rq) : row_perm<FA>(rq);
    rl[1] = rl[0] + 8;
  };
  load_job();

  float y[NT][2][YT];
#pragma unroll
  for (int i = 0; i < NT; ++i)
#pragma unroll
    for (int u = 0; u < YT; ++u) y[i][0][u] = y[i][1][u] = 0.f;
  auto tok = [&](int i, int u) { return TPT == 4 ? 4 * i + c : 8 * i + 2 * c + u; };
  auto holds = [&](int t) { return t < N && (LP == 32 || c == 0); };

  // End of this CTA's part of row block rb (stages seg0..st): y when the
  // part is the whole row block; else the part's sums go to the workspace
  // and the warp whose arrival completes the row block adds every part in
  // stage order and writes y.
  auto finish = [&]() {
    const TmaJob& jb = a.job[j];
    if (!(seg0 == 0 && st == jspb - 1)) {
      const size_t rstride = (size_t)kRowsBlk * N;
      float* const pbase = jb.partials + ((size_t)rb * jspb * kRowsBlk + warp * kWarpRows) * N;
      float* const part = pbase + (size_t)seg0 * rstride;
#pragma unroll
      for (int hh = 0; hh < 2; ++hh)
#pragma unroll
        for (int i = 0; i < NT; ++i)
#pragma unroll
          for (int u = 0; u < YT; ++u)
            if (holds(tok(i, u))) __stcg(part + (size_t)rl[hh] * N + tok(i, u), y[i][hh][u]);
      __threadfence();
      __syncwarp();
      const unsigned R0 = (unsigned)(jb.unit0 + rb * jspb);
      const int cf = cta_of_unit(R0, U, P), cl = cta_of_unit(R0 + jspb - 1, U, P);
      unsigned last = 0;
      if (lane == 0) {
        unsigned* cnt = a.counters + jb.tile0 + rb * kWarps + warp;
        last = atomicAdd(cnt, 1u) == (unsigned)(cl - cf);
        if (last) atomicExch(cnt, 0u);
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (!last) return;
      __threadfence();
#pragma unroll
      for (int i = 0; i < NT; ++i)
#pragma unroll
        for (int u = 0; u < YT; ++u) y[i][0][u] = y[i][1][u] = 0.f;
      for (int cc = cf; cc <= cl; ++cc) {
        const int s0 = max(cta_first_unit(cc, U, P), (int)R0) - (int)R0;
        const float* p = pbase + (size_t)s0 * rstride;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
#pragma unroll
          for (int i = 0; i < NT; ++i)
#pragma unroll
            for (int u = 0; u < YT; ++u)
              if (holds(tok(i, u))) y[i][hh][u] += __ldcg(p + (size_t)rl[hh] * N + tok(i, u));
      }
    }
#pragma unroll
    for (int hh = 0; hh < 2; ++hh) {
      const int grow = rb * kRowsBlk + warp * kWarpRows + rl[hh];
      if (grow >= jM) continue;
      const float bv = jb.bias ? jb.bias[grow] : 0.f;
      if (a.world > 0) {
        // the row goes straight into every rank's copy of the whole y (peer stores over NVLink)
        const size_t base = (size_t)jb.row0 + grow;
        for (int pr = 0; pr < a.world; ++pr) {
          float* yp = reinterpret_cast<float*>(a.peer[pr] + jb.yoff);
#pragma unroll
          for (int i = 0; i < NT; ++i)
#pragma unroll
            for (int u = 0; u < YT; ++u)
              if (holds(tok(i, u))) yp[(size_t)tok(i, u) * jb.m_full + base] = y[i][hh][u] + bv;
        }
      } else {
#pragma unroll
        for (int i = 0; i < NT; ++i)
#pragma unroll
          for (int u = 0; u < YT; ++u)
            if (holds(tok(i, u))) jb.y[(size_t)tok(i, u) * jM + grow] = y[i][hh][u] + bv;
      }
    }
  };

  int slot = 0;
  uint32_t phase = 0;
  bool live = true;
  for (int it = 0; it < nunits; ++it) {
    if (live && !mbar_wait(full0 + 8 * slot, phase, &abort_flag)) {
      live = false;
      if (lane == 0) {
        abort_flag = 1;
        atomicExch(a.status, (unsigned)PF_ERR_TIMEOUT);
      }
    }
    if (live) {
      const unsigned char* stg = base + (size_t)slot * SLOT;
      if (jfs)
        unit_body<FB, NT, LP, SMODE, TPT>(stg + warp * kWarpRows * SB::ROW, stg + SB::CW + warp * kWarpRows * SB::SROW,
                                          stg + SB::XOFF, rl, c, blane, jts, y);
      else
        unit_body<FA, NT, LP, SMODE, TPT>(stg + warp * kWarpRows * SA::ROW, stg + SA::CW + warp * kWarpRows * SA::SROW,
                                          stg + SA::XOFF, rl, c, blane, jts, y);
      // done with this stage: the last warp to finish it refills it
      __syncwarp();
      unsigned last = 0;
      if (lane == 0) {
        __threadfence_block();
        last = atomicAdd(&scnt[slot], 1u) == (unsigned)(kWarps - 1);
        if (last) {
          atomicExch(&scnt[slot], 0u);
          __threadfence_block();
        }
      }
      last = __shfl_sync(0xffffffffu, last, 0);
      if (last && it + NS < nunits) {
        fill(slot, it + NS, false);
        if (lane == 0) atomicMax(&flast, it + NS);
      }
    }
    if (++slot == NS) {
      slot = 0;
      phase ^= 1u;
    }
    const bool row_end = st == jspb - 1;
    if (row_end || it == nunits - 1) {
      if (live) finish();
#pragma unroll
      for (int i = 0; i < NT; ++i)
#pragma unroll
        for (int u = 0; u < YT; ++u) y[i][0][u] = y[i][1][u] = 0.f;
    }
    if (++st == jspb) {
      st = 0;
      if (++rb == jnrb) {
        rb = 0;
        if (++j < a.n_jobs) load_job();
      }
    }
    if (row_end) seg0 = 0;
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
  __syncthreads();
  if (abort_flag && threadIdx.x == 0) {
    // after a timeout: bounded waits on the stages still being filled
    volatile int keep_waiting = 0;
    for (int k = max(flast - NS + 1, 0); k <= flast; ++k) mbar_wait(full0 + 8 * (k % NS), (k / NS) & 1, &keep_waiting);
  }
  // (after a timeout too: the epochs of the ranks stay in step; the status word records it)
  signal_done();
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

// CTAs per SM of one launch (PF_TMA_CTAS_PER_SM=1 gives each CTA the whole
// SM's shared memory).
int ctas_per_sm() {
  static int v = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* e = getenv("PF_TMA_CTAS_PER_SM");
    v = (e && atoi(e) == 1) ? 1 : 2;
  });
  return v;
}

// Ring depth set by an environment variable (tuning sweeps), else `dflt`.
int ring_knob(const char* name, int dflt, int most) {
  const char* e = getenv(name);
  const int v = e ? atoi(e) : dflt;
  return v < 1 ? 1 : (v > most ? most : v);
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

int stage_groups(int fmt) { return is_int4(fmt) ? 2 : 4; }

// The shared-memory opt-in of kernel `kern`, once per device; `done` is the
// kernel's own per-device flags.
cudaError_t opt_in_smem(const void* kern, int bytes, bool (&done)[64]) {
  static std::mutex mu;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> lock(mu);
  if (dev < 0 || dev >= 64 || !done[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
    if (e != cudaSuccess) return e;
    if (dev >= 0 && dev < 64) done[dev] = true;
  }
  return cudaSuccess;
}

// A launch that may begin while the preceding kernel of the stream finishes
// (programmatic dependent launch; the kernel waits with griddepcontrol.wait).
cudaError_t launch_pdl(const void* fn, dim3 grid, dim3 block, size_t smem, cudaStream_t s, void** args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelExC(&cfg, fn, args);
}

// Tensor map of one job's packed rows: boxes of one row block (128 rows) x one stage.
template <int FMT>
CUresult encode_rows(CUtensorMap* m, const void* codes, int row_words, int M) {
  using F = TmaFmt<FMT>;
  cuuint64_t dims[2] = {(cuuint64_t)row_words, (cuuint64_t)M};
  cuuint64_t strides[1] = {(cuuint64_t)row_words * 4};
  cuuint32_t box[2] = {(cuuint32_t)(F::S * F::WPG), (cuuint32_t)kRowsBlk};
  cuuint32_t estr[2] = {1, 1};
  return encode_fn()(m, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(codes), dims, strides, box, estr,
                     CU_TENSOR_MAP_INTERLEAVE_NONE, F::SW128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                     CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
}

template <int FA, int FB, int NT, int LP, int SMODE, int TPT>
cudaError_t launch_one(TmaArgs& a, const void* const* codes, const int* row_words, cudaStream_t s) {
  using XR = XRec<NT, LP, TPT>;
  constexpr int S = TmaFmt<FA>::S;
  constexpr int XB = S * XR::R;
  static_assert(XB % 128 == 0, "x' stage must keep the ring stages 128-byte aligned");
  constexpr uint32_t SLOT = MixSlot<FA, FB, SMODE, XB>::BYTES;
  if (!encode_fn()) return cudaErrorNotSupported;
  TmaMaps maps;
  for (int k = 0; k < a.n_jobs; ++k) {
    const CUresult r = a.job[k].fsel ? encode_rows<FB>(&maps.m[k], codes[k], row_words[k], a.job[k].M)
                                     : encode_rows<FA>(&maps.m[k], codes[k], row_words[k], a.job[k].M);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  }
  for (int k = a.n_jobs; k < kTmaMaxJobs; ++k) maps.m[k] = maps.m[0];

  const int cps = ctas_per_sm();
  int P = sm_count() * cps;
  if (P > a.n_units) P = a.n_units;
  if (P < 1) P = 1;
  const int budget = smem_budget(cps);
  a.xstage = XB;
  // ring stages per CTA (PF_TMA_NS, default as many as fit)
  int NS = (int)(((uint32_t)budget - 1024u) / (SLOT + 8u));
  const int ns_want = ring_knob("PF_TMA_NS", kMaxStages, kMaxStages);
  if (NS > ns_want) NS = ns_want;
  if (NS > kMaxStages) NS = kMaxStages;
  if (NS < 2) return cudaErrorInvalidConfiguration;
  a.NS = NS;
  a.XS = 0;
  const size_t smem = 1024 + (size_t)NS * SLOT + (size_t)NS * 8;

  auto kern = gemv_tma_kernel<FA, FB, NT, LP, SMODE, TPT>;
  static bool opted[64] = {false};  // this instantiation's opt-in, per device
  cudaError_t e = opt_in_smem(reinterpret_cast<const void*>(kern), smem_budget(1) + 1024, opted);
  if (e != cudaSuccess) return e;
  void* args[2] = {&maps, &a};
  e = launch_pdl(reinterpret_cast<const void*>(kern), dim3(P), dim3(kThreadsT), smem, s, args);
  if (e == cudaSuccess) note_launch();
  return e;
}

template <int FA, int FB, int NT, int LP, int TPT>
cudaError_t launch_sm(TmaArgs& a, int smode, const void* const* codes, const int* rw, cudaStream_t s) {
  if constexpr (FA == PF_FMT_INT4 || FA == PF_FMT_INT2) {
    if (smode == kScaleRow) return launch_one<FA, FB, NT, LP, kScaleRow, TPT>(a, codes, rw, s);
    return launch_one<FA, FB, NT, LP, kScaleTensor, TPT>(a, codes, rw, s);
  } else {
    return launch_one<FA, FB, NT, LP, kScaleGroup, TPT>(a, codes, rw, s);
  }
}

// Up to 4 tokens: fp16 hi / lo halves of x' (4 tokens per MMA tile); more:
// one fp16 per token (8 per tile), half the MMAs and x' reads per token.
// The x' record layout follows the same choice (tma_xrec_bytes).
template <int FA, int FB = FA>
cudaError_t launch_fmt(TmaArgs& a, int smode, const void* const* codes, const int* rw, cudaStream_t s) {
  if (a.N == 1) return launch_sm<FA, FB, 1, 8, 4>(a, smode, codes, rw, s);
  if (a.N <= 4) return launch_sm<FA, FB, 1, 32, 4>(a, smode, codes, rw, s);
  if (a.N <= 8) return launch_sm<FA, FB, 1, 32, 8>(a, smode, codes, rw, s);
  return launch_sm<FA, FB, 2, 32, 8>(a, smode, codes, rw, s);
}

template <int NT, int LP, int TPT>
cudaError_t launch_prep_frag(XPrepArgs& a, int blocks, cudaStream_t s) {
  void* args[1] = {&a};
  cudaError_t e = launch_pdl(reinterpret_cast<const void*>(xprep_frag_kernel<NT, LP, TPT>), dim3(blocks),
                             dim3(kThreadsT), 0, s, args);
  if (e == cudaSuccess) note_launch();
  return e;
}

}  // namespace

int tma_block_rows() { return kRowsBlk; }

int row_words_of_tma(int fmt, int K) {
  switch (fmt) {
    case PF_FMT_INT4_G128: return (K / 128) * 16;
    case PF_FMT_INT3_G128: return (K / 128) * 13;
    case PF_FMT_INT2_G128: return (K / 128) * 8;
    case PF_FMT_INT4: return K / 8;
    case PF_FMT_INT3: return 3 * K / 32;
    case PF_FMT_INT2: return K / 16;
    default: return 0;
  }
}
int tma_stage_groups(int fmt) { return stage_groups(fmt); }

size_t tma_xrec_bytes(int N) {
  if (N <= 1) return XRec<1, 8, 4>::R;
  if (N <= 4) return XRec<1, 32, 4>::R;
  if (N <= 8) return XRec<1, 32, 8>::R;
  return XRec<2, 32, 8>::R;
}

bool tma_eligible(const TmaWeight& w) {
  const int f = w.format;
  if (!(f == PF_FMT_INT4_G128 || f == PF_FMT_INT3_G128 || f == PF_FMT_INT2_G128 || f == PF_FMT_INT4 ||
        f == PF_FMT_INT2))
    return false;
  if (w.K <= 0 || w.K % 512 != 0 || w.M <= 0) return false;
  if (reinterpret_cast<uintptr_t>(w.codes) % 16) return false;
  const uintptr_t sal = is_group_int_format(f) ? (uintptr_t)(stage_groups(f) * 2) : 4;
  if (w.scales && reinterpret_cast<uintptr_t>(w.scales) % sal) return false;
  if (w.mins && reinterpret_cast<uintptr_t>(w.mins) % sal) return false;
  if (w.had_block != 0) {
    if (w.had_block > 512 || (w.had_block & (w.had_block - 1)) || w.K % w.had_block) return false;
    if (!w.signs || reinterpret_cast<uintptr_t>(w.signs) % 4) return false;
  }
  return encode_fn() != nullptr;
}

int tma_tiles(const TmaWeight& w) { return ((w.M + kRowsBlk - 1) / kRowsBlk) * kWarps; }

size_t tma_partial_bytes(const TmaWeight& w, int N) {
  const size_t n_rb = (w.M + kRowsBlk - 1) / kRowsBlk;
  const size_t spb = (size_t)(w.K / 128) / stage_groups(w.format);
  if (spb <= 1) return 0;
  const size_t b = n_rb * spb * kRowsBlk * (size_t)N * sizeof(float);
  return (b + 255) / 256 * 256;
}

int launch_xprep_frag(XPrepJob* xj, int count, int N, int x_dtype, cudaStream_t s, cudaError_t* err) {
  *err = cudaSuccess;
  if (count < 1 || count > kXPrepMaxJobs || N < 1 || N > kMaxGemvTokens) return PF_ERR_INVALID_ARGUMENT;
  XPrepArgs a;
  memset(&a, 0, sizeof(a));
  int blocks = 0;
  for (int k = 0; k < count; ++k) {
    if (xj[k].K <= 0 || xj[k].K % kPrepCols) return PF_ERR_SHAPE;
    xj[k].blk0 = blocks;
    blocks += xj[k].K / kPrepCols;
    a.xj[k] = xj[k];
  }
  a.n_xj = count;
  a.N = N;
  a.x_dtype = x_dtype;
  cudaError_t e;
  if (N == 1)
    e = launch_prep_frag<1, 8, 4>(a, blocks, s);
  else if (N <= 4)
    e = launch_prep_frag<1, 32, 4>(a, blocks, s);
  else if (N <= 8)
    e = launch_prep_frag<1, 32, 8>(a, blocks, s);
  else
    e = launch_prep_frag<2, 32, 8>(a, blocks, s);
  if (e != cudaSuccess) {
    *err = e;
    return PF_ERR_CUDA;
  }
  return PF_OK;
}

int launch_gemv_tma(const TmaWeight* ws, const TmaIO* io, int count, int N, void* workspace, char* partials,
                    const pf_peers* peers, cudaStream_t s, cudaError_t* err) {
  *err = cudaSuccess;
  if (count < 1 || count > kTmaMaxJobs || N < 1 || N > kMaxGemvTokens) return PF_ERR_INVALID_ARGUMENT;
  // one format, or the group-128 INT3 and INT2 pair (same stage width)
  const int fa = ws[0].format;
  int fb = fa;
  for (int k = 1; k < count; ++k)
    if (ws[k].format != fa) fb = ws[k].format;
  const bool mixed = fb != fa;
  if (mixed && !((fa == PF_FMT_INT3_G128 && fb == PF_FMT_INT2_G128) || (fa == PF_FMT_INT2_G128 && fb == PF_FMT_INT3_G128)))
    return PF_ERR_INVALID_ARGUMENT;
  TmaArgs a;
  memset(&a, 0, sizeof(a));
  const void* codes[kTmaMaxJobs];
  int rw[kTmaMaxJobs];
  unsigned* counters = static_cast<unsigned*>(workspace);
  char* part = partials;
  int unit0 = 0, tile0 = 0;
  for (int k = 0; k < count; ++k) {
    const TmaWeight& w = ws[k];
    TmaJob& jb = a.job[k];
    if ((w.format != fa && w.format != fb) || !io[k].xq) return PF_ERR_INVALID_ARGUMENT;
    jb.scales = w.scales;
    jb.mins = static_cast<const __half*>(w.mins);
    jb.xq = io[k].xq;
    jb.tensor_scale = w.tensor_scale;
    jb.bias = io[k].bias;
    jb.y = io[k].y;
    jb.M = w.M;
    jb.K = w.K;
    jb.G = w.K / 128;
    jb.n_rb = (w.M + kRowsBlk - 1) / kRowsBlk;
    jb.spb = jb.G / stage_groups(w.format);
    jb.unit0 = unit0;
    jb.tile0 = tile0;
    // INT3 is always the launch's first format when mixed
    jb.fsel = mixed ? (w.format == PF_FMT_INT2_G128 ? 1 : 0) : 0;
    jb.yoff = io[k].yoff;
    jb.m_full = io[k].m_full;
    jb.row0 = io[k].row0;
    jb.partials = reinterpret_cast<float*>(part);
    part += tma_partial_bytes(w, N);
    unit0 += jb.n_rb * jb.spb;
    tile0 += tma_tiles(w);
    codes[k] = w.codes;
    rw[k] = row_words_of_tma(w.format, w.K);
  }
  if ((unsigned long long)unit0 * (unsigned long long)(sm_count() * ctas_per_sm() + 1) >= (1ull << 32))
    return PF_ERR_SHAPE;
  if ((size_t)tile0 > kWsDoneSlot) return PF_ERR_SHAPE;
  a.n_jobs = count;
  a.n_units = unit0;
  a.N = N;
  a.counters = counters;
  a.status = counters + kWsStatusSlot;
  a.done = counters + kWsDoneSlot;
  if (peers) {
    if (peers->world < 1 || peers->world > kMaxPeers) return PF_ERR_INVALID_ARGUMENT;
    a.world = peers->world;
    a.rank = peers->rank;
    for (int p = 0; p < peers->world; ++p) a.peer[p] = static_cast<unsigned char*>(peers->bases[p]);
  }
  cudaError_t e;
  if (mixed) {
    e = launch_fmt<PF_FMT_INT3_G128, PF_FMT_INT2_G128>(a, kScaleGroup, codes, rw, s);
  } else {
    switch (fa) {
      case PF_FMT_INT4_G128: e = launch_fmt<PF_FMT_INT4_G128>(a, kScaleGroup, codes, rw, s); break;
      case PF_FMT_INT3_G128: e = launch_fmt<PF_FMT_INT3_G128>(a, kScaleGroup, codes, rw, s); break;
      case PF_FMT_INT2_G128: e = launch_fmt<PF_FMT_INT2_G128>(a, kScaleGroup, codes, rw, s); break;
      case PF_FMT_INT4:
        e = launch_fmt<PF_FMT_INT4>(a, ws[0].scales ? kScaleRow : kScaleTensor, codes, rw, s);
        break;
      case PF_FMT_INT2:
        e = launch_fmt<PF_FMT_INT2>(a, ws[0].scales ? kScaleRow : kScaleTensor, codes, rw, s);
        break;
      default: return PF_ERR_UNSUPPORTED;
    }
  }
  if (e != cudaSuccess) {
    *err = e;
    return PF_ERR_CUDA;
  }
  return PF_OK;
}

}  // namespace pfb
