// Streaming fused dequant-GEMV for the INT formats (N <= 16 tokens): one
// launch computes y = x W^T for up to four weights ("jobs") of one format.
//
// Work unit = (job, 128-row block, stage of S groups of 128 columns), dealt to
// the CTAs stream-K style in stage-major order: a CTA's consecutive units
// share a column stage, so it transforms only the one or two stages of x it
// needs (x' = forward block RWHT of x, scaled and split for the tensor cores)
// straight into shared memory; there is no separate x-prep launch.
//
// CTA = 8 warps, two CTAs per SM.  Every warp owns 16 rows of each unit and
// streams them itself through a private ring of shared-memory slots: lane 0
// issues the 2-D TMA copy of its 16 x (S groups) tile of packed codes (L2
// evict-first), all lanes copy the tile's fp16 scales / zero points with
// cp.async, and the copies themselves arrive on the slot's mbarrier.  A warp
// refills a slot it has just consumed, so warps never wait for each other
// except at the x' preparation barrier, and the weights of the first slots
// are requested before the kernel waits for the preceding grid
// (programmatic dependent launch; packed weights and scales are never written
// by a kernel that precedes a GEMV in this library).
//
// Compute: the unit's code words are read into registers, every code pair
// becomes one AND (exact subnormal fp16 q 2^(p-24)), and mma.sync m16n8k16
// multiplies two groups at a time against the B fragments of x' (fp16 hi / lo
// halves of x' in the two columns of each token).
// Per 128-column group:  sum w x' = s 2^E Q + m Sx  with  Q = sum q x'/2^E.
// Each unit's 16 x N partial sums per warp go to the workspace (plain
// stores); combine_kernel, launched next as a programmatic dependent, adds a
// row block's stage partials in a fixed order (deterministic) and writes y.
// Every wait is bounded (2 s, %globaltimer): on expiry the kernel records
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
constexpr int kMaxXSlots = 3;

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

__device__ __forceinline__ const TmaJob& job_ref(const TmaArgs& a, int j) {
  return j == 0 ? a.job[0] : j == 1 ? a.job[1] : j == 2 ? a.job[2] : a.job[3];
}

// Job holding global unit u.
__device__ __forceinline__ int job_of(const TmaArgs& a, int u) {
  int j = 0;
#pragma unroll
  for (int k = 1; k < kTmaMaxJobs; ++k)
    if (k < a.n_jobs && u >= a.job[k].unit0) j = k;
  return j;
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
// fragments of x' 2^(14 - p - E) split into fp16 hi + lo, and {Sx, 1024 2^E}.
// Tokens t >= N write zeros.  Every global load is issued before any is used.
template <int NT, int LP, int E, int TPT>
__device__ __forceinline__ void prep_chunk(const TmaJob& jb, int N, int x_dtype, int col0, int g_lo, int g_hi, int t,
                                           unsigned char* xslot, float* scratch, int lane, const LaneCols& lc) {
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
  const int j8 = lane >> 2, c = lane & 3;
  // B-fragment lane of the token's column: hi at column 2 (t % 4), lo next to
  // it, or the token's own column t % 8
  const int fl = TPT == 4 ? 8 * (t & 3) + c : 4 * (t & 7) + c;
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
    unsigned char* rec = xslot + (size_t)(g - g_lo) * XR::R;
    unsigned char* fr = rec + (tile * 4 + (j8 >> 1)) * LP * 16 + (j8 & 1) * 8;
    *reinterpret_cast<uint2*>(fr + fl * 16) = make_uint2(hw[0], hw[1]);
    if (TPT == 4) *reinterpret_cast<uint2*>(fr + (fl + 4) * 16) = make_uint2(lw[0], lw[1]);
    if (lane == 0) *reinterpret_cast<float2*>(rec + XR::FRAG + t * 16) = make_float2(sg, 1024.f * pow2f(eg));
  }
  __syncwarp();
}

template <int FMT, int NT, int LP, int SMODE, int TPT>
__global__ void __launch_bounds__(kThreadsT, 2)
    gemv_tma_kernel(const __grid_constant__ CUtensorMap map0, const __grid_constant__ CUtensorMap map1,
                    const __grid_constant__ CUtensorMap map2, const __grid_constant__ CUtensorMap map3,
                    const __grid_constant__ TmaArgs a) {
  using F = TmaFmt<FMT>;
  using L = WarpSlot<FMT, SMODE>;
  using XR = XRec<NT, LP, TPT>;
  constexpr int S = F::S;
  constexpr int kOffset = IntFmt<FMT>::kOffset;
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
  if (threadIdx.x >= 32 && threadIdx.x < 32 + kTmaMaxJobs) {
    const int k = threadIdx.x - 32;
    const CUtensorMap* m = k == 0 ? &map0 : k == 1 ? &map1 : k == 2 ? &map2 : &map3;
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
  }

  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ int abort_flag;
  unsigned char* const base = smem_raw + ((1024u - (smem_u32(smem_raw) & 1023u)) & 1023u);
  const int NS = a.NS, XS = a.XS;
  constexpr uint32_t X = S * XR::R;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  unsigned char* const ring = base + (size_t)warp * NS * L::BYTES;  // this warp's slots
  unsigned char* const xarea = base + (size_t)kWarps * NS * L::BYTES;
  float* const scratch = reinterpret_cast<float*>(xarea + XS * X) + warp * a.chunk_max;
  const uint32_t full0 = smem_u32(reinterpret_cast<float*>(xarea + XS * X) + kWarps * a.chunk_max) + warp * NS * 8;

  if (threadIdx.x == 0) abort_flag = 0;
  if (lane == 0) {
    for (int s = 0; s < NS; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(full0 + 8 * s), "r"(33));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  const unsigned U = (unsigned)a.n_units, P = gridDim.x, cta = blockIdx.x;
  const int u0 = (int)(cta * U / P), u1 = (int)((cta + 1) * U / P);  // U * P < 2^32 (host-checked)
  const int nunits = u1 - u0;
  if (nunits <= 0) return;
  const int N = a.N;
  const int c = lane & 3, rq = lane >> 2;

  // ---- load side: this warp's next unit to request (job, stage, row block)
  int fj = job_of(a, u0), fst, frb;
  {
    const TmaJob& jb = job_ref(a, fj);
    const int v = u0 - jb.unit0;
    fst = v / jb.n_rb;
    frb = v - fst * jb.n_rb;
  }
  const CUtensorMap* fmap = nullptr;
  const __half* fsc = nullptr;
  const __half* fmn = nullptr;
  int fM = 0, fG = 0, fnrb = 1, fspb = 1;
  auto load_fjob = [&]() {
    const TmaJob& jb = job_ref(a, fj);
    fmap = fj == 0 ? &map0 : fj == 1 ? &map1 : fj == 2 ? &map2 : &map3;
    fsc = static_cast<const __half*>(jb.scales);
    fmn = jb.mins;
    fM = jb.M;
    fG = jb.G;
    fnrb = jb.n_rb;
    fspb = jb.spb;
  };
  load_fjob();
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  const uint32_t ring_s = smem_u32(ring);
  // request the next unit into `slot` (which this warp no longer reads)
  auto request = [&](int slot) {
    const uint32_t sb = ring_s + slot * L::BYTES, bar = full0 + 8 * slot;
    const int row0 = frb * kRowsBlk + warp * kWarpRows;
    __syncwarp();
    if (lane == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_expect(bar, L::W);
      tma_2d(sb, fmap, fst * S * F::WPG, row0, bar, policy);
    }
    if constexpr (SMODE == kScaleGroup) {
      const int row = lane & 15, which = lane >> 4, grow = row0 + row;
      const bool ok = grow < fM;
      const __half* src = (which ? fmn : fsc) + (ok ? (size_t)grow * fG + (size_t)fst * S : 0);
      const uint32_t d = sb + L::W + row * L::SROW + which * (S * 2);
      if constexpr (S == 4)
        cp_async8(d, src, ok ? 8u : 0u);
      else
        cp_async4(d, src, ok ? 4u : 0u);
    } else if constexpr (SMODE == kScaleRow) {
      const int grow = row0 + (lane & 15);
      const bool ok = lane < 16 && grow < fM;
      if (lane < 16)
        cp_async4(sb + L::W + lane * 4, reinterpret_cast<const float*>(fsc) + (ok ? grow : 0), ok ? 4u : 0u);
    }
    cp_async_arrive(bar);
    if (++frb == fnrb) {
      frb = 0;
      if (++fst == fspb) {
        fst = 0;
        ++fj;
        if (fj < a.n_jobs) load_fjob();
      }
    }
  };
  // the first two units (weights and scales never come from the preceding
  // grid); the rest of the ring is requested after the x' preparation, when
  // the copy engine's queue has drained
  int requested = 0;
  for (; requested < 2 && requested < NS && requested < nunits; ++requested) request(requested);

  // ---- compute side: unit walk (job, stage, row block) and its x' runs
  int j = job_of(a, u0), st, rb;
  {
    const TmaJob& jb = job_ref(a, j);
    const int v = u0 - jb.unit0;
    st = v / jb.n_rb;
    rb = v - st * jb.n_rb;
  }
  int rl[2];  // the thread's two rows within the warp's 16
  rl[0] = row_perm<FMT>(rq);
  rl[1] = rl[0] + 8;
  LaneCols lc;
  {
    int lo, hi, p;
    frag_cols2(FMT, c, 2 * rq, lo, hi, p);
    lc.col[0] = lo; lc.col[1] = hi; lc.p[0] = p;
    frag_cols2(FMT, c, 2 * rq + 1, lo, hi, p);
    lc.col[2] = lo; lc.col[3] = hi; lc.p[1] = p;
  }
  const uint32_t blane = (uint32_t)(lane & (LP - 1)) * 16;

  // x' windows over the CTA's runs (consecutive units with one job and stage);
  // XS runs are resident, run r in slot r % XS
  int nruns;
  {
    const int jl = job_of(a, u1 - 1);
    const TmaJob& jf = job_ref(a, j);
    const TmaJob& jL = job_ref(a, jl);
    nruns = (jL.run0 + (u1 - 1 - jL.unit0) / jL.n_rb) - (jf.run0 + (u0 - jf.unit0) / jf.n_rb) + 1;
  }
  int pj = j, pst = st;  // (job, stage) of the next run to prepare
  int win_end = 0;
  auto prep_window = [&](int r0) {
    const int r1 = (r0 + XS < nruns) ? r0 + XS : nruns;
    const int tslots = LP == 8 ? 1 : TPT * NT;
    int task = 0;
    for (int r = r0; r < r1; ++r) {
      const TmaJob& jb = job_ref(a, pj);
      const int b = jb.had_block;
      const int E = b > 256 ? 16 : (b > 128 ? 8 : 4);
      const int Cc = 32 * E;
      const int g_lo = pst * S, g_hi = g_lo + S;
      const int nchunk = (S * 128) / Cc > 0 ? (S * 128) / Cc : 1;
      const int cbase = ((g_lo * 128) / Cc) * Cc;
      unsigned char* xslot = xarea + (size_t)(r % XS) * X;
      for (int ci = 0; ci < nchunk; ++ci)
        for (int t = 0; t < tslots; ++t, ++task) {
          if (task % kWarps != warp) continue;
          const int col0 = cbase + ci * Cc;
          if (E == 4)
            prep_chunk<NT, LP, 4, TPT>(jb, N, a.x_dtype, col0, g_lo, g_hi, t, xslot, scratch, lane, lc);
          else if (E == 8)
            prep_chunk<NT, LP, 8, TPT>(jb, N, a.x_dtype, col0, g_lo, g_hi, t, xslot, scratch, lane, lc);
          else
            prep_chunk<NT, LP, 16, TPT>(jb, N, a.x_dtype, col0, g_lo, g_hi, t, xslot, scratch, lane, lc);
        }
      if (++pst == jb.spb) {
        pst = 0;
        ++pj;
      }
    }
    win_end = r1;
  };

  // x may be written by the preceding grid, and so may the workspace and y
  asm volatile("griddepcontrol.wait;" ::: "memory");
  prep_window(0);
  for (; requested < NS && requested < nunits; ++requested) request(requested);
  __syncthreads();

  // the current job's fields, reloaded when the walk enters the next job
  float* jpart = nullptr;
  float jts = 0.f;
  int jM = 0, jnrb = 1, jspb = 1;
  auto load_job = [&]() {
    const TmaJob& jb = job_ref(a, j);
    jpart = jb.partials;
    jts = jb.tensor_scale;
    jM = jb.M;
    jnrb = jb.n_rb;
    jspb = jb.spb;
  };
  load_job();

  int run = 0, xslot = 0, slot = 0;
  uint32_t phase = 0;
  bool live = true;
  for (int it = 0; it < nunits; ++it) {
    if (run >= win_end) {  // same decision in every warp of the CTA
      __syncthreads();
      prep_window(win_end);
      __syncthreads();
    }
    const unsigned char* stg = ring + slot * L::BYTES;
    const unsigned char* xs = xarea + xslot * X;
    if (live && !mbar_wait(full0 + 8 * slot, phase, &abort_flag)) {
      live = false;
      if (lane == 0) {
        abort_flag = 1;
        atomicExch(a.status, (unsigned)PF_ERR_TIMEOUT);
      }
    }
    if (live) {
      float y[NT][2][YT];
#pragma unroll
      for (int i = 0; i < NT; ++i)
#pragma unroll
        for (int u = 0; u < YT; ++u) y[i][0][u] = y[i][1][u] = 0.f;
#pragma unroll
      for (int pp = 0; pp < S / 2; ++pp) {
        // scales / zero points of the pair's two groups, then their code words
        uint32_t sv2[2], mv2[2];
        float frow[2];
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const unsigned char* sp = stg + L::W + rl[hh] * L::SROW;
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
            load_words<FMT>(stg, rl[hh], 2 * pp + gg, c, raw);
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
              mma16816(acc[gg][i], r0.h(4 * jp + 2), r1.h(4 * jp + 2), r0.h(4 * jp + 3), r1.h(4 * jp + 3), bq.z,
                       bq.w);
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

      if (jspb == 1) {
        const TmaJob& jb = job_ref(a, j);
#pragma unroll
        for (int hh = 0; hh < 2; ++hh) {
          const int grow = rb * kRowsBlk + warp * kWarpRows + rl[hh];
          if (grow >= jM) continue;
          const float bv = jb.bias ? jb.bias[grow] : 0.f;
#pragma unroll
          for (int i = 0; i < NT; ++i)
#pragma unroll
            for (int u = 0; u < YT; ++u) {
              const int t = TPT == 4 ? 4 * i + c : 8 * i + 2 * c + u;
              if (t < N && (LP == 32 || c == 0)) jb.y[(size_t)t * jM + grow] = y[i][hh][u] + bv;
            }
        }
      } else {
        // the stage partial sums; the combine kernel adds them in stage order
        float* part = jpart + (((size_t)rb * jspb + st) * kRowsBlk + warp * kWarpRows) * N;
#pragma unroll
        for (int hh = 0; hh < 2; ++hh)
#pragma unroll
          for (int i = 0; i < NT; ++i)
#pragma unroll
            for (int u = 0; u < YT; ++u) {
              const int t = TPT == 4 ? 4 * i + c : 8 * i + 2 * c + u;
              if (t < N && (LP == 32 || c == 0)) __stcg(part + (size_t)rl[hh] * N + t, y[i][hh][u]);
            }
      }
    }
    if (live && requested < nunits) {  // refill the slot just consumed
      request(slot);
      ++requested;
    }
    if (++slot == NS) {
      slot = 0;
      phase ^= 1u;
    }
    if (++rb == jnrb) {
      rb = 0;
      ++run;
      if (++xslot == XS) xslot = 0;
      if (++st == jspb) {
        st = 0;
        ++j;
        if (j < a.n_jobs) load_job();
      }
    }
  }
  if (!live && lane == 0) {
    // after a timeout: bounded waits on this warp's tiles that may still be in flight
    volatile int keep_waiting = 0;
    for (int k = requested > NS ? requested - NS : 0; k < requested; ++k)
      mbar_wait(full0 + 8 * (k % NS), (k / NS) & 1, &keep_waiting);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// y = the sum of a job's stage partial sums (+ bias).  A block covers 32
// consecutive (row, token) elements of one job; warp w adds stages w, w + 8,
// ... (all its loads in flight at once) and warp 0 adds the eight warp sums
// in warp order, so the result is the same on every run.  Launched after the
// GEMV as a programmatic dependent: it lets its own dependents start at once
// and waits for the GEMV's partial sums.
constexpr int kCombineWarps = 8;

__global__ void __launch_bounds__(kCombineWarps * 32) combine_kernel(const __grid_constant__ TmaArgs a) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  __shared__ float red[kCombineWarps][32];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int N = a.N;
  int blk = blockIdx.x, j = 0;
  for (; j < a.n_jobs; ++j) {
    const int nb = (((a.job[j].M + kRowsBlk - 1) / kRowsBlk) * kRowsBlk * N + 31) / 32;
    if (blk < nb) break;
    blk -= nb;
  }
  if (j >= a.n_jobs) return;
  const TmaJob& jb = a.job[j];
  if (jb.spb <= 1) return;
  const int e = blk * 32 + lane;  // element row * N + t of the job
  const int row = e / N, t = e - row * N;
  const bool valid = row < jb.M;
  float acc = 0.f;
  if (valid) {
    const int rb = row / kRowsBlk, r = row - rb * kRowsBlk;
    const float* p = jb.partials + (size_t)rb * jb.spb * kRowsBlk * N + (size_t)r * N + t;
    const size_t stride = (size_t)kRowsBlk * N;
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) {
      const int st = warp + k * kCombineWarps;
      v[k] = st < jb.spb ? __ldcg(p + st * stride) : 0.f;
    }
#pragma unroll
    for (int k = 0; k < 8; ++k) acc += v[k];
    for (int st = warp + 8 * kCombineWarps; st < jb.spb; st += kCombineWarps) acc += __ldcg(p + st * stride);
  }
  red[warp][lane] = acc;
  __syncthreads();
  if (warp == 0 && valid) {
    float s = 0.f;
#pragma unroll
    for (int w = 0; w < kCombineWarps; ++w) s += red[w][lane];
    jb.y[(size_t)t * jb.M + row] = s + (jb.bias ? jb.bias[row] : 0.f);
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

// Prep chunk (columns) of a rotation block size.
int chunk_cols(int had_block) { return had_block > 256 ? 512 : (had_block > 128 ? 256 : 128); }

// Global run index (job, stage) of unit u.
int run_of(const TmaArgs& a, int u) {
  int j = 0;
  for (int k = 1; k < a.n_jobs; ++k)
    if (u >= a.job[k].unit0) j = k;
  return a.job[j].run0 + (u - a.job[j].unit0) / a.job[j].n_rb;
}

template <int FMT, int NT, int LP, int SMODE, int TPT>
cudaError_t launch_one(TmaArgs& a, const void* const* codes, const int* row_words, cudaStream_t s) {
  using F = TmaFmt<FMT>;
  using L = WarpSlot<FMT, SMODE>;
  using XR = XRec<NT, LP, TPT>;
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  CUtensorMap maps[kTmaMaxJobs];
  for (int k = 0; k < a.n_jobs; ++k) {
    cuuint64_t dims[2] = {(cuuint64_t)row_words[k], (cuuint64_t)a.job[k].M};
    cuuint64_t strides[1] = {(cuuint64_t)row_words[k] * 4};
    cuuint32_t box[2] = {(cuuint32_t)(F::S * F::WPG), (cuuint32_t)kWarpRows};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(&maps[k], CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(codes[k]), dims, strides, box,
                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    F::SW128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  }
  for (int k = a.n_jobs; k < kTmaMaxJobs; ++k) maps[k] = maps[0];

  const int cps = ctas_per_sm();
  int P = sm_count() * cps;
  if (P > a.n_units) P = a.n_units;
  if (P < 1) P = 1;
  int max_runs = 1;
  for (int cta = 0; cta < P; ++cta) {
    const int u0 = (int)((long long)cta * a.n_units / P), u1 = (int)((long long)(cta + 1) * a.n_units / P);
    if (u1 <= u0) continue;
    const int r = run_of(a, u1 - 1) - run_of(a, u0) + 1;
    if (r > max_runs) max_runs = r;
  }
  const int budget = smem_budget(cps);
  const uint32_t X = F::S * XR::R;
  const uint32_t fixed = (uint32_t)kWarps * a.chunk_max * 4 + 1024;
  const uint32_t per_stage = (uint32_t)kWarps * (L::BYTES + 8);
  int XS = max_runs < kMaxXSlots ? max_runs : kMaxXSlots;
  while (XS > 1 && fixed + XS * X + 3 * per_stage > (uint32_t)budget) --XS;
  int NS = (int)(((uint32_t)budget - fixed - XS * X) / per_stage);
  if (NS > kMaxStages) NS = kMaxStages;
  if (NS < 2) return cudaErrorInvalidConfiguration;
  a.NS = NS;
  a.XS = XS;
  const size_t smem = (size_t)1024 + (size_t)kWarps * NS * L::BYTES + (size_t)XS * X +
                      (size_t)kWarps * a.chunk_max * 4 + (size_t)kWarps * NS * 8;

  auto kern = gemv_tma_kernel<FMT, NT, LP, SMODE, TPT>;
  {
    // the shared-memory opt-in is per device
    static std::mutex mu;
    static bool done[64] = {false};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64 || !done[dev]) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, smem_budget(1) + 1024);
      if (e != cudaSuccess) return e;
      if (dev >= 0 && dev < 64) done[dev] = true;
    }
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(P);
  cfg.blockDim = dim3(kThreadsT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, maps[0], maps[1], maps[2], maps[3], (const TmaArgs)a);
  if (e == cudaSuccess) note_launch();
  return e;
}

template <int FMT, int NT, int LP, int TPT>
cudaError_t launch_sm(TmaArgs& a, int smode, const void* const* codes, const int* rw, cudaStream_t s) {
  if constexpr (FMT == PF_FMT_INT4 || FMT == PF_FMT_INT2) {
    if (smode == kScaleRow) return launch_one<FMT, NT, LP, kScaleRow, TPT>(a, codes, rw, s);
    return launch_one<FMT, NT, LP, kScaleTensor, TPT>(a, codes, rw, s);
  } else {
    return launch_one<FMT, NT, LP, kScaleGroup, TPT>(a, codes, rw, s);
  }
}

template <int FMT>
cudaError_t launch_fmt(TmaArgs& a, int smode, const void* const* codes, const int* rw, cudaStream_t s) {
  // up to 4 tokens: fp16 hi / lo halves of x' (4 tokens per MMA tile); more:
  // one fp16 per token (8 per tile), half the MMAs and x' reads per token
  if (a.N == 1) return launch_sm<FMT, 1, 8, 4>(a, smode, codes, rw, s);
  if (a.N <= 4) return launch_sm<FMT, 1, 32, 4>(a, smode, codes, rw, s);
  if (a.N <= 8) return launch_sm<FMT, 1, 32, 8>(a, smode, codes, rw, s);
  return launch_sm<FMT, 2, 32, 8>(a, smode, codes, rw, s);
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

size_t tma_partial_bytes(const TmaWeight& w, int N) {
  const size_t n_rb = (w.M + kRowsBlk - 1) / kRowsBlk;
  const size_t spb = (size_t)(w.K / 128) / stage_groups(w.format);
  if (spb <= 1) return 0;
  const size_t b = n_rb * spb * kRowsBlk * (size_t)N * sizeof(float);
  return (b + 255) / 256 * 256;
}

int launch_gemv_tma(const TmaWeight* ws, const TmaIO* io, int count, int N, int x_dtype, void* workspace,
                    cudaStream_t s, cudaError_t* err) {
  *err = cudaSuccess;
  if (count < 1 || count > kTmaMaxJobs || N < 1 || N > kMaxGemvTokens) return PF_ERR_INVALID_ARGUMENT;
  TmaArgs a;
  memset(&a, 0, sizeof(a));
  const void* codes[kTmaMaxJobs];
  int rw[kTmaMaxJobs];
  unsigned* counters = static_cast<unsigned*>(workspace);
  char* part = static_cast<char*>(workspace) + kWsCounterBytes;
  int unit0 = 0, run0 = 0, chunk = 128;
  const int fmt = ws[0].format;
  const int S = stage_groups(fmt);
  for (int k = 0; k < count; ++k) {
    const TmaWeight& w = ws[k];
    TmaJob& jb = a.job[k];
    if (w.format != fmt) return PF_ERR_INVALID_ARGUMENT;
    jb.scales = w.scales;
    jb.mins = static_cast<const __half*>(w.mins);
    jb.tensor_scale = w.tensor_scale;
    jb.x = io[k].x;
    jb.signs = w.had_block ? w.signs : nullptr;
    jb.had_block = w.had_block;
    jb.had_rscale = w.had_block ? 1.f / sqrtf((float)w.had_block) : 1.f;
    jb.bias = io[k].bias;
    jb.y = io[k].y;
    jb.M = w.M;
    jb.K = w.K;
    jb.G = w.K / 128;
    jb.n_rb = (w.M + kRowsBlk - 1) / kRowsBlk;
    jb.spb = jb.G / S;
    jb.unit0 = unit0;
    jb.run0 = run0;
    jb.partials = reinterpret_cast<float*>(part);
    part += tma_partial_bytes(w, N);
    unit0 += jb.n_rb * jb.spb;
    run0 += jb.spb;
    const int cc = chunk_cols(w.had_block);
    if (cc > chunk) chunk = cc;
    codes[k] = w.codes;
    rw[k] = row_words_of_tma(fmt, w.K);
  }
  if ((unsigned long long)unit0 * (unsigned long long)(sm_count() * ctas_per_sm() + 1) >= (1ull << 32))
    return PF_ERR_SHAPE;
  a.n_jobs = count;
  a.n_units = unit0;
  a.N = N;
  a.x_dtype = x_dtype;
  a.chunk_max = chunk;
  a.status = counters + kWsStatusSlot;
  cudaError_t e;
  switch (fmt) {
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
  if (e != cudaSuccess) {
    *err = e;
    return PF_ERR_CUDA;
  }
  int blocks = 0, split = 0;
  for (int k = 0; k < count; ++k) {
    blocks += (((a.job[k].M + kRowsBlk - 1) / kRowsBlk) * kRowsBlk * N + 31) / 32;
    split |= a.job[k].spb > 1;
  }
  if (split) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(blocks);
    cfg.blockDim = dim3(kCombineWarps * 32);
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    e = cudaLaunchKernelEx(&cfg, combine_kernel, (const TmaArgs)a);
    if (e == cudaSuccess) note_launch();
    if (e != cudaSuccess) {
      *err = e;
      return PF_ERR_CUDA;
    }
  }
  return PF_OK;
}

}  // namespace pfb
