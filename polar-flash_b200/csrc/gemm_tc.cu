// Dequant-GEMM on the 5th-generation tensor cores (tcgen05 + TMEM) for
// batches of more than 16 tokens: Y[N][M] = X'[N][K] * W_hat^T, W_hat decoded
// from the packed payload inside the kernel (INT4 / INT3 / INT2 group-128
// asymmetric, E8 RVQ2, and, in the persistent kernel only, recursive polar
// with block 8 at 1.75 bpw), X' = the forward block RWHT of X in fp16 with a
// power-of-two scale per token (the same fusion identity as the GEMV).
//
// CTA = 128 weight rows x 128 tokens, one CTA per SM, ten warps:
//   warp 0    TMA producer: the x' tile of each 128-column stage, two
//             64-column boxes, 128B-swizzled (K-major canonical layout).
//   warps 1-8 two groups of four dequantising alternate stages, one weight
//             row per thread: the row's packed group is loaded with plain
//             loads one own stage ahead (and into L2 four ahead), every code
//             pair that sits 16 bits apart in its word becomes an fp16x2 with
//             one shift + LOP3, and w = q s + m is one fp16 FMA of the exact
//             code (one rounding; E8: s2 r[i2] + s1 r[i1], s1 r[i1] exact), written
//             into the A tile in the swizzled K-major layout (columns permuted
//             within each group, x' permuted alike); then the epilogue
//             (tcgen05.ld of their 32 TMEM lanes, token scale, bias).
//   warp 9    allocates 128 TMEM columns and issues tcgen05.mma (kind::f16,
//             M = 128, N = 128, K = 16; fp32 accumulator in TMEM) from one
//             lane; tcgen05.commit releases each stage's smem slot.
// Every wait is bounded (2 s on %globaltimer): on expiry the kernel records
// PF_ERR_TIMEOUT in the status word, skips the remaining waits, still frees
// its TMEM and exits.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <string.h>

#include <mutex>

#include "common.cuh"
#include "decode.cuh"
#include "gemv.cuh"

namespace pfb {

namespace {

constexpr int kBM = 128;  // weight rows per CTA (MMA M)
constexpr int kBN = 128;  // tokens per CTA (MMA N)
constexpr int kBK = 128;  // columns per stage: one scale group
constexpr int kStages = 3;
constexpr int kDqWarps = 8;                          // two groups of four: alternate stages
constexpr int kGemmThreads = (kDqWarps + 2) * 32;  // + TMA warp + MMA warp
constexpr int kMmaWarp = kDqWarps + 1;
constexpr uint32_t kATile = kBM * kBK * 2;  // two 64-column swizzle atoms of 16 KB
constexpr uint32_t kBTile = kBN * kBK * 2;
constexpr uint32_t kStageBytes = kATile + kBTile;
constexpr unsigned long long kGemmWaitNs = 2000000000ull;
constexpr int kTmemCols = 128;

struct GemmArgs {
  int fmt;
  const void* codes;
  const __half* scales;  // INT: [M][G]; E8: [M][G][2]
  const __half* mins;    // INT: [M][G]
  int M, K, N, G, row_words;
  const float* tok_scale;  // [N] 2^-e of the fp16 x'
  const float* bias;
  float* y;  // [N][M]
  unsigned* status;
  // persistent stream-K kernel: tiles per token column, (tile, group) units,
  // per-tile arrival counters (zero, left zero) and 2 partial tiles per CTA
  int n_mb;
  long long units;
  unsigned* counters;
  float* partials;
  // recursive polar: the radius scale (applied with the token scale) and the
  // learned angle table [7][64], or nullptr for the uniform angle grid
  float r_scale;
  const float* angles;
};

__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait on an mbarrier phase: try_wait with the hardware's own
// time limit per attempt, then the abort flag and the 2 s bound.
__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity, const volatile int* abort_flag) {
  unsigned long long t0 = 0;
  for (;;) {
    uint32_t done;
    asm volatile(
        "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
        : "=r"(done)
        : "r"(bar), "r"(parity)
        : "memory");
    if (done) return true;
    if (*abort_flag) return false;
    const unsigned long long t = gtime();
    if (t0 == 0)
      t0 = t;
    else if (t - t0 > kGemmWaitNs)
      return false;
  }
}

// K-major operand descriptor, 128B swizzle, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t kmajor_desc(uint32_t saddr) {
  return (uint64_t)((saddr & 0x3FFFFu) >> 4) | (1ull << 16) | ((uint64_t)(1024u >> 4) << 32) | (1ull << 46) |
         (2ull << 61);
}

// Instruction descriptor: fp16 A and B (K-major), fp32 D, M = 128, N = n
// (a multiple of 16 up to kBN).
__host__ __device__ constexpr uint32_t gemm_idesc(int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kBM >> 4) << 24);
}

// Byte offset of 16-byte chunk c (8 fp16, columns 8c..8c+7 of the stage) of
// tile row r: two 64-column atoms, rows of 128 bytes, chunk index XOR (r & 7).
__device__ __forceinline__ uint32_t a_chunk(int r, int c) {
  return (uint32_t)((c >> 3) * (kBM * 128) + r * 128 + (((c & 7) ^ (r & 7)) << 4));
}

// Column order of the A tile inside each 128-column group: slot s holds the
// code of group column gemm_slot_col(fmt, s).  Code pairs that sit 16 bits
// apart in their word fill one fp16x2 slot pair, so a pair decodes with one
// shift and one LOP3; the fp16 x' is written in the same order.
__host__ __device__ __forceinline__ int gemm_slot_col(int fmt, int s) {
  const int hi = s & 1;
  if (fmt == PF_FMT_INT4_G128) return 8 * (s >> 3) + ((s & 7) >> 1) + 4 * hi;
  if (fmt == PF_FMT_INT2_G128) return 16 * (s >> 4) + ((s & 15) >> 1) + 8 * hi;
  if (fmt == PF_FMT_INT3_G128) {
    const int p = s >> 1;
    return p < 60 ? 10 * (p / 5) + (p % 5) + 5 * hi : 120 + (p - 60) + 4 * hi;
  }
  return s;
}

// fp16x2 (q0, q1) from a word holding the codes at bits 0.. and 16.., already
// masked: 1024 + q as fp16 bits, minus 1024 (exact).
__device__ __forceinline__ __half2 pair_fp16(uint32_t masked) {
  const uint32_t b = masked | 0x64006400u;
  return __hsub2(*reinterpret_cast<const __half2*>(&b), __half2half2(__ushort_as_half(0x6400)));
}

template <int FMT>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                   const __grid_constant__ GemmArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ uint64_t bars[3 * kStages + 1];
  __shared__ uint32_t tmem_base_slot;
  __shared__ int abort_flag;
  // E8 roots as 8 fp16, indices 240..255 zero, four copies per root in
  // consecutive 16-byte slots: lane l reads copy l & 3, so the lanes of one
  // 8-lane phase of a 16-byte load mostly fall in different bank groups
  __shared__ uint4 roots16[256 * 4];
  __shared__ float tscale[kBN];

  unsigned char* const base = smem_raw + ((1024u - (su32(smem_raw) & 1023u)) & 1023u);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kBM, n0 = blockIdx.y * kBN;
  const uint32_t bfull0 = su32(&bars[0]), afull0 = su32(&bars[kStages]), free0 = su32(&bars[2 * kStages]);
  const uint32_t accbar = su32(&bars[3 * kStages]);

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kStages; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bfull0 + 8 * s));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(afull0 + 8 * s), "r"(kBM));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(free0 + 8 * s));
    }
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(accbar));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
  }
  if (FMT == PF_FMT_E8_RVQ2_G128) {
    for (int k = threadIdx.x; k < 256; k += blockDim.x) {
      float r[8];
      if (k < 240) {
        e8_root(k, r);
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) r[q] = 0.f;
      }
      uint32_t h[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const __half2 v = __floats2half2_rn(r[2 * q], r[2 * q + 1]);
        h[q] = *reinterpret_cast<const uint32_t*>(&v);
      }
#pragma unroll
      for (int c = 0; c < 4; ++c) roots16[4 * k + c] = make_uint4(h[0], h[1], h[2], h[3]);
    }
  }
  for (int t = threadIdx.x; t < kBN; t += blockDim.x) tscale[t] = (n0 + t < a.N) ? a.tok_scale[n0 + t] : 0.f;
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base_slot)),
                 "r"(kTmemCols));
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = tmem_base_slot;
  const int G = a.G;
  // tokens of this CTA, rounded up to the MMA's N granularity
  const int nv = a.N - n0 < kBN ? a.N - n0 : kBN;
  const int nmma = (nv + 15) & ~15;

  if (warp == 0) {
    // ------------------------------------------------------------ x' via TMA
    if (lane == 0) {
      for (int s = 0; s < G; ++s) {
        const int slot = s % kStages;
        if (s >= kStages && !bar_wait(free0 + 8 * slot, ((s / kStages) - 1) & 1, &abort_flag)) {
          abort_flag = 1;
          atomicExch(a.status, (unsigned)PF_ERR_TIMEOUT);
          break;
        }
        const uint32_t dst = su32(base + slot * kStageBytes + kATile), bar = bfull0 + 8 * slot;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(kBTile) : "memory");
#pragma unroll
        for (int h = 0; h < 2; ++h)
          asm volatile(
              "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
              "[%4];" ::"r"(dst + h * (kBN * 128)),
              "l"(reinterpret_cast<uint64_t>(&xmap)), "r"(s * kBK + h * 64), "r"(n0), "r"(bar)
              : "memory");
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      for (int s = 0; s < G; ++s) {
        const int slot = s % kStages;
        const uint32_t par = (s / kStages) & 1;
        if (!bar_wait(afull0 + 8 * slot, par, &abort_flag) || !bar_wait(bfull0 + 8 * slot, par, &abort_flag)) {
          abort_flag = 1;
          atomicExch(a.status, (unsigned)PF_ERR_TIMEOUT);
          break;
        }
        asm volatile("tcgen05.fence::after_thread_sync;");
        const uint32_t sa = su32(base + slot * kStageBytes), sb = sa + kATile;
#pragma unroll
        for (int k = 0; k < kBK / 16; ++k) {
          const uint32_t off = (k >> 2) * (kBM * 128) + (k & 3) * 32;
          const uint64_t da = kmajor_desc(sa + off), db = kmajor_desc(sb + off);
          const uint32_t acc = (s > 0 || k > 0) ? 1u : 0u;
          asm volatile(
              "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(
                  tmem),
              "l"(da), "l"(db), "r"(gemm_idesc(nmma)), "r"(acc));
        }
        asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(free0 +
                                                                                                        8 * slot)
                     : "memory");
      }
      asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(accbar)
                   : "memory");
    }
  } else {
    // ------------------------------------------------ dequant rows, epilogue
    const int grp = (warp - 1) >> 2;       // this group dequantises stages s with s % 2 == grp
    const int r = 32 * (warp & 3) + lane;  // tile row == this warp's TMEM lanes
    const int grow = m0 + r;
    const bool rvalid = grow < a.M;
    const int growc = rvalid ? grow : 0;
    bool live = true;
    constexpr int kGroupBytes = FMT == PF_FMT_INT4_G128 ? 64 : (FMT == PF_FMT_INT3_G128 ? 52 : 32);
    constexpr int kL2Ahead = 4;  // own stages requested into L2 ahead of the register loads
    const size_t rowb = FMT == PF_FMT_E8_RVQ2_G128 ? (size_t)a.K / 4 : (size_t)a.row_words * 4;
    const char* rowp = static_cast<const char*>(a.codes) + (size_t)growc * rowb;
    uint32_t pw[16];  // packed words of the next own stage (E8: 32 index bytes)
    uint32_t psc = 0;  // its fp16 scale and zero point (E8: the two stage scales)
#pragma unroll
    for (int q = 0; q < 16; ++q) pw[q] = 0u;
    auto l2_ahead = [&](int g) {
      if (g >= G) return;
      const char* p = rowp + (size_t)g * kGroupBytes;
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p));
      asm volatile("prefetch.global.L2 [%0];" ::"l"(p + kGroupBytes - 1));
    };
    auto load_group = [&](int g) {
      if constexpr (FMT == PF_FMT_E8_RVQ2_G128) {
        psc = __ldg(reinterpret_cast<const unsigned*>(a.scales + ((size_t)growc * G + g) * 2));
      } else {
        const uint32_t lo = __half_as_ushort(__ldg(a.scales + (size_t)growc * G + g));
        const uint32_t hi = __half_as_ushort(__ldg(a.mins + (size_t)growc * G + g));
        psc = lo | (hi << 16);
      }
      const char* p = rowp + (size_t)g * kGroupBytes;
      if constexpr (FMT == PF_FMT_INT3_G128) {
#pragma unroll
        for (int q = 0; q < 13; ++q) pw[q] = __ldg(reinterpret_cast<const uint32_t*>(p) + q);
      } else {
#pragma unroll
        for (int q = 0; q < kGroupBytes / 16; ++q) {
          const uint4 v = __ldg(reinterpret_cast<const uint4*>(p) + q);
          pw[4 * q] = v.x; pw[4 * q + 1] = v.y; pw[4 * q + 2] = v.z; pw[4 * q + 3] = v.w;
        }
      }
    };
    for (int k = 0; k < kL2Ahead; ++k) l2_ahead(grp + 2 * k);
    if (grp < G) load_group(grp);
    for (int s = grp; s < G; s += 2) {
      const int slot = s % kStages;
      unsigned char* at = base + slot * kStageBytes;
      // this stage's codes and scales; the group's next stage is requested into
      // registers before decoding, the ones after it into L2
      uint32_t cw[16];
#pragma unroll
      for (int q = 0; q < 16; ++q) cw[q] = pw[q];
      const uint32_t sc = psc;
      l2_ahead(s + 2 * kL2Ahead);
      if (s + 2 < G) load_group(s + 2);
      if (live && s >= kStages && !bar_wait(free0 + 8 * slot, ((s / kStages) - 1) & 1, &abort_flag)) {
        live = false;
        if (lane == 0) {
          abort_flag = 1;
          atomicExch(a.status, (unsigned)PF_ERR_TIMEOUT);
        }
      }
      if (!live) continue;
      if constexpr (FMT == PF_FMT_E8_RVQ2_G128) {
        // w = s1 r[i1] + s2 r[i2] in one fp16 FMA (s1 r[i1] is exact: r in {0, +-1/2, +-1})
        const __half2 s1 = __half2half2(__ushort_as_half((unsigned short)(sc & 0xFFFFu)));
        const __half2 s2 = __half2half2(__ushort_as_half((unsigned short)(sc >> 16)));
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          const uint32_t wv = cw[c >> 1] >> (16 * (c & 1));
          const uint32_t i1 = wv & 0xFFu, i2 = (wv >> 8) & 0xFFu;
          const uint4 ra = roots16[4 * i1 + (lane & 3)], rb = roots16[4 * i2 + (lane & 3)];
          const uint32_t* pa = reinterpret_cast<const uint32_t*>(&ra);
          const uint32_t* pb = reinterpret_cast<const uint32_t*>(&rb);
          uint4 o;
          uint32_t* ov = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const __half2 h = __hfma2(s2, *reinterpret_cast<const __half2*>(&pb[e]),
                                      __hmul2(s1, *reinterpret_cast<const __half2*>(&pa[e])));
            ov[e] = *reinterpret_cast<const uint32_t*>(&h);
          }
          *reinterpret_cast<uint4*>(at + a_chunk(r, c)) = o;  // rows past M: row 0's codes, never written out
        }
      } else {
        // w = q s + m as one fp16 FMA of the exact code (the stored fp16 s and m)
        const __half2 sx = __half2half2(__ushort_as_half((unsigned short)(sc & 0xFFFFu)));
        const __half2 mx = __half2half2(__ushort_as_half((unsigned short)(sc >> 16)));
        uint32_t g3[13];
        if constexpr (FMT == PF_FMT_INT3_G128) {
#pragma unroll
          for (int t = 0; t < 12; ++t) g3[t] = (cw[t] & 0x0000FFFFu) | ((cw[t] << 1) & 0xFFFF0000u);
          g3[12] = (cw[12] & 0x0000FFFFu) | ((cw[12] << 4) & 0xFFFF0000u);
        }
#pragma unroll
        for (int c = 0; c < 16; ++c) {
          uint4 o;
          uint32_t* ov = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            uint32_t mk;
            if constexpr (FMT == PF_FMT_INT4_G128) {
              mk = (cw[c] >> (4 * e)) & 0x000F000Fu;
            } else if constexpr (FMT == PF_FMT_INT2_G128) {
              mk = (cw[c >> 1] >> (2 * (4 * (c & 1) + e))) & 0x00030003u;
            } else {
              const int p = 4 * c + e;
              mk = p < 60 ? (g3[p / 5] >> (3 * (p % 5))) & 0x00070007u : (g3[12] >> (3 * (p - 60))) & 0x00070007u;
            }
            const __half2 h = __hfma2(pair_fp16(mk), sx, mx);
            ov[e] = *reinterpret_cast<const uint32_t*>(&h);
          }
          *reinterpret_cast<uint4*>(at + a_chunk(r, c)) = o;  // rows past M: row 0's codes, never written out
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(afull0 + 8 * slot) : "memory");
    }
    // ------------------------------------------------ epilogue (16-column chunks split between the groups)
    bool ok = live;
    if (ok) ok = bar_wait(accbar, 0, &abort_flag);
    ok = __all_sync(0xffffffffu, ok);
    if (ok) {
      asm volatile("tcgen05.fence::after_thread_sync;");
      const uint32_t taddr = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
      const float bv = (rvalid && a.bias) ? a.bias[grow] : 0.f;
#pragma unroll 1
      for (int c0 = 16 * grp; c0 < nmma; c0 += 32) {
        uint32_t v[16];
        asm volatile(
            "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
            : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
              "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
            : "r"(taddr + (uint32_t)c0));
        asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
        if (rvalid) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int t = n0 + c0 + j;
            if (t < a.N) a.y[(size_t)t * a.M + grow] = __uint_as_float(v[j]) * tscale[c0 + j] + bv;
          }
        }
      }
    } else if (lane == 0 && !abort_flag) {
      abort_flag = 1;
      atomicExch(a.status, (unsigned)PF_ERR_TIMEOUT);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// ---------------------------------------------------------------------------
// Variant with the packed codes and scales staged by TMA (shapes whose row
// strides allow 2-D tensor maps).  The producer warp also copies, per box of
// CB groups, the CTA's 128 rows of packed codes, and per box of SB groups their
// scales (and zero points), into double-buffered shared-memory slots; the
// dequant threads read their row from there, so no thread issues a global
// load (one 4-byte load per row per lane was the limit of the plain kernel:
// a warp touched 32 rows, 32 sectors per load).  The A/B ring is two stages.
template <int FMT>
struct TcBox;
template <>
struct TcBox<PF_FMT_INT4_G128> {
  static constexpr int GB = 64, CB = 2, SB = 8, SW = 2;  // group bytes, code / scale box groups, scale bytes
};
// Code boxes whose rows are exactly 128 bytes (INT4, INT2, E8) are loaded
// 128B-swizzled (16-byte chunk j of row r at chunk j ^ (r & 7)), so the 32
// rows a warp reads at one offset fall in eight different bank groups.
template <class B>
__host__ __device__ constexpr bool code_swizzled() { return B::CB * B::GB == 128; }
template <>
struct TcBox<PF_FMT_INT3_G128> {
  static constexpr int GB = 52, CB = 4, SB = 8, SW = 2;
};
template <>
struct TcBox<PF_FMT_INT2_G128> {
  static constexpr int GB = 32, CB = 4, SB = 8, SW = 2;
};
template <>
struct TcBox<PF_FMT_E8_RVQ2_G128> {
  static constexpr int GB = 32, CB = 4, SB = 4, SW = 4;  // scales: (s1, s2) fp16 per group
};
template <>
struct TcBox<PF_FMT_POLAR_RECURSIVE> {  // block 8, 14-bit blocks: 16 blocks = 28 bytes per group, no scales
  static constexpr int GB = 28, CB = 4, SB = 8, SW = 2;
};
// 128 weight rows x 256 tokens per CTA (one N = 256 MMA per k-step, 256 TMEM
// columns), so every decoded weight feeds twice the MACs of a 128-token tile;
// stages of 64 columns (half a scale group, the dequant groups take
// alternate halves) in a three-slot A/B ring.
constexpr int kBN2 = 256;
constexpr int kBK2 = 64;
constexpr int kStages2 = 3;
// Batches of at most kSmallN tokens: the x' box is at most 32 rows (4 KB per
// half-stage instead of 32 KB), so the ring holds seven slots and more
// half-stages are in flight while slots wait on their x' fetch and commit.
constexpr int kSmallN = 32;
constexpr int kStagesSmall = 5;
// Code and scale box slots: two for 256-token tiles; four for small batches,
// whose decode outruns the DRAM latency of two boxes in flight.
__host__ __device__ constexpr int sk_box_slots(int xr) { return xr == kBN2 ? 2 : 4; }
constexpr int kTmemCols2 = 256;
constexpr uint32_t kATile2 = kBM * kBK2 * 2;  // one 64-column swizzle atom

// Token rows of the x' box: 256, or the batch rounded up to 16 when it is
// smaller (the MMA reads no row past that).
__host__ __device__ constexpr int sk_box_rows(int N) { return N >= kBN2 ? kBN2 : ((N + 15) & ~15); }

__device__ __forceinline__ void tma2d_plain(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

// Decodes half H of a row's scale group (A-tile slots 64 H .. 64 H + 63, the
// 16-byte chunks 8 H .. 8 H + 7) from its packed words at cp into the
// half-stage A tile at `at` (one 64-column swizzle atom).
__device__ __forceinline__ __half2 u32_h2(uint32_t v) {
  __half2 h;
  memcpy(&h, &v, 4);
  return h;
}
__device__ __forceinline__ uint32_t h2_u32(__half2 h) {
  uint32_t v;
  memcpy(&v, &h, 4);
  return v;
}

// crow: this row's bytes in the code slot; gb: the group's byte offset in the
// row (logical, before the swizzle).  RC: copies of each root in roots16
// (entry RC k + c), read by lane group c = lane % RC.
template <int FMT, int H, int RC>
__device__ __forceinline__ void sk_decode(const unsigned char* crow, int gb, uint32_t sc, int r, int lane,
                                           unsigned char* at, const uint4* roots16, const float2* ptab) {
  using B = TcBox<FMT>;
  const unsigned char* cp = crow + gb;
  // the eight decoded chunks are kept in registers and stored together at the
  // end, so no A-tile store sits between two of the decode's shared loads
  uint4 ob[8];
  auto store_all = [&]() {
#pragma unroll
    for (int k = 0; k < 8; ++k)  // rows past M: zero codes (TMA fill)
      *reinterpret_cast<uint4*>(at + a_chunk(r, 8 * H + k) - H * (kBM * 128)) = ob[k];
  };
  if constexpr (FMT == PF_FMT_POLAR_RECURSIVE) {
    // Recursive polar, block 8, allocation [3 | 2 2 2 2 | 1 1 | 1]: block c of
    // the group is the 14 bits at bit 14 c of its 28 bytes (MSB first); code
    // fields from the LSB: psi 0, phi1 1, phi0 2, th3 3-4, th2 5-6, th1 7-8,
    // th0 9-10, radius 11-13.  inverse_recursive (polar_quant.py:252-272):
    // (a, b) = R (cos psi, sin psi); (A0, A1, A2, A3) = (a cos phi0,
    // a sin phi0, b cos phi1, b sin phi1); w(2i, 2i + 1) = A_i (cos th_i,
    // sin th_i), with R the radius code (r_scale joins the token scale) and
    // the cos / sin pairs from the angle tables (ptab: column j, code c at
    // 64 j + c).  The block's 8 weights are the 8 columns of A-tile chunk c.
    (void)sc;
    (void)lane;
    (void)roots16;
    uint32_t be[8];
#pragma unroll
    for (int q = 0; q < 7; ++q) be[q] = __byte_perm(*reinterpret_cast<const uint32_t*>(cp + 4 * q), 0u, 0x0123);
    be[7] = 0u;
#pragma unroll
    for (int c = 8 * H; c < 8 * H + 8; ++c) {
      constexpr int kBits = 14;
      const int o = kBits * c, i = o >> 5, sh = o & 31;
      const unsigned long long v = ((unsigned long long)be[i] << 32) | be[i + 1];
      const uint32_t w = (uint32_t)(v >> (64 - sh - kBits)) & 0x3FFFu;
      const float R = (float)(w >> 11);
      const float2 ps = ptab[6 * kPolarTabPerCol + (w & 1u)];
      const float2 f0 = ptab[4 * kPolarTabPerCol + ((w >> 2) & 1u)];
      const float2 f1 = ptab[5 * kPolarTabPerCol + ((w >> 1) & 1u)];
      const float ra = R * ps.x, rb = R * ps.y;
      const float2 t0 = ptab[0 * kPolarTabPerCol + ((w >> 9) & 3u)], t1 = ptab[1 * kPolarTabPerCol + ((w >> 7) & 3u)];
      const float2 t2 = ptab[2 * kPolarTabPerCol + ((w >> 5) & 3u)], t3 = ptab[3 * kPolarTabPerCol + ((w >> 3) & 3u)];
      const float a0 = ra * f0.x, a1 = ra * f0.y, a2 = rb * f1.x, a3 = rb * f1.y;
      const uint4 o4 = make_uint4(h2_u32(__floats2half2_rn(a0 * t0.x, a0 * t0.y)),
                                  h2_u32(__floats2half2_rn(a1 * t1.x, a1 * t1.y)),
                                  h2_u32(__floats2half2_rn(a2 * t2.x, a2 * t2.y)),
                                  h2_u32(__floats2half2_rn(a3 * t3.x, a3 * t3.y)));
      ob[c - 8 * H] = o4;
    }
    store_all();
    return;
  }
  uint32_t cw[16];
  if constexpr (FMT == PF_FMT_INT3_G128) {
#pragma unroll
    for (int q = 0; q < 13; ++q) cw[q] = *reinterpret_cast<const uint32_t*>(cp + 4 * q);
    cw[13] = cw[14] = cw[15] = 0u;
  } else {
#pragma unroll
    for (int q = 0; q < B::GB / 16; ++q) {
      const int off = code_swizzled<B>() ? ((((gb >> 4) + q) ^ (r & 7)) << 4) : gb + 16 * q;
      const uint4 v = *reinterpret_cast<const uint4*>(crow + off);
      cw[4 * q] = v.x; cw[4 * q + 1] = v.y; cw[4 * q + 2] = v.z; cw[4 * q + 3] = v.w;
    }
#pragma unroll
    for (int q = B::GB / 4; q < 16; ++q) cw[q] = 0u;
  }
  if constexpr (FMT == PF_FMT_E8_RVQ2_G128) {
    // w = s1 r[i1] + s2 r[i2] in one fp16 FMA (s1 r[i1] is exact: r in {0, +-1/2, +-1})
    const __half2 s1 = __half2half2(__ushort_as_half((unsigned short)(sc & 0xFFFFu)));
    const __half2 s2 = __half2half2(__ushort_as_half((unsigned short)(sc >> 16)));
#pragma unroll
    for (int c = 8 * H; c < 8 * H + 8; ++c) {
      const uint32_t wv = cw[c >> 1] >> (16 * (c & 1));
      const uint32_t i1 = wv & 0xFFu, i2 = (wv >> 8) & 0xFFu;
      const uint4 ra = roots16[RC * i1 + (lane % RC)], rb = roots16[RC * i2 + (lane % RC)];
      const uint4 o = make_uint4(h2_u32(__hfma2(s2, u32_h2(rb.x), __hmul2(s1, u32_h2(ra.x)))),
                                 h2_u32(__hfma2(s2, u32_h2(rb.y), __hmul2(s1, u32_h2(ra.y)))),
                                 h2_u32(__hfma2(s2, u32_h2(rb.z), __hmul2(s1, u32_h2(ra.z)))),
                                 h2_u32(__hfma2(s2, u32_h2(rb.w), __hmul2(s1, u32_h2(ra.w)))));
      ob[c - 8 * H] = o;
    }
    store_all();
  } else {
    // w = q s + m as one fp16 FMA of the exact code (the stored fp16 s and m)
    const __half2 sx = __half2half2(__ushort_as_half((unsigned short)(sc & 0xFFFFu)));
    const __half2 mx = __half2half2(__ushort_as_half((unsigned short)(sc >> 16)));
    uint32_t g3[13];
    if constexpr (FMT == PF_FMT_INT3_G128) {
#pragma unroll
      for (int t = 0; t < 12; ++t) g3[t] = (cw[t] & 0x0000FFFFu) | ((cw[t] << 1) & 0xFFFF0000u);
      g3[12] = (cw[12] & 0x0000FFFFu) | ((cw[12] << 4) & 0xFFFF0000u);
    }
#pragma unroll
    for (int c = 8 * H; c < 8 * H + 8; ++c) {
      uint32_t ov[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        uint32_t mk;
        if constexpr (FMT == PF_FMT_INT4_G128) {
          mk = (cw[c] >> (4 * e)) & 0x000F000Fu;
        } else if constexpr (FMT == PF_FMT_INT2_G128) {
          mk = (cw[c >> 1] >> (2 * (4 * (c & 1) + e))) & 0x00030003u;
        } else {
          const int p = 4 * c + e;
          mk = p < 60 ? (g3[p / 5] >> (3 * (p % 5))) & 0x00070007u : (g3[12] >> (3 * (p - 60))) & 0x00070007u;
        }
        ov[e] = h2_u32(__hfma2(pair_fp16(mk), sx, mx));
      }
      ob[c - 8 * H] = make_uint4(ov[0], ov[1], ov[2], ov[3]);
    }
    store_all();
  }
}

// Stream-K work split of the persistent GEMM: units are (tile, scale group)
// pairs, tile t = nb * n_mb + mb (128 rows x 256 tokens), and CTA c of P takes
// units [U c / P, U (c + 1) / P), so every CTA decodes the same number of
// groups whatever the tile count.  A tile covered by one CTA is written
// straight to y; the CTAs that share a tile store fp32 partial tiles and the
// last of them to arrive sums them in k order (deterministic) and writes y.
__device__ __forceinline__ long long sk_begin(long long U, int P, int c) { return U * c / P; }
__device__ __forceinline__ int sk_cta_of(long long U, int P, long long u) {
  const long long c = ((u + 1) * P - 1) / U;
  return (int)(c < P - 1 ? c : P - 1);
}

// Order of a CTA's segments: the partial ones first (the one ending its
// range, then the one starting it), whole tiles after, so the tiles it shares
// are finished early and their reductions overlap the whole tiles' work.
__device__ __forceinline__ int sk_items(long long ub, long long ue, int G) {
  const long long e0 = (ub / G + 1) * G;
  return e0 >= ue ? 1 : 2 + (int)((((ue - 1) / G) * G - e0) / G);
}
__device__ __forceinline__ void sk_item(long long ub, long long ue, int G, int j, long long* us, long long* ul) {
  const long long e0 = (ub / G + 1) * G;
  if (e0 >= ue) {
    *us = ub;
    *ul = ue;
    return;
  }
  const long long l0 = ((ue - 1) / G) * G;
  const int n = 2 + (int)((l0 - e0) / G);  // segments in range order: 0 = [ub, e0), n - 1 = [l0, ue)
  const bool p_first = ub % G != 0, p_last = ue % G != 0;
  int i;
  if (p_last && j == 0) {
    i = n - 1;
  } else {
    const int k = p_last ? 1 : 0;  // the rest in range order, after the partial ones
    i = (p_first && j == k) ? 0 : j - k;
  }
  if (i == 0) {
    *us = ub;
    *ul = e0;
  } else if (i == n - 1) {
    *us = l0;
    *ul = ue;
  } else {
    *us = e0 + (long long)(i - 1) * G;
    *ul = *us + G;
  }
}

// Two-SM (pair) helpers.
constexpr int kStagesPair = 5;  // A/B ring slots of the pair kernel (32 KB each)

__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Address of the same shared variable in the cluster's CTA 0.
__device__ __forceinline__ uint32_t map_rank0(uint32_t saddr) {
  uint32_t d;
  asm volatile("mapa.shared::cluster.u32 %0, %1, 0;" : "=r"(d) : "r"(saddr));
  return d;
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// One arrival on a barrier of this CTA (kPair: of the pair's first CTA, by
// its cluster address).
template <bool kPair>
__device__ __forceinline__ void bar_arrive_pair(uint32_t bar) {
  if constexpr (kPair)
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(bar) : "memory");
  else
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}
// Completion of this thread's earlier MMAs arrives on `bar` (kPair: on the
// same barrier of both CTAs of the pair).
template <bool kPair>
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  if constexpr (kPair)
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(bar),
        "h"((unsigned short)0x3)
        : "memory");
  else
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}
// x' half-tile load of a pair CTA; its bytes count on CTA 0's barrier (cluster address).
__device__ __forceinline__ void tma2d_pair(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
      "[%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}
// Instruction descriptor for an M x N kind::f16 MMA (fp16 A, B K-major, fp32 D).
__host__ __device__ constexpr uint32_t gemm_idesc_m(int m, int n) {
  return (1u << 4) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// Warp roles of the persistent kernel: 0 x' producer, 1-8 dequant, 9 MMA,
// 10-13 epilogue (one per TMEM lane quarter), 14 code and scale producer
// (runs ahead of the x' ring, bounded by the two code / scale slots).
constexpr int kEpiWarp0 = kDqWarps + 2;
constexpr int kCodeWarp = kDqWarps + 6;
constexpr int kSkThreads = (kDqWarps + 7) * 32;

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* v) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// 32 consecutive fp32 accumulator columns of this thread's TMEM lane, one wait.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* f) {
  uint32_t v[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,"
      "%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]), "=r"(v[8]),
        "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]), "=r"(v[16]),
        "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]),
        "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) f[i] = __uint_as_float(v[i]);
}

// kPair: a cluster of two CTAs on two SMs runs each 256-row tile with
// tcgen05.mma.cta_group::2 (M = 256): every CTA decodes its own 128 rows and
// loads half of the x' tile (128 tokens), the first CTA of the pair issues
// the MMAs (reading both CTAs' shared memory) and each CTA's TMEM holds its
// rows' accumulators.  Half the x' bytes per CTA leave room for five stages.
template <int FMT, bool kPair, int kXR>
__global__ void __launch_bounds__(kSkThreads, 1)
    gemm_sk_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap cmap,
                   const __grid_constant__ CUtensorMap smap, const __grid_constant__ CUtensorMap mmap,
                   const __grid_constant__ GemmArgs a) {
  using B = TcBox<FMT>;
  constexpr bool kE8 = FMT == PF_FMT_E8_RVQ2_G128;
  constexpr bool kPolar = FMT == PF_FMT_POLAR_RECURSIVE;  // no scale boxes
  static_assert(!kPair || kXR == kBN2, "pairs run 256-token tiles");
  constexpr int kSt = kPair ? kStagesPair : (kXR == kBN2 ? kStages2 : kStagesSmall);  // A/B ring slots
  constexpr int kXRows = kPair ? kBN2 / 2 : kXR;        // token rows of this CTA's x' box (at most)
  constexpr uint32_t kSB = kATile2 + kXRows * kBK2 * 2;  // bytes per stage
  constexpr int kRowsT = kPair ? 2 * kBM : kBM;          // weight rows per tile
  constexpr uint32_t kCodeSlot = kBM * B::CB * B::GB;  // 128 rows x CB groups
  constexpr uint32_t kScaleSlot = kBM * 16;            // 128 rows x SB groups x SW bytes (16)
  constexpr int kCS = kPair ? 2 : sk_box_slots(kXR);     // code (and scale) box slots
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // A/B ring full / free, then code full / free and scale full / free (kCS
  // slots each), then accumulator full and TMEM-buffer empty (two each)
  __shared__ uint64_t bars[2 * kSt + 4 * kCS + 4];
  __shared__ uint32_t tmem_base_slot;
  __shared__ int abort_flag;
  __shared__ unsigned arrival;
  constexpr int kRC = kPair ? 4 : 8;  // copies of each root (the pair kernel has less shared memory to spare)
  __shared__ uint4 roots16[kE8 ? 256 * kRC : 1];
  __shared__ float2 ptab[kPolar ? 7 * kPolarTabPerCol : 1];  // polar cos / sin by angle column and code
  __shared__ float etscale[kBN2];  // token scales of the epilogue's current segment

  unsigned char* const base = smem_raw + ((1024u - (su32(smem_raw) & 1023u)) & 1023u);
  unsigned char* const codes = base + kSt * kSB;  // [kCS][kCodeSlot]
  unsigned char* const scl = codes + kCS * kCodeSlot;           // [kCS][kScaleSlot] (+ [kCS][kScaleSlot] mins)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // full0: one barrier per ring slot for the decoded A stage and the x' bytes
  const uint32_t full0 = su32(&bars[0]), free0 = su32(&bars[kSt]);
  const uint32_t cfull0 = su32(&bars[2 * kSt]), cfree0 = cfull0 + 8 * kCS;
  const uint32_t sfull0 = cfree0 + 8 * kCS, sfree0 = sfull0 + 8 * kCS;
  const uint32_t accf0 = sfree0 + 8 * kCS, tempty0 = accf0 + 16;
  const uint32_t rank = kPair ? cta_rank() : 0u;
  // barriers of the pair's first CTA as cluster addresses (own ones without kPair)
  const uint32_t full_l = kPair ? map_rank0(full0) : full0;
  const uint32_t tempty_l = kPair ? map_rank0(tempty0) : tempty0;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kSt; ++s) {
      // the decoding warps (both CTAs' with kPair) and the x' producer's expect-tx
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(full0 + 8 * s),
                   "r"((kPair ? kDqWarps : kDqWarps / 2) + 1));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(free0 + 8 * s));
    }
    for (int s = 0; s < kCS; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(cfull0 + 8 * s));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(cfree0 + 8 * s), "r"(2 * kBM));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sfull0 + 8 * s));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sfree0 + 8 * s), "r"(2 * kBM));
    }
    for (int s = 0; s < 2; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(accf0 + 8 * s));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(tempty0 + 8 * s), "r"(kPair ? 8 : 4));
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&cmap)) : "memory");
    if (!kPolar) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&smap)) : "memory");
    if (!kE8 && !kPolar) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mmap)) : "memory");
  }
  if constexpr (kPolar) {
    const int alloc[8] = {3, 2, 2, 2, 2, 1, 1, 1};
    polar_fill_tables(ptab, 8, alloc, a.angles);
  }
  if constexpr (kE8) {
    for (int k = threadIdx.x; k < 256; k += blockDim.x) {
      float r[8];
      if (k < 240) {
        e8_root(k, r);
      } else {
#pragma unroll
        for (int q = 0; q < 8; ++q) r[q] = 0.f;
      }
      uint32_t h[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        const __half2 v = __floats2half2_rn(r[2 * q], r[2 * q + 1]);
        h[q] = *reinterpret_cast<const uint32_t*>(&v);
      }
#pragma unroll
      for (int c = 0; c < kRC; ++c) roots16[kRC * k + c] = make_uint4(h[0], h[1], h[2], h[3]);
    }
  }
  if (warp == kMmaWarp) {
    if constexpr (kPair) {
      asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base_slot)),
                   "r"(2 * kTmemCols2));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;");
    } else {
      asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(su32(&tmem_base_slot)),
                   "r"(2 * kTmemCols2));
      asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;");
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if constexpr (kPair) cluster_sync();  // both CTAs' barriers initialised before any cross-CTA signal
  asm volatile("tcgen05.fence::after_thread_sync;");
  const uint32_t tmem = tmem_base_slot;
  // stream-K over pairs (kPair) or CTAs
  const int G = a.G, P = kPair ? (int)gridDim.x / 2 : (int)gridDim.x;
  const int sk_id = kPair ? (int)blockIdx.x / 2 : (int)blockIdx.x;
  const long long U = a.units;
  const long long u_begin = sk_begin(U, P, sk_id), u_end = sk_begin(U, P, sk_id + 1);
  const int n_items = sk_items(u_begin, u_end, G);
  // x' bytes landing on one stage's full barrier (kPair: both CTAs' halves)
  const uint32_t xbox_bytes = kPair ? 2u * kXRows * (kBK2 * 2) : (uint32_t)sk_box_rows(a.N) * (kBK2 * 2);

  if (warp == 0) {
    // ------------------------------------------------ producer: x' tiles
    if (lane == 0) {
      // x' and the token scales come from the preparation kernel launched just before
      asm volatile("griddepcontrol.wait;" ::: "memory");
      bool ok = true;
      uint32_t q = 0;  // half-stages issued
      for (int it = 0; it < n_items && ok; ++it) {
        long long us, ul;
        sk_item(u_begin, u_end, G, it, &us, &ul);
        const int t = (int)(us / G), g0 = (int)(us - (long long)t * G), g1 = g0 + (int)(ul - us);
        const int n0 = (t / a.n_mb) * kBN2 + (int)rank * kXRows;
        for (int s = g0; s < g1 && ok; ++s) {
          for (int h = 0; h < 2; ++h, ++q) {
            const uint32_t slot = q % kSt;
            if (q >= kSt && !bar_wait(free0 + 8 * slot, ((q / kSt) - 1) & 1, &abort_flag)) {
              ok = false;
              break;
            }
            const uint32_t dst = su32(base + slot * kSB + kATile2);
            if (rank == 0)
              asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(full0 + 8 * slot),
                           "r"(xbox_bytes)
                           : "memory");
            if constexpr (kPair)
              tma2d_pair(dst, &xmap, (2 * s + h) * kBK2, n0, full_l + 8 * slot);
            else
              tma2d_plain(dst, &xmap, (2 * s + h) * kBK2, n0, full0 + 8 * slot);
          }
        }
      }
      if (!ok) {
        abort_flag = 1;
        atomicExch(a.status, (unsigned)PF_ERR_TIMEOUT);
      }
    }
  } else if (warp == kCodeWarp) {
    // ------------------------------------------------ producer: code and scale boxes
    if (lane == 0) {
      bool ok = true;
      uint32_t kc = 0, ks = 0;  // code boxes and scale boxes issued
      for (int it = 0; it < n_items && ok; ++it) {
        long long us, ul;
        sk_item(u_begin, u_end, G, it, &us, &ul);
        const int t = (int)(us / G), g0 = (int)(us - (long long)t * G), g1 = g0 + (int)(ul - us);
        const int m0 = (t % a.n_mb) * kRowsT + (int)rank * kBM;
        for (int s = g0; s < g1 && ok; ++s) {
          if (s == g0 || s % B::CB == 0) {
            const uint32_t cs = kc % kCS;
            if (kc >= kCS && !bar_wait(cfree0 + 8 * cs, ((kc / kCS) - 1) & 1, &abort_flag)) {
              ok = false;
              break;
            }
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(cfull0 + 8 * cs),
                         "r"(kCodeSlot)
                         : "memory");
            tma2d_plain(su32(codes + cs * kCodeSlot), &cmap, (s - s % B::CB) * (B::GB / 4), m0, cfull0 + 8 * cs);
            ++kc;
          }
          if (!kPolar && (s == g0 || s % B::SB == 0)) {
            const uint32_t ss = ks % kCS;
            if (ks >= kCS && !bar_wait(sfree0 + 8 * ss, ((ks / kCS) - 1) & 1, &abort_flag)) {
              ok = false;
              break;
            }
            asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sfull0 + 8 * ss),
                         "r"(kE8 ? kScaleSlot : 2 * kScaleSlot)
                         : "memory");
            // x in fp16 elements: E8 keeps two scales per group
            const int sx = s - s % B::SB;
            tma2d_plain(su32(scl + ss * kScaleSlot), &smap, kE8 ? 2 * sx : sx, m0, sfull0 + 8 * ss);
            if (!kE8) tma2d_plain(su32(scl + (kCS + ss) * kScaleSlot), &mmap, sx, m0, sfull0 + 8 * ss);
            ++ks;
          }
        }
      }
      if (!ok) {
        abort_flag = 1;
        atomicExch(a.status, (unsigned)PF_ERR_TIMEOUT);
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issue (the pair's first CTA)
    if (lane == 0 && rank == 0) {
      bool ok = true;
      uint32_t q = 0, j = 0;
      for (; (int)j < n_items && ok; ++j) {
        long long us, ul;
        sk_item(u_begin, u_end, G, (int)j, &us, &ul);
        const int t = (int)(us / G), g0 = (int)(us - (long long)t * G), g1 = g0 + (int)(ul - us);
        const int n0 = (t / a.n_mb) * kBN2;
        const int nv = a.N - n0 < kBN2 ? a.N - n0 : kBN2;
        // kPair: N = 256 always (each CTA's half of B is 128 tokens, zero past N)
        const uint32_t idesc = kPair ? gemm_idesc_m(2 * kBM, kBN2) : gemm_idesc((nv + 15) & ~15);
        const uint32_t buf = j & 1, acc_t = tmem + buf * kTmemCols2;
        if (j >= 2 && !bar_wait(tempty0 + 8 * buf, ((j >> 1) - 1) & 1, &abort_flag)) {
          ok = false;
          break;
        }
        for (int s = g0; s < g1 && ok; ++s) {
          for (int h = 0; h < 2; ++h, ++q) {
            const uint32_t slot = q % kSt, par = (q / kSt) & 1;
            if (!bar_wait(full0 + 8 * slot, par, &abort_flag)) {
              ok = false;
              break;
            }
            asm volatile("tcgen05.fence::after_thread_sync;");
            // descriptors of the slot's A and B tiles; each 16-column step
            // adds 32 bytes (2 in the descriptor's 16-byte address field)
            const uint32_t sa = su32(base + slot * kSB);
            const uint64_t da0 = kmajor_desc(sa), db0 = kmajor_desc(sa + kATile2);
            const uint32_t acc0 = (s > g0 || h > 0) ? 1u : 0u;
#pragma unroll
            for (int k = 0; k < kBK2 / 16; ++k) {
              const uint64_t da = da0 + 2u * k, db = db0 + 2u * k;
              const uint32_t acc = k > 0 ? 1u : acc0;
              if constexpr (kPair)
                asm volatile(
                    "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(
                        acc_t),
                    "l"(da), "l"(db), "r"(idesc), "r"(acc));
              else
                asm volatile(
                    "{ .reg .pred p; setp.ne.b32 p, %4, 0; tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(
                        acc_t),
                    "l"(da), "l"(db), "r"(idesc), "r"(acc));
            }
            mma_commit<kPair>(free0 + 8 * slot);
          }
        }
        if (ok) mma_commit<kPair>(accf0 + 8 * buf);
      }
      if (!ok) {
        abort_flag = 1;
        atomicExch(a.status, (unsigned)PF_ERR_TIMEOUT);
      }
    }
  } else if (warp <= kDqWarps) {
    // ------------------------------------------------ dequant rows
    const int grp = (warp - 1) >> 2;       // this group decodes half grp of every scale group
    const int r = 32 * (warp & 3) + lane;  // tile row
    bool live = true;
    auto fail = [&]() {
      live = false;
      if (lane == 0) {
        abort_flag = 1;
        atomicExch(a.status, (unsigned)PF_ERR_TIMEOUT);
      }
    };
    uint32_t gs = 0, kc = 0, ks = 0;  // groups, code boxes and scale boxes consumed
    for (int it = 0; it < n_items; ++it) {
      long long us, ul;
      sk_item(u_begin, u_end, G, it, &us, &ul);
      const int t = (int)(us / G), g0 = (int)(us - (long long)t * G), g1 = g0 + (int)(ul - us);
      uint32_t cs = 0, ss = 0, cpar = 0, spar = 0;
      for (int s = g0; s < g1; ++s, ++gs) {
        // a code / scale box stays put until this thread's last group in it:
        // wait for it once, on entering it
        if (s == g0 || s % B::CB == 0) {
          cs = kc % kCS;
          cpar = (kc / kCS) & 1;
          ++kc;
          if (live && !bar_wait(cfull0 + 8 * cs, cpar, &abort_flag)) fail();
        }
        if (!kPolar && (s == g0 || s % B::SB == 0)) {
          ss = ks % kCS;
          spar = (ks / kCS) & 1;
          ++ks;
          if (live && !bar_wait(sfull0 + 8 * ss, spar, &abort_flag)) fail();
        }
        const uint32_t q = 2 * gs + grp, slot = q % kSt;
        // this row's scale (and zero point) of group s
        uint32_t sc = 0u;
        if (live && !kPolar) {
          const unsigned char* sp = scl + ss * kScaleSlot + r * 16 + (s % B::SB) * B::SW;
          if constexpr (kE8) {
            sc = *reinterpret_cast<const uint32_t*>(sp);
          } else {
            const uint32_t lo = *reinterpret_cast<const uint16_t*>(sp);
            const uint32_t hi = *reinterpret_cast<const uint16_t*>(sp + kCS * kScaleSlot);
            sc = lo | (hi << 16);
          }
        }
        const unsigned char* crow = codes + cs * kCodeSlot + r * (B::CB * B::GB);
        if (live && q >= kSt && !bar_wait(free0 + 8 * slot, ((q / kSt) - 1) & 1, &abort_flag)) fail();
        if (live) {
          unsigned char* at = base + slot * kSB;
          if (grp == 0)
            sk_decode<FMT, 0, kRC>(crow, (s % B::CB) * B::GB, sc, r, lane, at, roots16, ptab);
          else
            sk_decode<FMT, 1, kRC>(crow, (s % B::CB) * B::GB, sc, r, lane, at, roots16, ptab);
        }
        // hand the code / scale boxes back after this thread's last group in them
        if (s + 1 == g1 || (s + 1) % B::CB == 0)
          asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(cfree0 + 8 * cs) : "memory");
        if (!kPolar && (s + 1 == g1 || (s + 1) % B::SB == 0))
          asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sfree0 + 8 * ss) : "memory");
        // every lane's A-tile stores visible to the tensor core, then one arrival per warp
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) bar_arrive_pair<kPair>(full_l + 8 * slot);
      }
    }
  } else {
    // ------------------------------------------------ epilogue warps: TMEM -> y / partial tiles
    const int quarter = warp & 3;
    const int r = 32 * quarter + lane;  // tile row == this warp's TMEM lanes
    const uint32_t lane_off = (uint32_t)(32 * quarter) << 16;
    const int ci = sk_id;             // this CTA's (kPair: pair's) place in the stream-K split
    const int cta = (int)blockIdx.x;  // partial slots are per CTA
    asm volatile("griddepcontrol.wait;" ::: "memory");
    uint32_t j = 0;
    for (; (int)j < n_items; ++j) {
      long long us, ul;
      sk_item(u_begin, u_end, G, (int)j, &us, &ul);
      const int t = (int)(us / G), g0 = (int)(us - (long long)t * G), g1 = g0 + (int)(ul - us);
      const int m0 = (t % a.n_mb) * kRowsT + (int)rank * kBM, n0 = (t / a.n_mb) * kBN2;
      const uint32_t buf = j & 1, taddr = tmem + buf * kTmemCols2 + lane_off;
      const int nv = a.N - n0 < kBN2 ? a.N - n0 : kBN2;
      const int nmma = (nv + 15) & ~15;
      const int grow = m0 + r;
      const bool rvalid = grow < a.M;
      const float bv = (rvalid && a.bias) ? a.bias[grow] : 0.f;
      const bool whole = g0 == 0 && g1 == G;
      // the segment holding the range's first unit keeps slot 2c, the one ending it 2c + 1
      float* const mine = a.partials + ((size_t)(2 * cta + (us == u_begin ? 0 : 1)) * kBN2) * kBM;
      // this segment's token scales in shared memory: the y stores below then
      // need no global load between them
      asm volatile("bar.sync 1, %0;" ::"r"(kBM) : "memory");
      for (int i = r; i < kBN2; i += kBM)
        etscale[i] = n0 + i < a.N ? a.tok_scale[n0 + i] * (kPolar ? a.r_scale : 1.f) : 0.f;
      asm volatile("bar.sync 1, %0;" ::"r"(kBM) : "memory");
      bool ok = bar_wait(accf0 + 8 * buf, (j >> 1) & 1, &abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok && lane == 0) {
        abort_flag = 1;
        atomicExch(a.status, (unsigned)PF_ERR_TIMEOUT);
      }
      asm volatile("tcgen05.fence::after_thread_sync;");
      // 32 columns per TMEM load (columns past nmma are read, never written out)
#pragma unroll 1
      for (int c0 = 0; c0 < nmma && ok; c0 += 32) {
        float v[32];
        tmem_ld32(taddr + (uint32_t)c0, v);
        if (whole) {
          if (rvalid) {
#pragma unroll
            for (int jj = 0; jj < 32; ++jj) {
              const int tk = n0 + c0 + jj;
              if (tk < a.N) a.y[(size_t)tk * a.M + grow] = v[jj] * etscale[c0 + jj] + bv;
            }
          }
        } else {
#pragma unroll
          for (int jj = 0; jj < 32; ++jj)
            if (c0 + jj < nmma) mine[(size_t)(c0 + jj) * kBM + r] = v[jj];
        }
      }
      if (!whole) {
        // the last CTA of this tile to arrive sums the partials in k order
        // (its own from TMEM, the others' from the workspace)
        __threadfence();
        asm volatile("bar.sync 1, %0;" ::"r"(kBM) : "memory");
        if (warp == kEpiWarp0 && lane == 0) {
          unsigned v = 0xFFFFFFFFu;
          if (ok && !abort_flag) {
            v = atomicAdd(a.counters + (kPair ? 2 * t + (int)rank : t), 1u);
            __threadfence();
          }
          arrival = v;
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kBM) : "memory");
        const long long tu0 = (long long)t * G;
        const int cf = sk_cta_of(U, P, tu0), cl = sk_cta_of(U, P, tu0 + G - 1);
        const unsigned got = arrival;
        if (ok && got != 0xFFFFFFFFu && got == (unsigned)(cl - cf)) {
#pragma unroll 1
          for (int c0 = 0; c0 < nmma; c0 += 16) {
            float accv[16];
#pragma unroll
            for (int jj = 0; jj < 16; ++jj) accv[jj] = 0.f;
            // contributors in k order, two at a time so their loads overlap
#pragma unroll 1
            for (int cb = cf; cb <= cl; cb += 2) {
              float pv[2][16];
#pragma unroll
              for (int i = 0; i < 2; ++i) {
                const int c = cb + i;
                if (c > cl) continue;
                if (c == ci) {
                  uint32_t w[16];
                  tmem_ld16(taddr + (uint32_t)c0, w);
#pragma unroll
                  for (int jj = 0; jj < 16; ++jj) pv[i][jj] = __uint_as_float(w[jj]);
                } else {
                  // CTA c holds this tile in its first segment (slot 2c) unless the tile starts after its range does
                  const int first_t = (int)(sk_begin(U, P, c) / G);
                  const int cc = kPair ? 2 * c + (int)rank : c;  // the contributing CTA holding these rows
                  const float* pp = a.partials + ((size_t)(2 * cc + (first_t == t ? 0 : 1)) * kBN2 + c0) * kBM + r;
#pragma unroll
                  for (int jj = 0; jj < 16; ++jj) pv[i][jj] = __ldcg(pp + (size_t)jj * kBM);
                }
              }
#pragma unroll
              for (int i = 0; i < 2; ++i) {
                if (cb + i > cl) continue;
#pragma unroll
                for (int jj = 0; jj < 16; ++jj) accv[jj] += pv[i][jj];
              }
            }
            if (rvalid) {
#pragma unroll
              for (int jj = 0; jj < 16; ++jj) {
                const int tk = n0 + c0 + jj;
                if (tk < a.N) a.y[(size_t)tk * a.M + grow] = accv[jj] * etscale[c0 + jj] + bv;
              }
            }
          }
          if (warp == kEpiWarp0 && lane == 0) a.counters[kPair ? 2 * t + (int)rank : t] = 0u;  // left zero for the next call
        }
        asm volatile("bar.sync 1, %0;" ::"r"(kBM) : "memory");  // arrival is rewritten by the next segment
      }
      // TMEM buffer free for the segment after next
      asm volatile("tcgen05.fence::before_thread_sync;");
      __syncwarp();
      if (lane == 0) bar_arrive_pair<kPair>(tempty_l + 8 * buf);
    }
  }
  asm volatile("tcgen05.fence::before_thread_sync;");
  __syncthreads();
  if constexpr (kPair) cluster_sync();  // the partner no longer reads this CTA's shared memory or signals it
  if (warp == kMmaWarp) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    if constexpr (kPair)
      asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kTmemCols2));
    else
      asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(2 * kTmemCols2));
  }
}


// Block-wide max of a non-negative float (all threads get it).
__device__ __forceinline__ float block_max(float mx, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = mx;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  return red[0];
}

// fp16 x'' of one token in the GEMM's slot order: x'' = x' 2^(15 - e) with
// max |x'| < 2^e, tok_scale = 2^(e - 15).
__device__ __forceinline__ void write_x16(const float* row, float mx, float rs, int K, int fmt, __half* out,
                                          float* tok_scale) {
  int ex = 0;
  if (mx > 0.f) frexpf(mx, &ex);  // mx < 2^ex
  const float sc = ldexpf(1.f, 15 - ex) * rs, inv = ldexpf(1.f, ex - 15);
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    const int g = k & ~127, sl = k & 127;
    out[k] = __float2half_rn(row[g + gemm_slot_col(fmt, sl)] * sc);
  }
  if (threadIdx.x == 0) *tok_scale = mx > 0.f ? inv : 1.f;
}

// From fp32 x' (prep_kernel, any rotation plan): one CTA per token.
__global__ void __launch_bounds__(256) xhalf_kernel(const float* __restrict__ xp, int Kp, int K, int fmt, __half* out,
                                                    float* tok_scale) {
  __shared__ float red[32];
  const int t = blockIdx.x;
  asm volatile("griddepcontrol.launch_dependents;");  // the GEMM's prologue may start
  const float* row = xp + (size_t)t * Kp;
  float mx = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) mx = fmaxf(mx, fabsf(row[k]));
  mx = block_max(mx, red);
  write_x16(row, mx, 1.f, K, fmt, out + (size_t)t * K, tok_scale + t);
}

// From x directly, for rotation blocks that tile K (no remainder cascade): one
// CTA per token, the token's row in shared memory, sign flip, Walsh-Hadamard
// butterflies of every block (one pass per level), 1/sqrt(b), max, fp16 out.
__global__ void __launch_bounds__(512) xprep16_kernel(const void* x, int x_dtype, const int8_t* signs, int K,
                                                      int block, float rs, int fmt, __half* out, float* tok_scale) {
  extern __shared__ float xrow[];
  __shared__ float red[32];
  const int t = blockIdx.x;
  asm volatile("griddepcontrol.launch_dependents;");  // the GEMM's prologue may start
  for (int k = threadIdx.x; k < K; k += blockDim.x) {
    float v = load_x(x, x_dtype, (size_t)t * K + k);
    if (block > 1 && signs[k] < 0) v = -v;
    xrow[k] = v;
  }
  __syncthreads();
  for (int h = 1; h < block; h <<= 1) {
    for (int j = threadIdx.x; j < K / 2; j += blockDim.x) {
      const int lo = (j / h) * 2 * h + (j % h);
      const float u = xrow[lo], w = xrow[lo + h];
      xrow[lo] = u + w;
      xrow[lo + h] = u - w;
    }
    __syncthreads();
  }
  float mx = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) mx = fmaxf(mx, fabsf(xrow[k]));
  mx = block_max(mx * rs, red);
  write_x16(xrow, mx, rs, K, fmt, out + (size_t)t * K, tok_scale + t);
}

// V consecutive activations of one token as fp32 (16-byte aligned x).
template <int V>
__device__ __forceinline__ void load_vec(const void* x, int dtype, size_t idx, float* v) {
  if (dtype == PF_DTYPE_F32) {
    const float4* p = reinterpret_cast<const float4*>(static_cast<const float*>(x) + idx);
#pragma unroll
    for (int q = 0; q < V / 4; ++q) {
      const float4 f = p[q];
      v[4 * q] = f.x; v[4 * q + 1] = f.y; v[4 * q + 2] = f.z; v[4 * q + 3] = f.w;
    }
  } else {
    const uint2* p = reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(x) + idx);
#pragma unroll
    for (int q = 0; q < V / 4; ++q) {
      const uint2 w = p[q];
      const uint32_t h[2] = {w.x, w.y};
#pragma unroll
      for (int e = 0; e < 2; ++e) {
        if (dtype == PF_DTYPE_F16) {
          const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&h[e]));
          v[4 * q + 2 * e] = f.x; v[4 * q + 2 * e + 1] = f.y;
        } else {
          v[4 * q + 2 * e] = __uint_as_float(h[e] << 16);
          v[4 * q + 2 * e + 1] = __uint_as_float(h[e] & 0xFFFF0000u);
        }
      }
    }
  }
}

// The same x' as xprep16_kernel with the butterflies in registers: each lane
// holds V consecutive columns of a 32 V-column segment (one segment per warp
// at a time, V >= block / 32), levels below V in-lane, the others by warp
// shuffles (same sums and differences in the same order, so the same bits);
// the rotated row goes to shared memory once for the max and the fp16 pass,
// which writes 8 slot-ordered fp16 per 16-byte store.
template <int V>
__global__ void __launch_bounds__(512) xprep16_vec_kernel(const void* x, int x_dtype, const int8_t* signs, int K,
                                                          int block, float rs, int fmt, __half* out,
                                                          float* tok_scale) {
  extern __shared__ float xrow[];
  __shared__ float red[32];
  constexpr int kSeg = 32 * V;
  const int t = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  asm volatile("griddepcontrol.launch_dependents;");  // the GEMM's prologue may start
  float mx = 0.f;
  for (int seg = warp; seg < K / kSeg; seg += nw) {
    const int k0 = seg * kSeg + lane * V;
    float v[V];
    load_vec<V>(x, x_dtype, (size_t)t * K + k0, v);
    if (block > 1) {
#pragma unroll
      for (int q = 0; q < V / 4; ++q) {
        const uint32_t sg = *reinterpret_cast<const uint32_t*>(signs + k0 + 4 * q);
#pragma unroll
        for (int e = 0; e < 4; ++e)
          if (sg & (0x80u << (8 * e))) v[4 * q + e] = -v[4 * q + e];
      }
    }
#pragma unroll
    for (int h = 1; h < V; h <<= 1) {
      if (h < block) {
#pragma unroll
        for (int i = 0; i < V; ++i) {
          if (!(i & h)) {
            const float u = v[i], w = v[i + h];
            v[i] = u + w;
            v[i + h] = u - w;
          }
        }
      }
    }
    for (int h = V; h < block; h <<= 1) {
      const int m = h / V;
      const bool upper = (lane & m) != 0;
#pragma unroll
      for (int i = 0; i < V; ++i) {
        const float p = __shfl_xor_sync(0xffffffffu, v[i], m);
        v[i] = upper ? p - v[i] : v[i] + p;
      }
    }
#pragma unroll
    for (int i = 0; i < V; ++i) mx = fmaxf(mx, fabsf(v[i]));
#pragma unroll
    for (int q = 0; q < V / 4; ++q)
      *reinterpret_cast<float4*>(xrow + k0 + 4 * q) = make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
  }
  mx = block_max(mx * rs, red);  // also orders the row's shared-memory writes before the reads below
  int ex = 0;
  if (mx > 0.f) frexpf(mx, &ex);  // mx < 2^ex
  const float sc = ldexpf(1.f, 15 - ex) * rs, inv = ldexpf(1.f, ex - 15);
  __half* o = out + (size_t)t * K;
  for (int k = 8 * threadIdx.x; k < K; k += 8 * blockDim.x) {
    const int g = k & ~127, sl = k & 127;
    uint32_t w[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const __half2 h2 = __floats2half2_rn(xrow[g + gemm_slot_col(fmt, sl + 2 * e)] * sc,
                                           xrow[g + gemm_slot_col(fmt, sl + 2 * e + 1)] * sc);
      w[e] = *reinterpret_cast<const uint32_t*>(&h2);
    }
    *reinterpret_cast<uint4*>(o + k) = make_uint4(w[0], w[1], w[2], w[3]);
  }
  if (threadIdx.x == 0) tok_scale[t] = mx > 0.f ? inv : 1.f;
}

PFN_cuTensorMapEncodeTiled_v12000 encode_fn_gemm() {
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

// PF_GEMM_TMA=0 keeps every launch on the plain kernel (for comparison).
bool gemm_tma_enabled() {
  static int v = -1;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* e = getenv("PF_GEMM_TMA");
    v = (e && atoi(e) == 0) ? 0 : 1;
  });
  return v == 1;
}

// Streaming multiprocessors of the current device (cached per device).
int sm_count() {
  static int cache[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess) return 0;
  if (dev >= 0 && dev < 64 && cache[dev]) return cache[dev];
  int n = 0;
  if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) return 0;
  if (dev >= 0 && dev < 64) cache[dev] = n;
  return n;
}

// Batches above 128 tokens run on two-SM pairs; PF_GEMM_PAIR=0 keeps them on
// the one-SM stream-K kernel.
bool gemm_pair_enabled() {
  static int v = -1;
  static std::once_flag once;
  std::call_once(once, [] {
    const char* e = getenv("PF_GEMM_PAIR");
    v = (e && atoi(e) == 0) ? 0 : 1;
  });
  return v == 1;
}

// The persistent stream-K kernel: 2-D tensor maps over the packed rows and
// the scale rows need 16-byte aligned bases and row strides, and the tile
// count must fit the workspace's arrival counters.  kPair: two-CTA clusters,
// as many as can be resident at once.
template <int FMT, bool kPair, int kXR = kBN2>
cudaError_t launch_gemm_sk_impl(GemmArgs a, const __half* x16, cudaStream_t s, bool* taken) {
  using B = TcBox<FMT>;
  constexpr bool kE8 = FMT == PF_FMT_E8_RVQ2_G128;
  constexpr bool kPolar = FMT == PF_FMT_POLAR_RECURSIVE;
  constexpr int kSt = kPair ? kStagesPair : (kXR == kBN2 ? kStages2 : kStagesSmall);
  constexpr int kXRows = kPair ? kBN2 / 2 : kXR;
  constexpr size_t kSB = kATile2 + (size_t)kXRows * kBK2 * 2;
  constexpr int kRowsT = kPair ? 2 * kBM : kBM;
  *taken = false;
  const size_t row_bytes = (size_t)a.G * B::GB, srow = (size_t)a.G * B::SW;
  if (!gemm_tma_enabled() || row_bytes % 16 || reinterpret_cast<uintptr_t>(a.codes) % 16 || !a.counters ||
      !a.partials)
    return cudaSuccess;
  if (!kPolar && (srow % 16 || reinterpret_cast<uintptr_t>(a.scales) % 16 ||
                  (!kE8 && reinterpret_cast<uintptr_t>(a.mins) % 16)))
    return cudaSuccess;
  const int n_mb = (a.M + kRowsT - 1) / kRowsT, n_nb = (a.N + kBN2 - 1) / kBN2;
  const long long tiles = (long long)n_mb * n_nb;
  const int sms = sm_count();
  if (sms <= 0 || (kPair ? 2 : 1) * tiles > (long long)kGemmCounterSlots) return cudaSuccess;
  a.n_mb = n_mb;
  a.units = tiles * a.G;
  auto fn = encode_fn_gemm();
  CUtensorMap xmap, cmap, smap, mmap;
  {
    // x' tiles of 64 columns x up to 256 tokens, 128B-swizzled
    cuuint64_t dims[2] = {(cuuint64_t)a.K, (cuuint64_t)a.N};
    cuuint64_t strides[1] = {(cuuint64_t)a.K * 2};
    cuuint32_t box[2] = {64, (cuuint32_t)(kPair ? kXRows : sk_box_rows(a.N))};
    cuuint32_t estr[2] = {1, 1};
    if (fn(&xmap, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(x16), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaSuccess;
  }
  {
    cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 4), (cuuint64_t)a.M};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)(B::CB * B::GB / 4), (cuuint32_t)kBM};
    cuuint32_t estr[2] = {1, 1};
    if (fn(&cmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(a.codes), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, code_swizzled<B>() ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
           CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaSuccess;
  }
  for (int k = 0; k < (kPolar ? 0 : kE8 ? 1 : 2); ++k) {
    // scale (and zero-point) rows: SB groups of SW bytes per box row (16 bytes)
    cuuint64_t dims[2] = {(cuuint64_t)(srow / 2), (cuuint64_t)a.M};
    cuuint64_t strides[1] = {(cuuint64_t)srow};
    cuuint32_t box[2] = {8, (cuuint32_t)kBM};
    cuuint32_t estr[2] = {1, 1};
    const void* src = k == 0 ? static_cast<const void*>(a.scales) : static_cast<const void*>(a.mins);
    if (fn(k == 0 ? &smap : &mmap, CU_TENSOR_MAP_DATA_TYPE_UINT16, 2, const_cast<void*>(src), dims, strides, box,
           estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaSuccess;
  }
  if (kPolar) smap = cmap;  // never read: polar has no scale boxes
  if (kE8 || kPolar) mmap = smap;
  constexpr int kCS = kPair ? 2 : sk_box_slots(kXR);
  const size_t smem = 1024 + (size_t)kSt * kSB + (size_t)kCS * kBM * B::CB * B::GB +
                      (size_t)kCS * (kPolar ? 0 : kE8 ? 1 : 2) * kBM * 16;
  auto kern = gemm_sk_kernel<FMT, kPair, kXR>;
  // programmatic dependent launch: barrier setup, TMEM allocation, the code and
  // scale loads and the first decodes overlap the x' preparation's tail
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  attr[1].id = cudaLaunchAttributeClusterDimension;
  attr[1].val.clusterDim.x = 2;
  attr[1].val.clusterDim.y = 1;
  attr[1].val.clusterDim.z = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(kSkThreads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = kPair ? 2 : 1;
  static int max_pairs[64] = {0};
  int dev = 0;
  {
    static std::mutex mu;
    static bool done[64] = {false};
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64 || !done[dev]) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      if (kPair) {
        // pairs that fit on the device at once (clusters sit inside one GPC)
        cfg.gridDim = dim3(2 * (sms / 2));
        int n = 0;
        e = cudaOccupancyMaxActiveClusters(&n, kern, &cfg);
        if (e != cudaSuccess) return e;
        if (dev >= 0 && dev < 64) max_pairs[dev] = n;
      }
      if (dev >= 0 && dev < 64) done[dev] = true;
    }
  }
  int P = sms;
  if (kPair) {
    P = (dev >= 0 && dev < 64) ? max_pairs[dev] : 0;
    if (P > sms / 2) P = sms / 2;
    if (P < 1) return cudaSuccess;  // no two-CTA cluster fits: the one-SM kernel runs
  }
  if (a.units < P) P = (int)a.units;
  *taken = true;
  cfg.gridDim = dim3((kPair ? 2 : 1) * P);
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, xmap, cmap, smap, mmap, (const GemmArgs)a);
  note_launch();
  return e != cudaSuccess ? e : cudaGetLastError();
}

template <int FMT>
cudaError_t launch_gemm_sk(const GemmArgs& a, const __half* x16, cudaStream_t s, bool* taken) {
  if (a.N > kBN2 / 2 && gemm_pair_enabled()) {
    const cudaError_t e = launch_gemm_sk_impl<FMT, true>(a, x16, s, taken);
    if (*taken || e != cudaSuccess) return e;
  }
  if (a.N <= kSmallN) return launch_gemm_sk_impl<FMT, false, kSmallN>(a, x16, s, taken);
  return launch_gemm_sk_impl<FMT, false>(a, x16, s, taken);
}

// Recursive polar runs on the persistent kernel only (the plain kernel has
// no polar decoder); the caller checks gemm_eligible and passes a workspace
// with the partial tiles.
cudaError_t launch_gemm_polar(const GemmArgs& a, const __half* x16, cudaStream_t s) {
  bool taken = false;
  const cudaError_t e = launch_gemm_sk<PF_FMT_POLAR_RECURSIVE>(a, x16, s, &taken);
  if (e != cudaSuccess) return e;
  return taken ? cudaSuccess : cudaErrorNotSupported;
}

template <int FMT>
cudaError_t launch_gemm_fmt(const GemmArgs& a, const __half* x16, cudaStream_t s) {
  auto fn = encode_fn_gemm();
  if (!fn) return cudaErrorNotSupported;
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)a.K, (cuuint64_t)a.N};
  cuuint64_t strides[1] = {(cuuint64_t)a.K * 2};
  cuuint32_t box[2] = {64, (cuuint32_t)kBN};
  cuuint32_t estr[2] = {1, 1};
  if (fn(&map, CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 2, const_cast<__half*>(x16), dims, strides, box, estr,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
         CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return cudaErrorInvalidValue;
  {
    bool taken = false;
    const cudaError_t e = launch_gemm_sk<FMT>(a, x16, s, &taken);
    if (taken || e != cudaSuccess) return e;
  }
  const size_t smem = 1024 + (size_t)kStages * kStageBytes;
  auto kern = gemm_tc_kernel<FMT>;
  {
    static std::mutex mu;
    static bool done[64] = {false};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) return e;
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64 || !done[dev]) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
      if (e != cudaSuccess) return e;
      if (dev >= 0 && dev < 64) done[dev] = true;
    }
  }
  dim3 grid((a.M + kBM - 1) / kBM, (a.N + kBN - 1) / kBN);
  kern<<<grid, kGemmThreads, smem, s>>>(map, a);
  note_launch();
  return cudaGetLastError();
}

}  // namespace

bool gemm_eligible(int fmt, int K) {
  if (fmt == PF_FMT_POLAR_RECURSIVE)  // block 8 at 1.75 bpw (the caller checks the allocation): 16-byte code rows
    return K % 512 == 0 && gemm_tma_enabled() && encode_fn_gemm() != nullptr;
  if (!(fmt == PF_FMT_INT4_G128 || fmt == PF_FMT_INT3_G128 || fmt == PF_FMT_INT2_G128 ||
        fmt == PF_FMT_E8_RVQ2_G128))
    return false;
  return K % kBK == 0 && encode_fn_gemm() != nullptr;
}

size_t gemm_x16_bytes(int N, int K) { return ((size_t)N * K * 2 + 255) / 256 * 256 + ((size_t)N * 4 + 255) / 256 * 256; }

size_t gemm_partial_bytes() { return (size_t)2 * sm_count() * kBN2 * kBM * sizeof(float); }

cudaError_t launch_gemm(const GemmIn& in, cudaStream_t s) {
  if (in.xplain) {
    xhalf_kernel<<<in.N, 256, 0, s>>>(in.xplain, in.Kp, in.K, in.fmt, in.x16, in.tok_scale);
  } else {
    const size_t smem = (size_t)in.K * sizeof(float);
    static std::mutex mu;
    static bool done[64] = {false};
    int dev = 0;
    cudaError_t e0 = cudaGetDevice(&dev);
    if (e0 != cudaSuccess) return e0;
    {
      std::lock_guard<std::mutex> lock(mu);
      if (dev < 0 || dev >= 64 || !done[dev]) {
        for (const void* f : {reinterpret_cast<const void*>(xprep16_kernel),
                              reinterpret_cast<const void*>(xprep16_vec_kernel<4>),
                              reinterpret_cast<const void*>(xprep16_vec_kernel<8>),
                              reinterpret_cast<const void*>(xprep16_vec_kernel<16>)}) {
          e0 = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmPrepMaxK * 4);
          if (e0 != cudaSuccess) return e0;
        }
        if (dev >= 0 && dev < 64) done[dev] = true;
      }
    }
    // register butterflies for rotation blocks up to 512 columns (16-byte aligned x, 4-byte aligned signs)
    const int blk = in.block > 1 ? in.block : 1;
    const bool vec = blk <= 512 && reinterpret_cast<uintptr_t>(in.x) % 16 == 0 &&
                     (blk == 1 || reinterpret_cast<uintptr_t>(in.signs) % 4 == 0);
    if (vec && blk <= 128)
      xprep16_vec_kernel<4><<<in.N, 512, smem, s>>>(in.x, in.x_dtype, in.signs, in.K, blk, in.rscale, in.fmt, in.x16,
                                                   in.tok_scale);
    else if (vec && blk == 256)
      xprep16_vec_kernel<8><<<in.N, 512, smem, s>>>(in.x, in.x_dtype, in.signs, in.K, blk, in.rscale, in.fmt, in.x16,
                                                   in.tok_scale);
    else if (vec && blk == 512)
      xprep16_vec_kernel<16><<<in.N, 512, smem, s>>>(in.x, in.x_dtype, in.signs, in.K, blk, in.rscale, in.fmt,
                                                    in.x16, in.tok_scale);
    else
      xprep16_kernel<<<in.N, 512, smem, s>>>(in.x, in.x_dtype, in.signs, in.K, in.block, in.rscale, in.fmt, in.x16,
                                             in.tok_scale);
  }
  note_launch();
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  GemmArgs a;
  memset(&a, 0, sizeof(a));
  a.fmt = in.fmt;
  a.codes = in.codes;
  a.scales = in.scales;
  a.mins = in.mins;
  a.M = in.M;
  a.K = in.K;
  a.N = in.N;
  a.G = in.K / kBK;
  a.row_words = in.row_words;
  a.tok_scale = in.tok_scale;
  a.bias = in.bias;
  a.y = in.y;
  a.status = in.status;
  a.counters = in.counters;
  a.partials = in.partials;
  a.r_scale = in.r_scale;
  a.angles = in.angles;
  switch (in.fmt) {
    case PF_FMT_INT4_G128: return launch_gemm_fmt<PF_FMT_INT4_G128>(a, in.x16, s);
    case PF_FMT_INT3_G128: return launch_gemm_fmt<PF_FMT_INT3_G128>(a, in.x16, s);
    case PF_FMT_INT2_G128: return launch_gemm_fmt<PF_FMT_INT2_G128>(a, in.x16, s);
    case PF_FMT_E8_RVQ2_G128: return launch_gemm_fmt<PF_FMT_E8_RVQ2_G128>(a, in.x16, s);
    case PF_FMT_POLAR_RECURSIVE: return launch_gemm_polar(a, in.x16, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace pfb
