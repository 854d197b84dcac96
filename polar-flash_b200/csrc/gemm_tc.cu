// Dequant-GEMM on the 5th-generation tensor cores (tcgen05 + TMEM) for
// batches of more than 16 tokens: Y[N][M] = X'[N][K] * W_hat^T, W_hat decoded
// from the packed payload inside the kernel (INT4 / INT3 / INT2 group-128
// asymmetric and E8 RVQ2), X' = the forward block RWHT of X in fp16 with a
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
};

__device__ __forceinline__ uint32_t su32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ bool bar_wait(uint32_t bar, uint32_t parity, const volatile int* abort_flag) {
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
      if (*abort_flag) return false;
      const unsigned long long t = gtime();
      if (t0 == 0)
        t0 = t;
      else if (t - t0 > kGemmWaitNs)
        return false;
    }
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
constexpr int kStages2 = 2;  // the dequant groups take alternate stages: one slot each

__device__ __forceinline__ void tma2d_plain(uint32_t dst, const CUtensorMap* map, int x, int y, uint32_t bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::"r"(
          dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar)
      : "memory");
}

template <int FMT>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tc2_kernel(const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap cmap,
                    const __grid_constant__ CUtensorMap smap, const __grid_constant__ CUtensorMap mmap,
                    const __grid_constant__ GemmArgs a) {
  using B = TcBox<FMT>;
  constexpr bool kE8 = FMT == PF_FMT_E8_RVQ2_G128;
  constexpr uint32_t kCodeSlot = kBM * B::CB * B::GB;  // 128 rows x CB groups
  constexpr uint32_t kScaleSlot = kBM * 16;            // 128 rows x SB groups x SW bytes (16)
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  // A/B ring full / A full / free, accumulator, then code full / free and scale full / free (two slots each)
  __shared__ uint64_t bars[3 * kStages2 + 1 + 8];
  __shared__ uint32_t tmem_base_slot;
  __shared__ int abort_flag;
  __shared__ uint4 roots16[kE8 ? 256 * 4 : 1];
  __shared__ float tscale[kBN];

  unsigned char* const base = smem_raw + ((1024u - (su32(smem_raw) & 1023u)) & 1023u);
  unsigned char* const codes = base + kStages2 * kStageBytes;          // [2][kCodeSlot]
  unsigned char* const scl = codes + 2 * kCodeSlot;                    // [2][kScaleSlot] (+ [2][kScaleSlot] mins)
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int m0 = blockIdx.x * kBM, n0 = blockIdx.y * kBN;
  const uint32_t bfull0 = su32(&bars[0]), afull0 = su32(&bars[kStages2]), free0 = su32(&bars[2 * kStages2]);
  const uint32_t accbar = su32(&bars[3 * kStages2]);
  const uint32_t cfull0 = su32(&bars[3 * kStages2 + 1]), cfree0 = cfull0 + 16;
  const uint32_t sfull0 = cfull0 + 32, sfree0 = cfull0 + 48;

  if (threadIdx.x == 0) {
    abort_flag = 0;
    for (int s = 0; s < kStages2; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(bfull0 + 8 * s));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(afull0 + 8 * s), "r"(kBM));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(free0 + 8 * s));
    }
    for (int s = 0; s < 2; ++s) {  // the code and scale boxes are double-buffered
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(cfull0 + 8 * s));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(cfree0 + 8 * s), "r"(2 * kBM));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(sfull0 + 8 * s));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(sfree0 + 8 * s), "r"(2 * kBM));
    }
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(accbar));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&cmap)) : "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&smap)) : "memory");
    if (!kE8) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&mmap)) : "memory");
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
  const int nv = a.N - n0 < kBN ? a.N - n0 : kBN;
  const int nmma = (nv + 15) & ~15;

  if (warp == 0) {
    // ------------------------------------------------ producer: codes, scales, x'
    if (lane == 0) {
      bool ok = true;
      for (int s = 0; s < G && ok; ++s) {
        if (s % B::CB == 0) {
          const int b = s / B::CB, cs = b & 1;
          if (b >= 2 && !bar_wait(cfree0 + 8 * cs, ((b >> 1) - 1) & 1, &abort_flag)) {
            ok = false;
            break;
          }
          asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(cfull0 + 8 * cs),
                       "r"(kCodeSlot)
                       : "memory");
          tma2d_plain(su32(codes + cs * kCodeSlot), &cmap, s * (B::GB / 4), m0, cfull0 + 8 * cs);
        }
        if (s % B::SB == 0) {
          const int c = s / B::SB, ss = c & 1;
          if (c >= 2 && !bar_wait(sfree0 + 8 * ss, ((c >> 1) - 1) & 1, &abort_flag)) {
            ok = false;
            break;
          }
          asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(sfull0 + 8 * ss),
                       "r"(kE8 ? kScaleSlot : 2 * kScaleSlot)
                       : "memory");
          // x in fp16 elements: E8 keeps two scales per group
          tma2d_plain(su32(scl + ss * kScaleSlot), &smap, kE8 ? 2 * s : s, m0, sfull0 + 8 * ss);
          if (!kE8) tma2d_plain(su32(scl + (2 + ss) * kScaleSlot), &mmap, s, m0, sfull0 + 8 * ss);
        }
        const int slot = s % kStages2;
        if (s >= kStages2 && !bar_wait(free0 + 8 * slot, ((s / kStages2) - 1) & 1, &abort_flag)) {
          ok = false;
          break;
        }
        const uint32_t dst = su32(base + slot * kStageBytes + kATile), bar = bfull0 + 8 * slot;
        asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(kBTile) : "memory");
#pragma unroll
        for (int h = 0; h < 2; ++h) tma2d_plain(dst + h * (kBN * 128), &xmap, s * kBK + h * 64, n0, bar);
      }
      if (!ok) {
        abort_flag = 1;
        atomicExch(a.status, (unsigned)PF_ERR_TIMEOUT);
      }
    }
  } else if (warp == kMmaWarp) {
    // ------------------------------------------------------------ MMA issue
    if (lane == 0) {
      for (int s = 0; s < G; ++s) {
        const int slot = s % kStages2;
        const uint32_t par = (s / kStages2) & 1;
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
    bool live = true;
    auto fail = [&]() {
      live = false;
      if (lane == 0) {
        abort_flag = 1;
        atomicExch(a.status, (unsigned)PF_ERR_TIMEOUT);
      }
    };
    for (int s = grp; s < G; s += 2) {
      const int slot = s % kStages2;
      const int b = s / B::CB, cs = b & 1, sbx = s / B::SB, ss = sbx & 1;
      if (live && !bar_wait(cfull0 + 8 * cs, (b >> 1) & 1, &abort_flag)) fail();
      if (live && !bar_wait(sfull0 + 8 * ss, (sbx >> 1) & 1, &abort_flag)) fail();
      // this row's codes and scales of stage s
      uint32_t cw[16];
      uint32_t sc = 0u;
      if (live) {
        const unsigned char* cp = codes + cs * kCodeSlot + r * (B::CB * B::GB) + (s % B::CB) * B::GB;
        if constexpr (FMT == PF_FMT_INT3_G128) {
#pragma unroll
          for (int q = 0; q < 13; ++q) cw[q] = *reinterpret_cast<const uint32_t*>(cp + 4 * q);
          cw[13] = cw[14] = cw[15] = 0u;
        } else {
#pragma unroll
          for (int q = 0; q < B::GB / 16; ++q) {
            const uint4 v = *reinterpret_cast<const uint4*>(cp + 16 * q);
            cw[4 * q] = v.x; cw[4 * q + 1] = v.y; cw[4 * q + 2] = v.z; cw[4 * q + 3] = v.w;
          }
#pragma unroll
          for (int q = B::GB / 4; q < 16; ++q) cw[q] = 0u;
        }
        const unsigned char* sp = scl + ss * kScaleSlot + r * 16 + (s % B::SB) * B::SW;
        if constexpr (kE8) {
          sc = *reinterpret_cast<const uint32_t*>(sp);
        } else {
          const uint32_t lo = *reinterpret_cast<const uint16_t*>(sp);
          const uint32_t hi = *reinterpret_cast<const uint16_t*>(sp + 2 * kScaleSlot);
          sc = lo | (hi << 16);
        }
      }
      // hand the code / scale boxes back after this thread's last stage in them
      if (s + 2 >= (b + 1) * B::CB || s + 2 >= G) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(cfree0 + 8 * cs) : "memory");
      if (s + 2 >= (sbx + 1) * B::SB || s + 2 >= G) asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(sfree0 + 8 * ss) : "memory");
      if (live && s >= kStages2 && !bar_wait(free0 + 8 * slot, ((s / kStages2) - 1) & 1, &abort_flag)) fail();
      if (!live) continue;
      unsigned char* at = base + slot * kStageBytes;
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
          *reinterpret_cast<uint4*>(at + a_chunk(r, c)) = o;  // rows past M: zero codes (TMA fill)
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
          *reinterpret_cast<uint4*>(at + a_chunk(r, c)) = o;  // rows past M: zero codes (TMA fill)
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

// The TMA-staged variant: 2-D tensor maps over the packed rows and the scale
// rows need 16-byte aligned bases and row strides.
template <int FMT>
cudaError_t launch_gemm_tc2(const GemmArgs& a, const CUtensorMap& xmap, cudaStream_t s, bool* taken) {
  using B = TcBox<FMT>;
  constexpr bool kE8 = FMT == PF_FMT_E8_RVQ2_G128;
  *taken = false;
  const size_t row_bytes = (size_t)a.G * B::GB, srow = (size_t)a.G * B::SW;
  if (!gemm_tma_enabled() || row_bytes % 16 || srow % 16 || reinterpret_cast<uintptr_t>(a.codes) % 16 ||
      reinterpret_cast<uintptr_t>(a.scales) % 16 || (!kE8 && reinterpret_cast<uintptr_t>(a.mins) % 16))
    return cudaSuccess;
  auto fn = encode_fn_gemm();
  CUtensorMap cmap, smap, mmap;
  {
    cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 4), (cuuint64_t)a.M};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)(B::CB * B::GB / 4), (cuuint32_t)kBM};
    cuuint32_t estr[2] = {1, 1};
    if (fn(&cmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(a.codes), dims, strides, box, estr,
           CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
      return cudaSuccess;
  }
  for (int k = 0; k < (kE8 ? 1 : 2); ++k) {
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
  if (kE8) mmap = smap;
  const size_t smem = 1024 + (size_t)kStages2 * kStageBytes + 2 * (size_t)kBM * B::CB * B::GB +
                      (kE8 ? 2 : 4) * (size_t)kBM * 16;
  auto kern = gemm_tc2_kernel<FMT>;
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
  *taken = true;
  dim3 grid((a.M + kBM - 1) / kBM, (a.N + kBN - 1) / kBN);
  kern<<<grid, kGemmThreads, smem, s>>>(xmap, cmap, smap, mmap, a);
  note_launch();
  return cudaGetLastError();
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
    const cudaError_t e = launch_gemm_tc2<FMT>(a, map, s, &taken);
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
  if (!(fmt == PF_FMT_INT4_G128 || fmt == PF_FMT_INT3_G128 || fmt == PF_FMT_INT2_G128 ||
        fmt == PF_FMT_E8_RVQ2_G128))
    return false;
  return K % kBK == 0 && encode_fn_gemm() != nullptr;
}

size_t gemm_x16_bytes(int N, int K) { return ((size_t)N * K * 2 + 255) / 256 * 256 + ((size_t)N * 4 + 255) / 256 * 256; }

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
        e0 = cudaFuncSetAttribute(xprep16_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kGemmPrepMaxK * 4);
        if (e0 != cudaSuccess) return e0;
        if (dev >= 0 && dev < 64) done[dev] = true;
      }
    }
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
  switch (in.fmt) {
    case PF_FMT_INT4_G128: return launch_gemm_fmt<PF_FMT_INT4_G128>(a, in.x16, s);
    case PF_FMT_INT3_G128: return launch_gemm_fmt<PF_FMT_INT3_G128>(a, in.x16, s);
    case PF_FMT_INT2_G128: return launch_gemm_fmt<PF_FMT_INT2_G128>(a, in.x16, s);
    case PF_FMT_E8_RVQ2_G128: return launch_gemm_fmt<PF_FMT_E8_RVQ2_G128>(a, in.x16, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace pfb
