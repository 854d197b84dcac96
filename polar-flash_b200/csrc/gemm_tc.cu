// Dequant-GEMM on the 5th-generation tensor cores (tcgen05 + TMEM) for
// batches of more than 16 tokens: Y[N][M] = X'[N][K] * W_hat^T, W_hat decoded
// from the packed payload inside the kernel (INT4 / INT3 / INT2 group-128
// asymmetric and E8 RVQ2), X' = the forward block RWHT of X in fp16 with a
// power-of-two scale per token (the same fusion identity as the GEMV).
//
// CTA = 128 weight rows x 128 tokens, one CTA per SM, six warps:
//   warp 0    TMA producer: the x' tile of each 128-column stage, two
//             64-column boxes, 128B-swizzled (K-major canonical layout).
//   warps 1-4 one weight row per thread: load the row's packed group with
//             plain 16-byte loads (one stage ahead), decode every weight to
//             fp16 q*s + m (one rounding: an fp16 FMA of the exact code) or,
//             for E8, s1*r[i1] + s2*r[i2] (fp32, one rounding), and write it
//             into the A tile in the same swizzled K-major layout; then the
//             epilogue (tcgen05.ld of their 32 TMEM lanes, token scale, bias).
//   warp 5    allocates 128 TMEM columns and issues tcgen05.mma (kind::f16,
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
constexpr int kGemmThreads = 192;
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

// fp16 pair (q0, q1) from two small codes: 1024 + q as fp16 bits, minus 1024.
__device__ __forceinline__ __half2 code_pair(uint32_t q0, uint32_t q1) {
  const uint32_t b = q0 | (q1 << 16) | 0x64006400u;
  return __hsub2(*reinterpret_cast<const __half2*>(&b), __half2half2(__ushort_as_half(0x6400)));
}

template <int FMT>
__global__ void __launch_bounds__(kGemmThreads, 1) gemm_tc_kernel(const __grid_constant__ CUtensorMap xmap,
                                                                   const __grid_constant__ GemmArgs a) {
  extern __shared__ __align__(1024) unsigned char smem_raw[];
  __shared__ uint64_t bars[3 * kStages + 1];
  __shared__ uint32_t tmem_base_slot;
  __shared__ int abort_flag;
  __shared__ __align__(16) float roots[240][8];  // read as float4
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
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(afull0 + 8 * s), "r"(128));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(free0 + 8 * s));
    }
    asm volatile("mbarrier.init.shared::cta.b64 [%0], 1;" ::"r"(accbar));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&xmap)) : "memory");
  }
  if (FMT == PF_FMT_E8_RVQ2_G128) {
    for (int k = threadIdx.x; k < 240; k += blockDim.x) {
      float r[8];
      e8_root(k, r);
#pragma unroll
      for (int q = 0; q < 8; ++q) roots[k][q] = r[q];
    }
  }
  for (int t = threadIdx.x; t < kBN; t += blockDim.x) tscale[t] = (n0 + t < a.N) ? a.tok_scale[n0 + t] : 0.f;
  if (warp == 5) {
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
  } else if (warp == 5) {
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
    const int r = 32 * (warp & 3) + lane;  // tile row == this warp's TMEM lanes
    const int grow = m0 + r;
    const bool rvalid = grow < a.M;
    const int growc = rvalid ? grow : 0;
    bool live = true;
    uint4 pk[4];  // the row's packed group (E8: 32 index bytes)
    uint32_t p13 = 0;
    uint32_t psc = 0;  // its fp16 scale and zero point (E8: the two stage scales)
    constexpr int kL2Ahead = 4;  // groups requested into L2 ahead of the register loads
    auto row_bytes = [&]() -> size_t {
      return FMT == PF_FMT_E8_RVQ2_G128 ? (size_t)a.K / 4 : (size_t)a.row_words * 4;
    };
    constexpr int kGroupBytes = FMT == PF_FMT_INT4_G128 ? 64 : (FMT == PF_FMT_INT3_G128 ? 52 : 32);
    auto l2_ahead = [&](int g) {
      if (g >= G) return;
      const char* p = static_cast<const char*>(a.codes) + (size_t)growc * row_bytes() + (size_t)g * kGroupBytes;
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
      if constexpr (FMT == PF_FMT_INT4_G128) {
        const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint32_t*>(a.codes) +
                                                        (size_t)growc * a.row_words + (size_t)g * 16);
#pragma unroll
        for (int q = 0; q < 4; ++q) pk[q] = __ldg(p + q);
      } else if constexpr (FMT == PF_FMT_INT2_G128) {
        const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint32_t*>(a.codes) +
                                                        (size_t)growc * a.row_words + (size_t)g * 8);
        pk[0] = __ldg(p);
        pk[1] = __ldg(p + 1);
      } else if constexpr (FMT == PF_FMT_INT3_G128) {
        const uint32_t* p = static_cast<const uint32_t*>(a.codes) + (size_t)growc * a.row_words + (size_t)g * 13;
        uint32_t w[13];
#pragma unroll
        for (int q = 0; q < 13; ++q) w[q] = __ldg(p + q);
        pk[0] = make_uint4(w[0], w[1], w[2], w[3]);
        pk[1] = make_uint4(w[4], w[5], w[6], w[7]);
        pk[2] = make_uint4(w[8], w[9], w[10], w[11]);
        p13 = w[12];
      } else {  // E8: [M][K/8][2] bytes, 32 per group
        const uint4* p = reinterpret_cast<const uint4*>(static_cast<const uint8_t*>(a.codes) +
                                                        (size_t)growc * (a.K / 4) + (size_t)g * 32);
        pk[0] = __ldg(p);
        pk[1] = __ldg(p + 1);
      }
    };
    auto word = [&](int i) -> uint32_t {  // i-th 32-bit word of pk
      const uint4 v = pk[i >> 2];
      const int q = i & 3;
      return q == 0 ? v.x : (q == 1 ? v.y : (q == 2 ? v.z : v.w));
    };
    for (int g = 0; g < kL2Ahead; ++g) l2_ahead(g);
    if (G > 0) load_group(0);
    for (int s = 0; s < G; ++s) {
      const int slot = s % kStages;
      unsigned char* at = base + slot * kStageBytes;
      // the codes and scales of this stage; the next stage's are requested
      // into registers before decoding, the one after that into L2
      uint32_t cw[16];
      uint32_t c12 = p13;
      const uint32_t sc = psc;
#pragma unroll
      for (int i = 0; i < 16; ++i) cw[i] = word(i);
      float sv = 0.f, s2v = 0.f;
      if constexpr (FMT == PF_FMT_E8_RVQ2_G128) {
        const __half2 ss = *reinterpret_cast<const __half2*>(&sc);
        sv = __low2float(ss);
        s2v = __high2float(ss);
      }
      l2_ahead(s + kL2Ahead);
      if (s + 1 < G) load_group(s + 1);
      if (live && s >= kStages && !bar_wait(free0 + 8 * slot, ((s / kStages) - 1) & 1, &abort_flag)) {
        live = false;
        if (lane == 0) {
          abort_flag = 1;
          atomicExch(a.status, (unsigned)PF_ERR_TIMEOUT);
        }
      }
      if (live) {
        if constexpr (FMT == PF_FMT_E8_RVQ2_G128) {
          // 16 vectors of 8 columns: chunk c = vector c
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            const uint32_t wv = cw[c >> 1];
            const int i1 = (wv >> (16 * (c & 1))) & 0xFF, i2 = (wv >> (16 * (c & 1) + 8)) & 0xFF;
            const float4 r1a = *reinterpret_cast<const float4*>(&roots[i1 < 240 ? i1 : 0][0]);
            const float4 r1b = *reinterpret_cast<const float4*>(&roots[i1 < 240 ? i1 : 0][4]);
            const float4 r2a = *reinterpret_cast<const float4*>(&roots[i2 < 240 ? i2 : 0][0]);
            const float4 r2b = *reinterpret_cast<const float4*>(&roots[i2 < 240 ? i2 : 0][4]);
            const __half2 h0 = __floats2half2_rn(fmaf(sv, r1a.x, s2v * r2a.x), fmaf(sv, r1a.y, s2v * r2a.y));
            const __half2 h1 = __floats2half2_rn(fmaf(sv, r1a.z, s2v * r2a.z), fmaf(sv, r1a.w, s2v * r2a.w));
            const __half2 h2 = __floats2half2_rn(fmaf(sv, r1b.x, s2v * r2b.x), fmaf(sv, r1b.y, s2v * r2b.y));
            const __half2 h3 = __floats2half2_rn(fmaf(sv, r1b.z, s2v * r2b.z), fmaf(sv, r1b.w, s2v * r2b.w));
            uint4 o;
            o.x = *reinterpret_cast<const uint32_t*>(&h0);
            o.y = *reinterpret_cast<const uint32_t*>(&h1);
            o.z = *reinterpret_cast<const uint32_t*>(&h2);
            o.w = *reinterpret_cast<const uint32_t*>(&h3);
            *reinterpret_cast<uint4*>(at + a_chunk(r, c)) = rvalid ? o : make_uint4(0, 0, 0, 0);
          }
        } else {
          // the stored fp16 scale / zero point
          const __half2 sx = __half2half2(__ushort_as_half((unsigned short)(sc & 0xFFFFu)));
          const __half2 mx = __half2half2(__ushort_as_half((unsigned short)(sc >> 16)));
#pragma unroll
          for (int c = 0; c < 16; ++c) {
            uint32_t q[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const int k = 8 * c + e;  // column in the group
              if constexpr (FMT == PF_FMT_INT4_G128) {
                q[e] = (cw[k >> 3] >> (4 * (k & 7))) & 15u;
              } else if constexpr (FMT == PF_FMT_INT2_G128) {
                q[e] = (cw[k >> 4] >> (2 * (k & 15))) & 3u;
              } else {
                const int wi = k / 10, sh = 3 * (k % 10);
                q[e] = ((wi < 12 ? cw[wi] : c12) >> sh) & 7u;
              }
            }
            uint4 o;
            uint32_t* ov = reinterpret_cast<uint32_t*>(&o);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const __half2 h = __hfma2(code_pair(q[2 * e], q[2 * e + 1]), sx, mx);
              ov[e] = *reinterpret_cast<const uint32_t*>(&h);
            }
            *reinterpret_cast<uint4*>(at + a_chunk(r, c)) = rvalid ? o : make_uint4(0, 0, 0, 0);
          }
        }
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(afull0 + 8 * slot) : "memory");
      }
    }
    // ------------------------------------------------ epilogue
    if (live && bar_wait(accbar, 0, &abort_flag)) {
      asm volatile("tcgen05.fence::after_thread_sync;");
      const uint32_t taddr = tmem + ((uint32_t)(32 * (warp & 3)) << 16);
      const float bv = (rvalid && a.bias) ? a.bias[grow] : 0.f;
#pragma unroll 1
      for (int c0 = 0; c0 < nmma; c0 += 16) {
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
  if (warp == 5) {
    asm volatile("tcgen05.fence::after_thread_sync;");
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemCols));
  }
}

// x'' (fp16) = x' * 2^e per token with max |x'| 2^e in [2^14, 2^15); tok_scale = 2^-e.
__global__ void __launch_bounds__(256) xhalf_kernel(const float* __restrict__ xp, int Kp, int K, __half* out,
                                                    float* tok_scale) {
  const int t = blockIdx.x;
  const float* row = xp + (size_t)t * Kp;
  float mx = 0.f;
  for (int k = threadIdx.x; k < K; k += blockDim.x) mx = fmaxf(mx, fabsf(row[k]));
  __shared__ float red[8];
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
  mx = red[0];
  int ex = 0;
  if (mx > 0.f) frexpf(mx, &ex);  // mx < 2^ex
  const float sc = ldexpf(1.f, 15 - ex), inv = ldexpf(1.f, ex - 15);
  __half* o = out + (size_t)t * K;
  for (int k = threadIdx.x; k < K; k += blockDim.x) o[k] = __float2half_rn(row[k] * sc);
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
  xhalf_kernel<<<in.N, 256, 0, s>>>(in.xplain, in.Kp, in.K, in.x16, in.tok_scale);
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
