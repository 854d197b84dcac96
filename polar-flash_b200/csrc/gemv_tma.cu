// TMA-pipelined fused dequant-GEMV for the INT formats (N <= 16 tokens).
//
// CTA = 4 consumer warps + 1 producer warp.  The producer streams 64-row x
// S-group tiles of packed codes with 2-D TMA copies (plus the matching x'
// records with 1-D bulk copies) into a 4-stage shared-memory ring guarded by
// mbarriers; the weights of the first stages are requested before the
// kernel waits for the x-prep grid (programmatic dependent launch), so weight
// streaming overlaps the preceding kernel.  Consumers read their rows' words
// from shared memory (128B-swizzled tiles, row order permuted so the reads
// are bank-conflict free), decode each code pair with one AND (plus OR of the
// exponent for normal-magic codes) -- codes that already sit below mantissa
// bit 10 are not shifted; the per-position power of two lives in x' instead
// -- and multiply on the tensor cores (mma.sync m16n8k16, register A).
//
// Codes become fp16 values  h = q 2^(p-24)  (subnormal, exact) and x' was
// scaled by 2^(14-p-E), so  sum h B = 2^-10 sum q x'/2^E  with no bias term;
// with the normal magic h = 1 + q 2^(p-10), B = x' 2^(10-p-E) and
// sum h B = SB + sum q x'/2^E.  Per 128-column group:
//     sum w x' = s 2^E Q + m Sx,   Q = sum q x'/2^E.
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

constexpr int kRows = 64;
constexpr int kCWarps = 4;
constexpr int kThreadsT = (kCWarps + 1) * 32;
constexpr int kStagesT = 4;
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

// Box row of quad-row rq: under the 128B swizzle a warp's smem reads are
// split into 8-lane (LDS.128) or 16-lane (LDS.64) phases; these orders put
// rows whose swizzle masks differ in the right bits into one phase.
template <int FMT>
__device__ __forceinline__ int row_perm(int rq) {
  if constexpr (FMT == PF_FMT_INT4_G128 || FMT == PF_FMT_INT4)
    return ((rq & 1) << 2) | (rq >> 1);
  else if constexpr (FMT == PF_FMT_INT2_G128 || FMT == PF_FMT_INT2)
    return ((rq & 3) << 1) | (rq >> 2);
  else
    return rq;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
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
    if ((it & 63) == 0) {
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

// ---- in-place decoders: words of one row and group -> 16 half2 (see frag_cols2)
template <int FMT, uint32_t MAGIC>
struct Dec2;

template <uint32_t MAGIC>
struct Dec2<PF_FMT_INT4_G128, MAGIC> {
  static __device__ __forceinline__ void run(const uint32_t (&w)[4], int, uint32_t (&h)[16]) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      const uint32_t v = w[t] >> 8;
      h[4 * t + 0] = (w[t] & 0x000F000Fu) | MAGIC;
      h[4 * t + 1] = (w[t] & 0x00F000F0u) | MAGIC;
      h[4 * t + 2] = (v & 0x000F000Fu) | MAGIC;
      h[4 * t + 3] = (v & 0x00F000F0u) | MAGIC;
    }
  }
};
template <uint32_t MAGIC>
struct Dec2<PF_FMT_INT4, MAGIC> : Dec2<PF_FMT_INT4_G128, MAGIC> {};

template <uint32_t MAGIC>
struct Dec2<PF_FMT_INT2_G128, MAGIC> {
  static __device__ __forceinline__ void run(const uint32_t (&w)[4], int, uint32_t (&h)[16]) {
#pragma unroll
    for (int t = 0; t < 2; ++t) {
#pragma unroll
      for (int k = 0; k < 5; ++k) h[8 * t + k] = (w[t] & (0x00030003u << (2 * k))) | MAGIC;
      const uint32_t v = w[t] >> 10;
#pragma unroll
      for (int k = 0; k < 3; ++k) h[8 * t + 5 + k] = (v & (0x00030003u << (2 * k))) | MAGIC;
    }
  }
};
template <uint32_t MAGIC>
struct Dec2<PF_FMT_INT2, MAGIC> : Dec2<PF_FMT_INT2_G128, MAGIC> {};

template <uint32_t MAGIC>
struct Dec2<PF_FMT_INT3_G128, MAGIC> {
  static __device__ __forceinline__ void run(const uint32_t (&w)[4], int c, uint32_t (&h)[16]) {
#pragma unroll
    for (int t = 0; t < 3; ++t) {
      const uint32_t g = (w[t] & 0x0000FFFFu) | ((w[t] << 1) & 0xFFFF0000u);
      h[5 * t + 0] = (g & 0x00070007u) | MAGIC;
      h[5 * t + 1] = (g & 0x00380038u) | MAGIC;
      h[5 * t + 2] = (g & 0x01C001C0u) | MAGIC;
      const uint32_t v = g >> 9;
      h[5 * t + 3] = (v & 0x00070007u) | MAGIC;
      h[5 * t + 4] = (v & 0x00380038u) | MAGIC;
    }
    const uint32_t t12 = w[3] >> (6 * c);
    h[15] = ((t12 & 7u) | MAGIC) | ((t12 << 13) & 0x00070000u);
  }
};

// Words of box row r, stage group j, for quad thread c.
template <int FMT>
__device__ __forceinline__ void lds_words(const unsigned char* stage, int r, int j, int c, uint32_t (&w)[4]) {
  if constexpr (FMT == PF_FMT_INT4_G128 || FMT == PF_FMT_INT4) {
    const int chunk = (4 * j + c) ^ (r & 7);
    const uint4 v = *reinterpret_cast<const uint4*>(stage + r * 128 + (chunk << 4));
    w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
  } else if constexpr (FMT == PF_FMT_INT2_G128 || FMT == PF_FMT_INT2) {
    const int chunk = (2 * j + (c >> 1)) ^ (r & 7);
    const uint2 v = *reinterpret_cast<const uint2*>(stage + r * 128 + (chunk << 4) + ((c & 1) << 3));
    w[0] = v.x; w[1] = v.y;
    w[2] = w[3] = 0u;
  } else {
    const uint32_t* row = reinterpret_cast<const uint32_t*>(stage) + r * (TmaFmt<FMT>::S * 13) + 13 * j;
    w[0] = row[c];
    w[1] = row[c + 4];
    w[2] = row[c + 8];
    w[3] = row[12];
  }
}

__device__ __forceinline__ long long cta_of(long long u, long long U, long long P) {
  return ((u + 1) * P + U - 1) / U - 1;
}

template <int FMT, int NT, bool SUBN, int SMODE>
__global__ void __launch_bounds__(kThreadsT, NT == 1 ? 3 : 2)
    gemv_tma_kernel(const __grid_constant__ CUtensorMap tmap, const TmaArgs a) {
  using F = TmaFmt<FMT>;
  constexpr int S = F::S;
  constexpr uint32_t kMagic = SUBN ? 0u : 0x3C003C00u;
  constexpr uint32_t kWBytes = kRows * S * F::WPG * 4;
  constexpr int kOffset = IntFmt<FMT>::kOffset;

  asm volatile("griddepcontrol.launch_dependents;");

  extern __shared__ unsigned char smem_raw[];
  unsigned char* smem =
      reinterpret_cast<unsigned char*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t xbytes = (uint32_t)(S * a.rec_bytes);
  unsigned char* wbuf = smem;                                  // kStagesT x kWBytes
  unsigned char* xbuf = smem + kStagesT * kWBytes;              // kStagesT x xbytes
  uint64_t* bars = reinterpret_cast<uint64_t*>(xbuf + kStagesT * ((xbytes + 127) & ~127u));
  const uint32_t full0 = smem_u32(bars), empty0 = smem_u32(bars + kStagesT);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStagesT; ++s) {
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(full0 + 8 * s), "r"(1));
      asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(empty0 + 8 * s), "r"(kCWarps));
    }
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  const long long U = a.n_units, P = gridDim.x, cta = blockIdx.x;
  const int u0 = (int)(cta * U / P), u1 = (int)((cta + 1) * U / P);
  const int nunits = u1 - u0;

  if (warp == kCWarps) {
    // ------------------------------------------------------------ producer
    if (lane == 0 && nunits > 0) {
      const int first = nunits < kStagesT ? nunits : kStagesT;
      for (int k = 0; k < first; ++k) {
        const int u = u0 + k, rb = u / a.spb, st = u % a.spb;
        mbar_expect(full0 + 8 * k, kWBytes + xbytes);
        tma_2d(smem_u32(wbuf + k * kWBytes), &tmap, st * S * F::WPG, rb * kRows, full0 + 8 * k);
      }
      // x' comes from the x-prep grid: wait for it before reading the records
      asm volatile("griddepcontrol.wait;" ::: "memory");
      for (int k = 0; k < first; ++k) {
        const int st = (u0 + k) % a.spb;
        bulk_1d(smem_u32(xbuf + k * ((xbytes + 127) & ~127u)), a.rec + (size_t)st * S * a.rec_bytes, xbytes,
                full0 + 8 * k);
      }
      for (int it = first; it < nunits; ++it) {
        const int slot = it % kStagesT;
        const uint32_t parity = ((it / kStagesT) & 1) ^ 1;
        if (!mbar_wait(empty0 + 8 * slot, parity)) {
          atomicExch(a.counters + kWsStatusSlot, (unsigned)PF_ERR_TIMEOUT);
          return;
        }
        const int u = u0 + it, rb = u / a.spb, st = u % a.spb;
        mbar_expect(full0 + 8 * slot, kWBytes + xbytes);
        tma_2d(smem_u32(wbuf + slot * kWBytes), &tmap, st * S * F::WPG, rb * kRows, full0 + 8 * slot);
        bulk_1d(smem_u32(xbuf + slot * ((xbytes + 127) & ~127u)), a.rec + (size_t)st * S * a.rec_bytes, xbytes,
                full0 + 8 * slot);
      }
    }
    return;
  }

  // -------------------------------------------------------------- consumers
  const int c = lane & 3, rq = lane >> 2;
  const int r0 = warp * 16 + row_perm<FMT>(rq), r1 = r0 + 8;  // box rows
  const int Lp = tma_lanes(a.N, NT);
  const int spb = a.spb;

  // Raw fp16 scale/zero words of the thread's two rows for one unit (S
  // groups), prefetched one unit ahead so HBM latency stays off the epilogue.
  constexpr int SW = S / 2;
  struct Raw {
    uint32_t s0[SW], m0[SW], s1[SW], m1[SW];
  };
  auto load_raw = [&](int u, Raw& d) {
    const int rb = u / spb, st = u % spb;
    const int ga = rb * kRows + r0, gb = rb * kRows + r1;
#pragma unroll
    for (int q = 0; q < SW; ++q) {
      d.s0[q] = d.m0[q] = d.s1[q] = d.m1[q] = 0u;
    }
    if constexpr (SMODE == kScaleGroup) {
      const uint32_t* sc = static_cast<const uint32_t*>(a.scales);
      const uint32_t* mn = reinterpret_cast<const uint32_t*>(a.mins);
      const size_t oa = ((size_t)ga * a.G + (size_t)st * S) / 2, ob = ((size_t)gb * a.G + (size_t)st * S) / 2;
#pragma unroll
      for (int q = 0; q < SW; ++q) {
        if (ga < a.M) {
          d.s0[q] = __ldg(sc + oa + q);
          d.m0[q] = __ldg(mn + oa + q);
        }
        if (gb < a.M) {
          d.s1[q] = __ldg(sc + ob + q);
          d.m1[q] = __ldg(mn + ob + q);
        }
      }
    }
  };

  float y0[NT], y1[NT];
  int seg_st0 = 0;
  Raw cur, nxt;
  if (nunits > 0) load_raw(u0, cur);
  for (int it = 0; it < nunits; ++it) {
    const int u = u0 + it, rb = u / spb, st = u % spb;
    const int slot = it % kStagesT;
    if (it + 1 < nunits) load_raw(u + 1, nxt);
    if (it == 0 || st == 0) {
      seg_st0 = st;
#pragma unroll
      for (int i = 0; i < NT; ++i) y0[i] = y1[i] = 0.f;
    }
    const int grow0 = rb * kRows + r0, grow1 = rb * kRows + r1;
    const bool v0 = grow0 < a.M, v1 = grow1 < a.M;
    float s0[S], m0[S], s1[S], m1[S];
    if constexpr (SMODE == kScaleGroup) {
#pragma unroll
      for (int q = 0; q < SW; ++q) {
        const float2 fs0 = __half22float2(*reinterpret_cast<const __half2*>(&cur.s0[q]));
        const float2 fm0 = __half22float2(*reinterpret_cast<const __half2*>(&cur.m0[q]));
        const float2 fs1 = __half22float2(*reinterpret_cast<const __half2*>(&cur.s1[q]));
        const float2 fm1 = __half22float2(*reinterpret_cast<const __half2*>(&cur.m1[q]));
        s0[2 * q] = fs0.x; s0[2 * q + 1] = fs0.y;
        m0[2 * q] = fm0.x; m0[2 * q + 1] = fm0.y;
        s1[2 * q] = fs1.x; s1[2 * q + 1] = fs1.y;
        m1[2 * q] = fm1.x; m1[2 * q + 1] = fm1.y;
      }
    } else {
      float sa = a.tensor_scale, sb = a.tensor_scale;
      if constexpr (SMODE == kScaleRow) {
        sa = v0 ? static_cast<const float*>(a.scales)[grow0] : 0.f;
        sb = v1 ? static_cast<const float*>(a.scales)[grow1] : 0.f;
      }
#pragma unroll
      for (int j = 0; j < S; ++j) {
        s0[j] = sa;
        m0[j] = -(float)kOffset * sa;
        s1[j] = sb;
        m1[j] = -(float)kOffset * sb;
      }
    }
    cur = nxt;
    if (!mbar_wait(full0 + 8 * slot, (it / kStagesT) & 1)) {
      atomicExch(a.counters + kWsStatusSlot, (unsigned)PF_ERR_TIMEOUT);
      return;
    }
    const unsigned char* ws = wbuf + slot * kWBytes;
    const unsigned char* xs = xbuf + slot * ((xbytes + 127) & ~127u);
#pragma unroll
    for (int j = 0; j < S; ++j) {
      uint32_t w0[4], w1[4];
      lds_words<FMT>(ws, r0, j, c, w0);
      lds_words<FMT>(ws, r1, j, c, w1);
      uint32_t h0[16], h1[16];
      Dec2<FMT, kMagic>::run(w0, c, h0);
      Dec2<FMT, kMagic>::run(w1, c, h1);
      const unsigned char* rec = xs + (size_t)j * a.rec_bytes;
      const float4* gs = reinterpret_cast<const float4*>(rec + (size_t)NT * 8 * Lp * 8);
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        float acc[4] = {0.f, 0.f, 0.f, 0.f};
        const uint2* fr = reinterpret_cast<const uint2*>(rec) + (size_t)i * 8 * Lp + lane;
#pragma unroll
        for (int j8 = 0; j8 < 8; ++j8) {
          const uint2 b = lane < Lp ? fr[j8 * Lp] : make_uint2(0u, 0u);
          mma16816(acc, h0[2 * j8], h1[2 * j8], h0[2 * j8 + 1], h1[2 * j8 + 1], b.x, b.y);
        }
        const int t = 4 * i + c;
        if (t < a.N) {
          const float4 g4 = gs[t];
          const float q0 = SUBN ? 1024.f * (acc[0] + acc[1]) : (acc[0] + acc[1]) - g4.z;
          const float q1 = SUBN ? 1024.f * (acc[2] + acc[3]) : (acc[2] + acc[3]) - g4.z;
          y0[i] += (s0[j] * g4.y) * q0 + m0[j] * g4.x;
          y1[i] += (s1[j] * g4.y) * q1 + m1[j] * g4.x;
        }
      }
    }
    __syncwarp();
    if (lane == 0) mbar_arrive(empty0 + 8 * slot);

    // -------------------------------------------------- end of a row-block segment
    if (st == spb - 1 || it == nunits - 1) {
      const bool whole = (seg_st0 == 0 && st == spb - 1);
      if (whole) {
#pragma unroll
        for (int i = 0; i < NT; ++i) {
          const int t = 4 * i + c;
          if (t >= a.N) continue;
          if (v0) a.y[(size_t)t * a.M + grow0] = y0[i] + (a.bias ? a.bias[grow0] : 0.f);
          if (v1) a.y[(size_t)t * a.M + grow1] = y1[i] + (a.bias ? a.bias[grow1] : 0.f);
        }
        continue;
      }
      const int my_slot = (rb == u0 / spb) ? (int)(2 * cta) : (int)(2 * cta + 1);
      float* part = a.partials + (size_t)my_slot * kRows * a.N;
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        const int t = 4 * i + c;
        if (t >= a.N) continue;
        part[(size_t)r0 * a.N + t] = y0[i];
        part[(size_t)r1 * a.N + t] = y1[i];
      }
      __threadfence();
      __syncwarp();
      const long long first = cta_of((long long)rb * spb, U, P), last = cta_of((long long)(rb + 1) * spb - 1, U, P);
      const unsigned n_share = (unsigned)(last - first + 1);
      unsigned* ctr = a.counters + (size_t)rb * kCWarps + warp;
      unsigned prev = 0;
      if (lane == 0) prev = atomicAdd(ctr, 1u);
      prev = __shfl_sync(0xffffffffu, prev, 0);
      if (prev != n_share - 1) continue;
      __threadfence();
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        const int t = 4 * i + c;
        if (t >= a.N) continue;
        float acc0 = 0.f, acc1 = 0.f;
        for (long long k = first; k <= last; ++k) {
          const long long ku0 = k * U / P;
          const int ks = (rb == (int)(ku0 / spb)) ? (int)(2 * k) : (int)(2 * k + 1);
          const float* pk = a.partials + (size_t)ks * kRows * a.N;
          acc0 += __ldcg(pk + (size_t)r0 * a.N + t);
          acc1 += __ldcg(pk + (size_t)r1 * a.N + t);
        }
        if (v0) a.y[(size_t)t * a.M + grow0] = acc0 + (a.bias ? a.bias[grow0] : 0.f);
        if (v1) a.y[(size_t)t * a.M + grow1] = acc1 + (a.bias ? a.bias[grow1] : 0.f);
      }
      if (lane == 0) *ctr = 0u;
    }
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

template <int FMT>
size_t smem_bytes(int rec_bytes) {
  using F = TmaFmt<FMT>;
  const size_t wb = (size_t)kRows * F::S * F::WPG * 4;
  const size_t xb = ((size_t)F::S * rec_bytes + 127) & ~size_t(127);
  return 1024 + kStagesT * (wb + xb) + 2 * kStagesT * 8;
}

template <int FMT, int NT, bool SUBN, int SMODE>
cudaError_t launch_one(const TmaArgs& a, cudaStream_t s) {
  using F = TmaFmt<FMT>;
  auto fn = encode_fn();
  if (!fn) return cudaErrorNotSupported;
  CUtensorMap map;
  cuuint64_t dims[2] = {(cuuint64_t)a.row_words, (cuuint64_t)a.M};
  cuuint64_t strides[1] = {(cuuint64_t)a.row_words * 4};
  cuuint32_t box[2] = {(cuuint32_t)(F::S * F::WPG), (cuuint32_t)kRows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(a.codes), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE,
                  F::SW128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return cudaErrorInvalidValue;
  const size_t smem = smem_bytes<FMT>(a.rec_bytes);
  auto kern = gemv_tma_kernel<FMT, NT, SUBN, SMODE>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  static int occ = 0;
  static size_t occ_smem = 0;
  if (occ == 0 || occ_smem != smem) {
    int n = 0;
    if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&n, kern, kThreadsT, smem) != cudaSuccess || n < 1) n = 1;
    occ = n < kMaxCtasPerSm ? n : kMaxCtasPerSm;
    occ_smem = smem;
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

template <int FMT, int NT, bool SUBN>
cudaError_t launch_sm(const TmaArgs& a, int smode, cudaStream_t s) {
  if (smode == kScaleGroup) return launch_one<FMT, NT, SUBN, kScaleGroup>(a, s);
  if (smode == kScaleRow) return launch_one<FMT, NT, SUBN, kScaleRow>(a, s);
  return launch_one<FMT, NT, SUBN, kScaleTensor>(a, s);
}

template <int FMT, int NT>
cudaError_t launch_sub(const TmaArgs& a, int smode, int subnormal, cudaStream_t s) {
  return subnormal ? launch_sm<FMT, NT, true>(a, smode, s) : launch_sm<FMT, NT, false>(a, smode, s);
}

template <int FMT>
cudaError_t launch_fmt(const TmaArgs& a, int smode, int subnormal, cudaStream_t s) {
  switch (a.NT) {
    case 1: return launch_sub<FMT, 1>(a, smode, subnormal, s);
    case 2: return launch_sub<FMT, 2>(a, smode, subnormal, s);
    default: return launch_sub<FMT, 4>(a, smode, subnormal, s);
  }
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
  const long long n_rb = (M + kRows - 1) / kRows;
  if (n_rb * kCWarps >= (long long)kWsStatusSlot) return false;
  return encode_fn() != nullptr;
}

// CTAs of one launch: never more than the units, at most kMaxCtasPerSm per SM
// (shared memory bounds the real residency; the partial-slot area is sized
// for this count).
int tma_grid(int fmt, int NT, int n_units) {
  (void)fmt;
  (void)NT;
  long long g = (long long)sm_count() * kMaxCtasPerSm;
  if (g > n_units) g = n_units;
  return (int)(g < 1 ? 1 : g);
}

cudaError_t launch_gemv_tma(int fmt, const TmaArgs& a, int smode, int subnormal, cudaStream_t s) {
  switch (fmt) {
    case PF_FMT_INT4_G128: return launch_fmt<PF_FMT_INT4_G128>(a, smode, subnormal, s);
    case PF_FMT_INT3_G128: return launch_fmt<PF_FMT_INT3_G128>(a, smode, subnormal, s);
    case PF_FMT_INT2_G128: return launch_fmt<PF_FMT_INT2_G128>(a, smode, subnormal, s);
    case PF_FMT_INT4: return launch_fmt<PF_FMT_INT4>(a, smode, subnormal, s);
    case PF_FMT_INT2: return launch_fmt<PF_FMT_INT2>(a, smode, subnormal, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace pfb
