// Fused dequant-GEMV for the INT formats (N <= 16 tokens).
//
// Data flow per warp: a work item is 16*TR weight rows x a chunk of 128-column
// groups.  Each thread streams its words of two rows (r, r+8) straight from HBM
// with vector loads (the quad of threads of a row reads the row's group
// contiguously), decodes every code pair into one half2 in registers with a
// shift + LOP3, and feeds the pairs as the A operand of m16n8k16 tensor-core
// MMAs whose B operand is x' (the rotated activations, hi+lo fp16 split,
// prepared once by prep.cu).  The codes become the exact fp16 values
//     h = 1 + q * 2^-b        (q placed in the top mantissa bits),
// so the fp32 accumulator holds  A = sum h x' = Sx + 2^-b sum q x'  and, per
// group, with w = q s + m (compressed_kv.py:145 convention):
//     sum w x' = 2^b s A + (m - 2^b s) Sx .
// No decoded weight is ever written to memory: HBM traffic is the packed
// codes, the fp16 scales and the tiny x'.  Tensor cores are used here as the
// multiply-add engine because the CUDA-core alternative (convert + FFMA per
// weight) needs ~3 instructions per weight, more than the SM issue rate allows
// at 2-3 bit HBM rates; the register-operand MMA leaves ~1 decode instruction
// per weight.
#include "common.cuh"
#include "gemv.cuh"

namespace pfb {

namespace {

constexpr int kWarps = 4;

template <int S>
__device__ __forceinline__ uint32_t shl(uint32_t x) {
  if constexpr (S >= 0)
    return x << S;
  else
    return x >> (-S);
}

__device__ __forceinline__ uint32_t shl_rt(uint32_t x, int s) { return s >= 0 ? (x << s) : (x >> (-s)); }

template <int FMT>
struct Dec;

// INT4: words 4c..4c+3; half2 4t+p = codes (p, p+4) of word t at bits 6..9 / 22..25.
template <>
struct Dec<PF_FMT_INT4_G128> {
  static __device__ __forceinline__ void run(const uint32_t (&w)[4], int, uint32_t (&h)[16]) {
#pragma unroll
    for (int t = 0; t < 4; ++t) {
      h[4 * t + 0] = (shl<6>(w[t]) & 0x03C003C0u) | 0x3C003C00u;
      h[4 * t + 1] = (shl<2>(w[t]) & 0x03C003C0u) | 0x3C003C00u;
      h[4 * t + 2] = (shl<-2>(w[t]) & 0x03C003C0u) | 0x3C003C00u;
      h[4 * t + 3] = (shl<-6>(w[t]) & 0x03C003C0u) | 0x3C003C00u;
    }
  }
};
template <>
struct Dec<PF_FMT_INT4> : Dec<PF_FMT_INT4_G128> {};

// INT2: words 2c, 2c+1; half2 8t+p = codes (p, p+8) at bits 8..9 / 24..25.
template <>
struct Dec<PF_FMT_INT2_G128> {
  static __device__ __forceinline__ void run(const uint32_t (&w)[4], int, uint32_t (&h)[16]) {
#pragma unroll
    for (int t = 0; t < 2; ++t) {
      h[8 * t + 0] = (shl<8>(w[t]) & 0x03000300u) | 0x3C003C00u;
      h[8 * t + 1] = (shl<6>(w[t]) & 0x03000300u) | 0x3C003C00u;
      h[8 * t + 2] = (shl<4>(w[t]) & 0x03000300u) | 0x3C003C00u;
      h[8 * t + 3] = (shl<2>(w[t]) & 0x03000300u) | 0x3C003C00u;
      h[8 * t + 4] = (w[t] & 0x03000300u) | 0x3C003C00u;
      h[8 * t + 5] = (shl<-2>(w[t]) & 0x03000300u) | 0x3C003C00u;
      h[8 * t + 6] = (shl<-4>(w[t]) & 0x03000300u) | 0x3C003C00u;
      h[8 * t + 7] = (shl<-6>(w[t]) & 0x03000300u) | 0x3C003C00u;
    }
  }
};
template <>
struct Dec<PF_FMT_INT2> : Dec<PF_FMT_INT2_G128> {};

// A 10-code word (code i at bits 3i): merging its low half with the high half
// of (word << 1) puts codes (p, p+5) exactly 16 bits apart.
__device__ __forceinline__ void dec10(uint32_t w, uint32_t* h) {
  uint32_t g = (w & 0x0000FFFFu) | ((w << 1) & 0xFFFF0000u);
  h[0] = (shl<7>(g) & 0x03800380u) | 0x3C003C00u;
  h[1] = (shl<4>(g) & 0x03800380u) | 0x3C003C00u;
  h[2] = (shl<1>(g) & 0x03800380u) | 0x3C003C00u;
  h[3] = (shl<-2>(g) & 0x03800380u) | 0x3C003C00u;
  h[4] = (shl<-5>(g) & 0x03800380u) | 0x3C003C00u;
}

// INT3 group-128 (10 codes/word, 13 words): words c, c+4, c+8, and word 12
// whose codes (2c, 2c+1) sit at bits 6c and 6c+3.
template <>
struct Dec<PF_FMT_INT3_G128> {
  static __device__ __forceinline__ void run(const uint32_t (&w)[4], int c, uint32_t (&h)[16]) {
    dec10(w[0], h);
    dec10(w[1], h + 5);
    dec10(w[2], h + 10);
    h[15] = (shl_rt(w[3], 7 - 6 * c) & 0x00000380u) | (shl_rt(w[3], 20 - 6 * c) & 0x03800000u) | 0x3C003C00u;
  }
};

// INT3 reference stream: words 3c..3c+2 = 96 bits = codes 32c..32c+31; funnel
// shifts cut three 10-code windows, codes 30 and 31 sit at bits 26 and 29.
template <>
struct Dec<PF_FMT_INT3> {
  static __device__ __forceinline__ void run(const uint32_t (&w)[4], int, uint32_t (&h)[16]) {
    dec10(w[0], h);
    dec10(__funnelshift_r(w[0], w[1], 30), h + 5);
    dec10(__funnelshift_r(w[1], w[2], 28), h + 10);
    h[15] = ((w[2] >> 19) & 0x00000380u) | ((w[2] >> 6) & 0x03800000u) | 0x3C003C00u;
  }
};

// Loads this thread's words of one row for group g (zeros past the row end).
template <int FMT>
__device__ __forceinline__ void load_words(const uint32_t* __restrict__ row, int g, int row_words, int c,
                                           uint32_t (&w)[4]) {
  using F = IntFmt<FMT>;
  const int base = g * F::kWordsPerGroup;
  if constexpr (FMT == PF_FMT_INT4_G128 || FMT == PF_FMT_INT4) {
    int wi = base + 4 * c;
    if (row != nullptr && wi < row_words) {
      uint4 v = __ldg(reinterpret_cast<const uint4*>(row + wi));
      w[0] = v.x; w[1] = v.y; w[2] = v.z; w[3] = v.w;
    } else {
      w[0] = w[1] = w[2] = w[3] = 0u;
    }
  } else if constexpr (FMT == PF_FMT_INT2_G128 || FMT == PF_FMT_INT2) {
    int wi = base + 2 * c;
    if (row != nullptr && wi < row_words) {
      uint2 v = __ldg(reinterpret_cast<const uint2*>(row + wi));
      w[0] = v.x; w[1] = v.y;
    } else {
      w[0] = w[1] = 0u;
    }
    w[2] = w[3] = 0u;
  } else if constexpr (FMT == PF_FMT_INT3_G128) {
    if (row != nullptr) {
      w[0] = __ldg(row + base + c);
      w[1] = __ldg(row + base + c + 4);
      w[2] = __ldg(row + base + c + 8);
      w[3] = __ldg(row + base + 12);
    } else {
      w[0] = w[1] = w[2] = w[3] = 0u;
    }
  } else {  // PF_FMT_INT3 reference stream
    int wi = base + 3 * c;
    if (row != nullptr && wi < row_words) {
      w[0] = __ldg(row + wi);
      w[1] = __ldg(row + wi + 1);
      w[2] = __ldg(row + wi + 2);
    } else {
      w[0] = w[1] = w[2] = 0u;
    }
    w[3] = 0u;
  }
}

__device__ __forceinline__ void mma16816(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                         uint32_t b0, uint32_t b1) {
  asm volatile(
      "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
      "{%0,%1,%2,%3};\n"
      : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
      : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

template <int FMT, int NT, int TR, int SMODE>
__global__ void __launch_bounds__(kWarps * 32) gemv_int_kernel(GemvIntArgs a) {
  using F = IntFmt<FMT>;
  constexpr float kPow = (float)(1 << F::kBits);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int item = blockIdx.x * kWarps + warp;
  if (item >= a.n_items) return;
  const int chunk = item / a.n_row_items;
  const int ritem = item - chunk * a.n_row_items;
  const int g_begin = chunk * a.CG;
  const int g_end = min(g_begin + a.CG, a.G);
  const int c = lane & 3, rq = lane >> 2;
  const uint32_t* __restrict__ codes = static_cast<const uint32_t*>(a.codes);

  int rows[TR][2];
  const uint32_t* rp[TR][2];
#pragma unroll
  for (int tr = 0; tr < TR; ++tr)
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) {
      int row = ritem * 16 * TR + tr * 16 + rq + 8 * rr;
      rows[tr][rr] = row;
      rp[tr][rr] = row < a.M ? codes + (size_t)row * a.row_words : nullptr;
    }

  // per-row scale (row / tensor modes)
  float S_u[TR][2], M_u[TR][2];
  if constexpr (SMODE != kScaleGroup) {
#pragma unroll
    for (int tr = 0; tr < TR; ++tr)
#pragma unroll
      for (int rr = 0; rr < 2; ++rr) {
        float s = a.tensor_scale;
        if constexpr (SMODE == kScaleRow)
          s = rp[tr][rr] ? static_cast<const float*>(a.scales)[rows[tr][rr]] : 0.f;
        float m = -(float)F::kOffset * s;
        S_u[tr][rr] = kPow * s;
        M_u[tr][rr] = m - kPow * s;
      }
  }

  float yacc[TR][NT][2];
  float acc_u[TR][NT][4];
  float sx_u[NT];
#pragma unroll
  for (int tr = 0; tr < TR; ++tr)
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      yacc[tr][i][0] = yacc[tr][i][1] = 0.f;
      acc_u[tr][i][0] = acc_u[tr][i][1] = acc_u[tr][i][2] = acc_u[tr][i][3] = 0.f;
    }
#pragma unroll
  for (int i = 0; i < NT; ++i) sx_u[i] = 0.f;

  uint32_t wc[TR][2][4];
#pragma unroll
  for (int tr = 0; tr < TR; ++tr)
#pragma unroll
    for (int rr = 0; rr < 2; ++rr) load_words<FMT>(rp[tr][rr], g_begin, a.row_words, c, wc[tr][rr]);

  for (int g = g_begin; g < g_end; ++g) {
    uint32_t wn[TR][2][4];
    if (g + 1 < g_end) {
#pragma unroll
      for (int tr = 0; tr < TR; ++tr)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) load_words<FMT>(rp[tr][rr], g + 1, a.row_words, c, wn[tr][rr]);
    }
    // B fragments of x' for this group (slots >= 2N are zero and skipped)
    uint2 bf[NT][8];
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      const bool live = (8 * i + rq) < 2 * a.N;
      const uint2* src = a.xfrag + ((size_t)(i * a.Gp + g) * 8) * 32 + lane;
#pragma unroll
      for (int j = 0; j < 8; ++j) bf[i][j] = live ? __ldg(src + 32 * j) : make_uint2(0u, 0u);
    }
    float sxt[NT];
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      const float2 s2 = *reinterpret_cast<const float2*>(a.sx + (size_t)g * (8 * NT) + 8 * i + 2 * c);
      sxt[i] = s2.x + s2.y;
    }
    float Sg[TR][2], Mg[TR][2];
    if constexpr (SMODE == kScaleGroup) {
#pragma unroll
      for (int tr = 0; tr < TR; ++tr)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          float s = 0.f, m = 0.f;
          if (rp[tr][rr]) {
            size_t si = (size_t)rows[tr][rr] * a.G + g;
            s = __half2float(static_cast<const __half*>(a.scales)[si]);
            m = __half2float(a.mins[si]);
          }
          Sg[tr][rr] = kPow * s;
          Mg[tr][rr] = m - kPow * s;
        }
    }
#pragma unroll
    for (int tr = 0; tr < TR; ++tr) {
      uint32_t h0[16], h1[16];
      Dec<FMT>::run(wc[tr][0], c, h0);
      Dec<FMT>::run(wc[tr][1], c, h1);
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        if constexpr (SMODE == kScaleGroup) {
          float acc[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
          for (int j = 0; j < 8; ++j)
            mma16816(acc, h0[2 * j], h1[2 * j], h0[2 * j + 1], h1[2 * j + 1], bf[i][j].x, bf[i][j].y);
          yacc[tr][i][0] += Sg[tr][0] * (acc[0] + acc[1]) + Mg[tr][0] * sxt[i];
          yacc[tr][i][1] += Sg[tr][1] * (acc[2] + acc[3]) + Mg[tr][1] * sxt[i];
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j)
            mma16816(acc_u[tr][i], h0[2 * j], h1[2 * j], h0[2 * j + 1], h1[2 * j + 1], bf[i][j].x, bf[i][j].y);
        }
      }
    }
    if constexpr (SMODE != kScaleGroup) {
#pragma unroll
      for (int i = 0; i < NT; ++i) sx_u[i] += sxt[i];
    }
    if (g + 1 < g_end) {
#pragma unroll
      for (int tr = 0; tr < TR; ++tr)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr)
#pragma unroll
          for (int q = 0; q < 4; ++q) wc[tr][rr][q] = wn[tr][rr][q];
    }
  }

  if constexpr (SMODE != kScaleGroup) {
#pragma unroll
    for (int tr = 0; tr < TR; ++tr)
#pragma unroll
      for (int i = 0; i < NT; ++i) {
        yacc[tr][i][0] = S_u[tr][0] * (acc_u[tr][i][0] + acc_u[tr][i][1]) + M_u[tr][0] * sx_u[i];
        yacc[tr][i][1] = S_u[tr][1] * (acc_u[tr][i][2] + acc_u[tr][i][3]) + M_u[tr][1] * sx_u[i];
      }
  }

  // Split-K combine.  One chunk: write y directly.  Several chunks: every
  // item stores its partial, the last item of a row block (found with a
  // counter) sums the partials in chunk order -- deterministic, no atomics
  // on y -- adds the bias, writes y and re-arms the counter.
  if (a.n_chunks == 1) {
#pragma unroll
    for (int i = 0; i < NT; ++i) {
      const int t = 4 * i + c;
      if (t < a.N) {
#pragma unroll
        for (int tr = 0; tr < TR; ++tr)
#pragma unroll
          for (int rr = 0; rr < 2; ++rr)
            if (rp[tr][rr])
              a.y[(size_t)t * a.M + rows[tr][rr]] = yacc[tr][i][rr] + (a.bias ? a.bias[rows[tr][rr]] : 0.f);
      }
    }
    return;
  }
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    const int t = 4 * i + c;
    if (t < a.N) {
#pragma unroll
      for (int tr = 0; tr < TR; ++tr)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr)
          if (rp[tr][rr]) a.partials[((size_t)chunk * a.N + t) * a.M + rows[tr][rr]] = yacc[tr][i][rr];
    }
  }
  __threadfence();
  __syncwarp();
  unsigned prev = 0;
  if (lane == 0) prev = atomicAdd(a.counters + ritem, 1u);
  prev = __shfl_sync(0xffffffffu, prev, 0);
  if (prev != (unsigned)(a.n_chunks - 1)) return;
  __threadfence();
#pragma unroll
  for (int i = 0; i < NT; ++i) {
    const int t = 4 * i + c;
    if (t < a.N) {
#pragma unroll
      for (int tr = 0; tr < TR; ++tr)
#pragma unroll
        for (int rr = 0; rr < 2; ++rr) {
          if (!rp[tr][rr]) continue;
          const int row = rows[tr][rr];
          float v = 0.f;
          for (int ch = 0; ch < a.n_chunks; ++ch)
            v += (ch == chunk) ? yacc[tr][i][rr] : __ldcg(a.partials + ((size_t)ch * a.N + t) * a.M + row);
          a.y[(size_t)t * a.M + row] = v + (a.bias ? a.bias[row] : 0.f);
        }
    }
  }
  if (lane == 0) a.counters[ritem] = 0u;
}

template <int FMT, int NT, int TR>
cudaError_t launch_fmt_nt(const GemvIntArgs& a, int smode, cudaStream_t s) {
  dim3 grid((a.n_items + kWarps - 1) / kWarps);
  if (smode == kScaleGroup)
    gemv_int_kernel<FMT, NT, TR, kScaleGroup><<<grid, kWarps * 32, 0, s>>>(a);
  else if (smode == kScaleRow)
    gemv_int_kernel<FMT, NT, TR, kScaleRow><<<grid, kWarps * 32, 0, s>>>(a);
  else
    gemv_int_kernel<FMT, NT, TR, kScaleTensor><<<grid, kWarps * 32, 0, s>>>(a);
  note_launch();
  return cudaGetLastError();
}

template <int FMT>
cudaError_t launch_fmt(const GemvIntArgs& a, int smode, cudaStream_t s) {
  switch (a.NT) {
    case 1: return launch_fmt_nt<FMT, 1, 2>(a, smode, s);
    case 2: return launch_fmt_nt<FMT, 2, 2>(a, smode, s);
    default: return launch_fmt_nt<FMT, 4, 1>(a, smode, s);
  }
}

}  // namespace

int gemv_int_rows_per_item(int NT) { return NT <= 2 ? 32 : 16; }

cudaError_t launch_gemv_int(int fmt, const GemvIntArgs& a, int smode, cudaStream_t s) {
  switch (fmt) {
    case PF_FMT_INT4_G128: return launch_fmt<PF_FMT_INT4_G128>(a, smode, s);
    case PF_FMT_INT3_G128: return launch_fmt<PF_FMT_INT3_G128>(a, smode, s);
    case PF_FMT_INT2_G128: return launch_fmt<PF_FMT_INT2_G128>(a, smode, s);
    case PF_FMT_INT4: return launch_fmt<PF_FMT_INT4>(a, smode, s);
    case PF_FMT_INT3: return launch_fmt<PF_FMT_INT3>(a, smode, s);
    case PF_FMT_INT2: return launch_fmt<PF_FMT_INT2>(a, smode, s);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace pfb
