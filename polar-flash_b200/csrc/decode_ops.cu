// Decode-step kernels around the packed linears (batch 1, fp32): the
// residual add + RMSNorm, RoPE with the KV-cache write, a GQA attention over
// the cache and the SwiGLU gate.  They restate the reference decode forward
// (polarflash_core/model_integration.py: RMSNorm :27-37, apply_rotary_pos_emb
// :40-60, PFlashAttentionBlock.forward :97-147, PFlashMLPBlock.forward
// :160-163) for one new token, reading the token's position from device
// memory so that a whole step can be captured once as a CUDA graph.
#include <math.h>

#include "common.cuh"
#include "gemv.cuh"

namespace pfb {
namespace {

constexpr int kNormThreads = 256;
constexpr int kAttnThreads = 256;
constexpr int kDecodeMaxSeq = 32768;  // positions one attention call may cover

// Programmatic dependent launch: every kernel here lets the next launch start
// and waits for the previous grid to complete before touching its data.
__device__ __forceinline__ void pdl_enter() {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ float block_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  __syncthreads();  // red is reused by consecutive reductions
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float s = 0.f;
  for (int w = 0; w < (int)(blockDim.x >> 5); ++w) s += red[w];
  return s;
}

// One row per block: h += delta (when given), out = h / sqrt(mean(h^2) + eps) * w.
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_kernel(float* __restrict__ h, const float* __restrict__ delta,
                                                                   const float* __restrict__ w, float* __restrict__ out,
                                                                   int H, float eps) {
  __shared__ float red[kNormThreads / 32];
  pdl_enter();
  float* hr = h + (size_t)blockIdx.x * H;
  const float* dr = delta ? delta + (size_t)blockIdx.x * H : nullptr;
  float ss = 0.f;
  for (int i = threadIdx.x; i < H; i += blockDim.x) {
    float v = hr[i];
    if (dr) {
      v += dr[i];
      hr[i] = v;
    }
    ss += v * v;
  }
  const float r = rsqrtf(block_sum(ss, red) / (float)H + eps);
  for (int i = threadIdx.x; i < H; i += blockDim.x) out[(size_t)blockIdx.x * H + i] = hr[i] * r * w[i];
}

// The same for rows of H % 4 == 0 floats (16-byte aligned): each thread
// issues all its float4 loads of h, delta and w (at most V of each) before
// any arithmetic, so a row costs one memory latency instead of one per
// strided iteration.
template <int V>
__global__ void __launch_bounds__(kNormThreads) add_rmsnorm_vec_kernel(float* __restrict__ h,
                                                                       const float* __restrict__ delta,
                                                                       const float* __restrict__ w,
                                                                       float* __restrict__ out, int H, float eps) {
  __shared__ float red[kNormThreads / 32];
  pdl_enter();
  const int n4 = H >> 2;
  float4* hr = reinterpret_cast<float4*>(h + (size_t)blockIdx.x * H);
  const float4* dr = delta ? reinterpret_cast<const float4*>(delta + (size_t)blockIdx.x * H) : nullptr;
  const float4* wr = reinterpret_cast<const float4*>(w);
  float4 hv[V], dv[V], wv[V];
#pragma unroll
  for (int k = 0; k < V; ++k) {
    const int i = threadIdx.x + k * kNormThreads;
    if (i < n4) {
      hv[k] = hr[i];
      dv[k] = dr ? dr[i] : make_float4(0.f, 0.f, 0.f, 0.f);
      wv[k] = wr[i];
    }
  }
  float ss = 0.f;
#pragma unroll
  for (int k = 0; k < V; ++k) {
    const int i = threadIdx.x + k * kNormThreads;
    if (i < n4) {
      if (dr) {
        hv[k].x += dv[k].x;
        hv[k].y += dv[k].y;
        hv[k].z += dv[k].z;
        hv[k].w += dv[k].w;
        hr[i] = hv[k];
      }
      ss += hv[k].x * hv[k].x;
      ss += hv[k].y * hv[k].y;
      ss += hv[k].z * hv[k].z;
      ss += hv[k].w * hv[k].w;
    }
  }
  const float r = rsqrtf(block_sum(ss, red) / (float)H + eps);
  float4* orow = reinterpret_cast<float4*>(out + (size_t)blockIdx.x * H);
#pragma unroll
  for (int k = 0; k < V; ++k) {
    const int i = threadIdx.x + k * kNormThreads;
    if (i < n4)
      orow[i] = make_float4(hv[k].x * r * wv[k].x, hv[k].y * r * wv[k].y, hv[k].z * r * wv[k].z,
                            hv[k].w * r * wv[k].w);
  }
}

// The pair (x1, x2) rotated by the angle with cosine c and sine s, each
// product and sum rounded on its own (as the reference's separate tensor
// ops round them; no fma contraction, so every kernel rotates alike).
__device__ __forceinline__ void rope_pair(float x1, float x2, float c, float s, float& o1, float& o2) {
  o1 = __fsub_rn(__fmul_rn(x1, c), __fmul_rn(x2, s));
  o2 = __fadd_rn(__fmul_rn(x1, s), __fmul_rn(x2, c));
}

// Blocks 0..nh-1 rotate q's heads in place; blocks nh..nh+nkv-1 rotate k's
// heads into the key cache at position *pos and copy v's heads into the value
// cache there.  Thread i handles the pair (i, i + hd/2): angle pos * inv_freq[i].
__global__ void rope_kv_kernel(float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                               float* __restrict__ kc, float* __restrict__ vc, const long long* __restrict__ pos,
                               const float* __restrict__ inv_freq, int nh, int nkv, int hd, int max_seq) {
  pdl_enter();
  const long long p = *pos;
  if (p < 0 || p >= max_seq) return;  // rejected on the host when it can see it; never written out of range
  const int half = hd >> 1, i = threadIdx.x;
  if (i >= half) return;
  const float f = (float)p * inv_freq[i];
  const float c = cosf(f), s = sinf(f);
  const int head = blockIdx.x;
  if (head < nh) {
    float* x = q + (size_t)head * hd;
    rope_pair(x[i], x[i + half], c, s, x[i], x[i + half]);
  } else {
    const int kh = head - nh;
    const float* x = k + (size_t)kh * hd;
    const float x1 = x[i], x2 = x[i + half];
    float* kd = kc + ((size_t)p * nkv + kh) * hd;
    rope_pair(x1, x2, c, s, kd[i], kd[i + half]);
    float* vd = vc + ((size_t)p * nkv + kh) * hd;
    const float* vs = v + (size_t)kh * hd;
    vd[i] = vs[i];
    vd[i + half] = vs[i + half];
  }
}

// ---- compressed KV cache ----------------------------------------------------
// Rows of head_dim values (one token of one KV head) quantized as
// CompressedKVCache does (polarflash_rt/kv_cache/compressed_kv.py):
//   int8 (:68-77):      s = max(max|x| / 127, 1e-8), c = clamp(rint(x / s), -128, 127), x' = c s
//   2bit (:79-112):     s = max(max|x| / 1.75, 1e-8), c = clamp(floor(x / s + 2), 0, 3), x' = (c - 1.5) s
//   2bit_asym (:114-150): z = min x, s = max((max x - z) / 3, 1e-8), c = clamp(rint((x - z) / s), 0, 3),
//                       x' = c s + z
// 2-bit codes are packed four to a byte, first value in the top bits
// (c0 << 6 | c1 << 4 | c2 << 2 | c3), a ragged last byte padded with zero
// codes.  Every operation is an explicitly rounded single-precision op (no
// contraction to fma), so codes, scales and dequantized values are
// bit-identical to the reference's fp32 arithmetic.
template <bool kMin>
__device__ __forceinline__ float block_minmax(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = kMin ? fminf(v, w) : fmaxf(v, w);
  }
  __syncthreads();  // red is reused by consecutive reductions
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  float r = red[0];
  for (int w = 1; w < (int)(blockDim.x >> 5); ++w) r = kMin ? fminf(r, red[w]) : fmaxf(r, red[w]);
  return r;
}

// The whole block (a multiple of 32 threads) quantizes the row x[0..dim).
template <int MODE>
__device__ void quantize_row(const float* x, int dim, uint8_t* codes, float* scale_out, float* zero_out, float* red) {
  const int t = threadIdx.x, nt = blockDim.x;
  float lo = INFINITY, hi = MODE == PF_KV_2BIT_ASYM ? -INFINITY : 0.f;
  for (int i = t; i < dim; i += nt) {
    const float v = x[i];
    if (MODE == PF_KV_2BIT_ASYM) {
      lo = fminf(lo, v);
      hi = fmaxf(hi, v);
    } else {
      hi = fmaxf(hi, fabsf(v));
    }
  }
  float z = 0.f, s;
  hi = block_minmax<false>(hi, red);
  if (MODE == PF_KV_2BIT_ASYM) z = block_minmax<true>(lo, red);
  if (MODE == PF_KV_INT8)
    s = fmaxf(__fdiv_rn(hi, 127.f), 1e-8f);
  else if (MODE == PF_KV_2BIT)
    s = fmaxf(__fdiv_rn(hi, 1.75f), 1e-8f);
  else
    s = fmaxf(__fdiv_rn(__fsub_rn(hi, z), 3.f), 1e-8f);
  if (MODE == PF_KV_INT8) {
    for (int i = t; i < dim; i += nt) {
      const float r = fminf(fmaxf(rintf(__fdiv_rn(x[i], s)), -128.f), 127.f);
      reinterpret_cast<int8_t*>(codes)[i] = (int8_t)(int)r;
    }
  } else {
    for (int j = t; j < (dim + 3) >> 2; j += nt) {
      unsigned byte = 0;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int i = 4 * j + e;
        if (i < dim) {
          const float r = MODE == PF_KV_2BIT ? floorf(__fadd_rn(__fdiv_rn(x[i], s), 2.f))
                                             : rintf(__fdiv_rn(__fsub_rn(x[i], z), s));
          byte |= (unsigned)fminf(fmaxf(r, 0.f), 3.f) << (6 - 2 * e);
        }
      }
      codes[j] = (uint8_t)byte;
    }
  }
  if (t == 0) {
    *scale_out = s;
    if (MODE == PF_KV_2BIT_ASYM) *zero_out = z;
  }
}

// Value d of a quantized row (codes of the row, its scale and zero).
template <int MODE>
__device__ __forceinline__ float kv_value(const uint8_t* row, int d, float s, float z) {
  if (MODE == PF_KV_INT8) return __fmul_rn((float)reinterpret_cast<const int8_t*>(row)[d], s);
  const float c = (float)((row[d >> 2] >> (6 - 2 * (d & 3))) & 3u);
  if (MODE == PF_KV_2BIT) return __fmul_rn(__fsub_rn(c, 1.5f), s);
  return __fadd_rn(__fmul_rn(c, s), z);
}

__host__ __device__ __forceinline__ int kv_row_bytes(int mode, int dim) {
  return mode == PF_KV_INT8 ? dim : mode == PF_KV_FP32 ? 4 * dim : (dim + 3) / 4;
}

constexpr int kQuantThreads = 128;

template <int MODE>
__global__ void __launch_bounds__(kQuantThreads) kv_quantize_kernel(const float* __restrict__ x, int dim,
                                                                    uint8_t* __restrict__ codes,
                                                                    float* __restrict__ scales,
                                                                    float* __restrict__ zeros) {
  __shared__ float red[kQuantThreads / 32];
  pdl_enter();
  const size_t r = blockIdx.x;
  quantize_row<MODE>(x + r * dim, dim, codes + r * kv_row_bytes(MODE, dim), scales + r, zeros ? zeros + r : nullptr,
                     red);
}

template <int MODE>
__global__ void kv_dequantize_kernel(const uint8_t* __restrict__ codes, const float* __restrict__ scales,
                                     const float* __restrict__ zeros, long long rows, int dim,
                                     float* __restrict__ out) {
  pdl_enter();
  const long long n = rows * dim;
  const int rb = kv_row_bytes(MODE, dim);
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const long long r = i / dim;
    const int d = (int)(i - r * dim);
    out[i] = kv_value<MODE>(codes + r * rb, d, scales[r], MODE == PF_KV_2BIT_ASYM ? zeros[r] : 0.f);
  }
}

// As rope_kv_kernel, with the rotated key and the value quantized into the
// compressed caches' row (*pos, head).  Blocks of the KV heads stage both
// rows in shared memory and quantize them with the whole block.
constexpr int kRopeMaxHd = 2048;

struct KvRows {  // one layer's compressed cache: rows [max_seq][n_kv_heads]
  uint8_t* codes;
  float* scales;
  float* zeros;  // 2bit_asym only
};

template <int MODE>
__global__ void rope_kvq_kernel(float* __restrict__ q, const float* __restrict__ k, const float* __restrict__ v,
                                KvRows kc, KvRows vc, const long long* __restrict__ pos,
                                const float* __restrict__ inv_freq, int nh, int nkv, int hd, int max_seq) {
  __shared__ float xs[2][kRopeMaxHd];
  __shared__ float red[32];
  pdl_enter();
  const long long p = *pos;
  if (p < 0 || p >= max_seq) return;  // block-uniform
  const int half = hd >> 1, head = blockIdx.x;
  if (head < nh) {
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
      const float f = (float)p * inv_freq[i];
      const float c = cosf(f), s = sinf(f);
      float* x = q + (size_t)head * hd;
      rope_pair(x[i], x[i + half], c, s, x[i], x[i + half]);
    }
    return;  // block-uniform
  }
  const int kh = head - nh;
  for (int i = threadIdx.x; i < half; i += blockDim.x) {
    const float f = (float)p * inv_freq[i];
    const float c = cosf(f), s = sinf(f);
    const float* x = k + (size_t)kh * hd;
    rope_pair(x[i], x[i + half], c, s, xs[0][i], xs[0][i + half]);
    xs[1][i] = v[(size_t)kh * hd + i];
    xs[1][i + half] = v[(size_t)kh * hd + i + half];
  }
  __syncthreads();
  const size_t r = (size_t)p * nkv + kh;
  const int rb = kv_row_bytes(MODE, hd);
  quantize_row<MODE>(xs[0], hd, kc.codes + r * rb, kc.scales + r, kc.zeros ? kc.zeros + r : nullptr, red);
  quantize_row<MODE>(xs[1], hd, vc.codes + r * rb, vc.scales + r, vc.zeros ? vc.zeros + r : nullptr, red);
}

// Attention of one new token over positions 0..*pos of the cache, split over
// chunks of kAttnChunk positions (flash decoding).  attn_chunk_kernel: one
// block per (KV head, chunk) serves the KV head's G query heads.  Each cache
// row (one position of one KV head) is read as vectors, four consecutive
// head dimensions per thread: a float4 of the fp32 cache, one 32-bit word of
// int8 codes or one byte of 2-bit codes, with the row's scale (and zero)
// loaded once.  Scores: one warp per position, eight positions per warp in
// flight, their dot products reduced over the warp together; then the
// chunk's softmax statistics; then the value sums, thread groups of
// head_dim / 4 threads over the chunk's positions (all of a thread's
// positions loaded in one batch), merged across groups in shared memory.
// It stores per query head (max, sum of exponentials, unnormalised output);
// chunks past *pos store an empty entry (never read).
// attn_combine_kernel merges a head's chunks:
// out = sum_c e^(m_c - m) o_c / sum_c e^(m_c - m) l_c.
constexpr int kAttnChunk = 64;
constexpr int kAttnG = 8;  // query heads per KV head handled by one block

// KV cache rows [max_seq][n_kv_heads]: fp32 values, or codes with a scale
// (and, for 2bit_asym, a zero) per row.
struct KvView {
  const void* codes;
  const float* scales;
  const float* zeros;
};

// Values d0..d0+3 of row r (d0 and head_dim multiples of 4) in two steps:
// kv_fetch issues the loads (a float4 of the fp32 cache; one 32-bit word of
// int8 codes or one byte of 2-bit codes, with the row's scale and zero),
// kv_decode does the arithmetic.  Loops fetch all their rows first and decode
// afterwards, so the loads of every row are in flight together; rows outside
// the chunk are zero-filled, which decodes to zeros in every mode.
struct KvRaw {
  float4 f;    // fp32 values
  unsigned w;  // int8 codes (d0 in the low byte) or the 2-bit code byte
  float s, z;  // scale, zero
};

template <int MODE>
__device__ __forceinline__ void kv_fetch(const KvView& c, size_t r, int d0, int hd, KvRaw& x) {
  if (MODE == PF_KV_FP32) {
    x.f = __ldg(reinterpret_cast<const float4*>(static_cast<const float*>(c.codes) + r * hd + d0));
    return;
  }
  const uint8_t* row = static_cast<const uint8_t*>(c.codes) + r * kv_row_bytes(MODE, hd);
  x.s = __ldg(c.scales + r);
  if (MODE == PF_KV_2BIT_ASYM) x.z = __ldg(c.zeros + r);
  if (MODE == PF_KV_INT8)
    x.w = __ldg(reinterpret_cast<const unsigned*>(row + d0));
  else
    x.w = __ldg(row + (d0 >> 2));
}

__device__ __forceinline__ void kv_zero(KvRaw& x) {
  x.f = make_float4(0.f, 0.f, 0.f, 0.f);
  x.w = 0u;
  x.s = 0.f;
  x.z = 0.f;
}

template <int MODE>
__device__ __forceinline__ void kv_decode(const KvRaw& x, float v[4]) {
  if (MODE == PF_KV_FP32) {
    v[0] = x.f.x;
    v[1] = x.f.y;
    v[2] = x.f.z;
    v[3] = x.f.w;
  } else if (MODE == PF_KV_INT8) {
#pragma unroll
    for (int i = 0; i < 4; ++i) v[i] = __fmul_rn((float)(int)(signed char)((x.w >> (8 * i)) & 0xffu), x.s);
  } else {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float cv = (float)((x.w >> (6 - 2 * i)) & 3u);
      v[i] = MODE == PF_KV_2BIT ? __fmul_rn(__fsub_rn(cv, 1.5f), x.s) : __fadd_rn(__fmul_rn(cv, x.s), x.z);
    }
  }
}

template <int MODE>
__global__ void __launch_bounds__(kAttnThreads, 3) attn_chunk_kernel(const float* __restrict__ q, KvView kc,
                                                                     KvView vc, const long long* __restrict__ pos,
                                                                     float* __restrict__ part, int nh, int nkv,
                                                                     int hd, int max_seq, int nchunk, float scale) {
  __shared__ __align__(16) float qs[kAttnG][128];
  __shared__ float sc[kAttnG][kAttnChunk];
  __shared__ float mx[kAttnG], sm[kAttnG];
  __shared__ float po[kAttnG * 1024];  // [group][g][hd]: groups x head_dim <= 1024
  const int kvh = blockIdx.x, chunk = blockIdx.y, G = nh / nkv;
  pdl_enter();
  const long long p = *pos;
  const int T = (p < 0) ? 0 : (p >= max_seq ? max_seq : (int)p + 1);
  const int t0 = chunk * kAttnChunk, t1 = min(T, t0 + kAttnChunk), n = t1 - t0;
  const int rec = hd + 2;  // per (head, chunk): m, l, o[hd]
  if (n <= 0) {
    for (int g = threadIdx.x; g < G; g += blockDim.x) {
      float* r = part + ((size_t)(kvh * G + g) * nchunk + chunk) * rec;
      r[0] = -INFINITY;
      r[1] = 0.f;
    }
    return;
  }
  for (int i = threadIdx.x; i < G * hd; i += blockDim.x) qs[i / hd][i % hd] = q[(size_t)(kvh * G + i / hd) * hd + i % hd];
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  const int d0 = 4 * lane;
  const bool act = d0 < hd;
  // scores: warp w takes positions t0 + w, t0 + w + nw, ... (eight at a time)
  for (int j0 = warp; j0 < n; j0 += 8 * nw) {
    float kv[8][4];
    {
      KvRaw raw[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = j0 + u * nw;
        kv_zero(raw[u]);
        if (act && j < n) kv_fetch<MODE>(kc, (size_t)(t0 + j) * nkv + kvh, d0, hd, raw[u]);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) kv_decode<MODE>(raw[u], kv[u]);
    }
    for (int g = 0; g < G; ++g) {
      const float4 qv = act ? *reinterpret_cast<const float4*>(&qs[g][d0]) : make_float4(0.f, 0.f, 0.f, 0.f);
      float a[8];
#pragma unroll
      for (int u = 0; u < 8; ++u) a[u] = qv.x * kv[u][0] + qv.y * kv[u][1] + qv.z * kv[u][2] + qv.w * kv[u][3];
      // Transpose-reduce the eight dot products over the warp (9 shuffles,
      // not 40): at the xor-16, 8 and 4 steps each lane keeps half of its
      // partial sums (the upper half when its lane bit is set) and adds the
      // partner's copy of that half, so lane l ends with a partial sum of
      // position u = (l >> 2) & 7; the xor-2 and 1 steps complete it.
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const bool up = lane & 16;
        const float send = up ? a[i] : a[i + 4], keep = up ? a[i + 4] : a[i];
        a[i] = keep + __shfl_xor_sync(0xffffffffu, send, 16);
      }
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const bool up = lane & 8;
        const float send = up ? a[i] : a[i + 2], keep = up ? a[i + 2] : a[i];
        a[i] = keep + __shfl_xor_sync(0xffffffffu, send, 8);
      }
      {
        const bool up = lane & 4;
        const float send = up ? a[0] : a[1], keep = up ? a[1] : a[0];
        a[0] = keep + __shfl_xor_sync(0xffffffffu, send, 4);
      }
      float dot = a[0];
      dot += __shfl_xor_sync(0xffffffffu, dot, 2);
      dot += __shfl_xor_sync(0xffffffffu, dot, 1);
      const int j = j0 + ((lane >> 2) & 7) * nw;
      if ((lane & 3) == 0 && j < n) sc[g][j] = dot * scale;
    }
  }
  __syncthreads();
  // per query head: chunk max and exponentials (warp g)
  if (warp < G) {
    float m = -INFINITY;
    for (int j = lane; j < n; j += 32) m = fmaxf(m, sc[warp][j]);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    float l = 0.f;
    for (int j = lane; j < n; j += 32) {
      const float e = expf(sc[warp][j] - m);
      sc[warp][j] = e;
      l += e;
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) l += __shfl_xor_sync(0xffffffffu, l, o);
    if (lane == 0) {
      mx[warp] = m;
      sm[warp] = l;
    }
  }
  __syncthreads();
  // values: group gi (head_dim / 4 threads, thread li holds dimensions
  // 4 li .. 4 li + 3) sums positions gi, gi + ngr, ... for every query head
  const int tpr = hd >> 2, ngr = blockDim.x / tpr;
  const int gi = threadIdx.x / tpr, e0 = 4 * (threadIdx.x % tpr);
  if (gi < ngr) {
    float acc[kAttnG][4];
#pragma unroll
    for (int g = 0; g < kAttnG; ++g)
#pragma unroll
      for (int i = 0; i < 4; ++i) acc[g][i] = 0.f;
    for (int jb = gi; jb < n; jb += 8 * ngr) {
      float val[8][4];
      {
        KvRaw raw[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          const int j = jb + u * ngr;
          kv_zero(raw[u]);
          if (j < n) kv_fetch<MODE>(vc, (size_t)(t0 + j) * nkv + kvh, e0, hd, raw[u]);
        }
#pragma unroll
        for (int u = 0; u < 8; ++u) kv_decode<MODE>(raw[u], val[u]);
      }
#pragma unroll
      for (int u = 0; u < 8; ++u) {
        const int j = jb + u * ngr;
        if (j < n) {
#pragma unroll
          for (int g = 0; g < kAttnG; ++g) {
            if (g < G) {
              const float w = sc[g][j];
#pragma unroll
              for (int i = 0; i < 4; ++i) acc[g][i] += w * val[u][i];
            }
          }
        }
      }
    }
#pragma unroll
    for (int g = 0; g < kAttnG; ++g) {
      if (g < G) {
#pragma unroll
        for (int i = 0; i < 4; ++i) po[(gi * G + g) * hd + e0 + i] = acc[g][i];
      }
    }
  }
  __syncthreads();
  for (int i = threadIdx.x; i < G * hd; i += blockDim.x) {
    const int g = i / hd, e = i % hd;
    float o = 0.f;
    for (int k = 0; k < ngr; ++k) o += po[(k * G + g) * hd + e];
    float* r = part + ((size_t)(kvh * G + g) * nchunk + chunk) * rec;
    r[2 + e] = o;
    if (e == 0) {
      r[0] = mx[g];
      r[1] = sm[g];
    }
  }
}

// Only the chunks that hold positions (all non-empty) are read; warps take
// chunks in turn (w, w + 8, ...) with lanes over head dimensions, and the
// eight warp partials are summed in shared memory.
constexpr int kCombThreads = 256;

__global__ void __launch_bounds__(kCombThreads) attn_combine_kernel(const float* __restrict__ part,
                                                                    const long long* __restrict__ pos,
                                                                    float* __restrict__ out, int hd, int nchunk,
                                                                    int max_seq) {
  __shared__ float so[kCombThreads / 32][128];
  __shared__ float sl[kCombThreads / 32];
  __shared__ float red[kCombThreads / 32];
  const int head = blockIdx.x, rec = hd + 2;
  pdl_enter();
  const long long p = *pos;
  const int T = (p < 0) ? 0 : (p >= max_seq ? max_seq : (int)p + 1);
  const int nc = min(nchunk, (T + kAttnChunk - 1) / kAttnChunk);
  const float* base = part + (size_t)head * nchunk * rec;
  float m = -INFINITY;
  for (int c = threadIdx.x; c < nc; c += blockDim.x) m = fmaxf(m, base[(size_t)c * rec]);
  m = block_minmax<false>(m, red);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  float o[4] = {0.f, 0.f, 0.f, 0.f}, l = 0.f;
#pragma unroll 4
  for (int c = warp; c < nc; c += nw) {
    const float* r = base + (size_t)c * rec;
    const float w = expf(r[0] - m);
    l += w * r[1];
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = lane + 32 * e;
      if (d < hd) o[e] += w * r[2 + d];
    }
  }
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const int d = lane + 32 * e;
    if (d < hd) so[warp][d] = o[e];
  }
  if (lane == 0) sl[warp] = l;
  __syncthreads();
  for (int d = threadIdx.x; d < hd; d += blockDim.x) {
    float a = 0.f, b = 0.f;
    for (int w = 0; w < nw; ++w) {
      a += so[w][d];
      b += sl[w];
    }
    out[(size_t)head * hd + d] = b > 0.f ? a / b : 0.f;
  }
}

__global__ void silu_mul_kernel(const float* __restrict__ g, const float* __restrict__ u, float* __restrict__ out,
                                long long n) {
  pdl_enter();
  for (long long i = (long long)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (long long)gridDim.x * blockDim.x) {
    const float x = g[i];
    out[i] = x / (1.f + expf(-x)) * u[i];
  }
}

int status_of(cudaError_t e) { return e == cudaSuccess ? PF_OK : PF_ERR_CUDA; }

template <typename... KArgs, typename... Args>
cudaError_t launch_pdl(void (*kern)(KArgs...), dim3 grid, int threads, cudaStream_t s, Args... args) {
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = dim3(threads);
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  const cudaError_t e = cudaLaunchKernelEx(&cfg, kern, static_cast<KArgs>(args)...);
  note_launch();
  return e != cudaSuccess ? e : cudaGetLastError();
}
bool al4(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 3u) == 0; }
bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

}  // namespace
}  // namespace pfb

using namespace pfb;

int pf_add_rmsnorm(float* h, const float* delta, const float* w, float* out, int rows, int H, float eps, void* stream) {
  if (!h || !w || !out || rows < 0 || H <= 0 || !(eps >= 0.f)) return PF_ERR_INVALID_ARGUMENT;
  if (!al4(h) || !al4(w) || !al4(out) || (delta && !al4(delta))) return PF_ERR_ALIGNMENT;
  if (rows == 0) return PF_OK;
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  const bool vec = H % 4 == 0 && al16(h) && al16(w) && al16(out) && (!delta || al16(delta));
  const int per = (H / 4 + kNormThreads - 1) / kNormThreads;  // float4 per thread
  if (vec && per <= 1) return status_of(launch_pdl(add_rmsnorm_vec_kernel<1>, dim3(rows), kNormThreads, st, h, delta, w, out, H, eps));
  if (vec && per <= 2) return status_of(launch_pdl(add_rmsnorm_vec_kernel<2>, dim3(rows), kNormThreads, st, h, delta, w, out, H, eps));
  if (vec && per <= 4) return status_of(launch_pdl(add_rmsnorm_vec_kernel<4>, dim3(rows), kNormThreads, st, h, delta, w, out, H, eps));
  if (vec && per <= 8) return status_of(launch_pdl(add_rmsnorm_vec_kernel<8>, dim3(rows), kNormThreads, st, h, delta, w, out, H, eps));
  return status_of(launch_pdl(add_rmsnorm_kernel, dim3(rows), kNormThreads, st, h, delta, w, out, H, eps));
}

int pf_rope_kv(float* q, const float* k, const float* v, float* k_cache, float* v_cache, const long long* pos,
               const float* inv_freq, int n_heads, int n_kv_heads, int head_dim, int max_seq, void* stream) {
  if (!q || !k || !v || !k_cache || !v_cache || !pos || !inv_freq) return PF_ERR_INVALID_ARGUMENT;
  if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || (head_dim & 1) || head_dim > 2048 || max_seq <= 0)
    return PF_ERR_SHAPE;
  if (!al4(q) || !al4(k) || !al4(v) || !al4(k_cache) || !al4(v_cache) || !al4(inv_freq) ||
      (reinterpret_cast<uintptr_t>(pos) & 7u))
    return PF_ERR_ALIGNMENT;
  return status_of(launch_pdl(rope_kv_kernel, dim3(n_heads + n_kv_heads), head_dim / 2,
                              static_cast<cudaStream_t>(stream), q, k, v, k_cache, v_cache, pos, inv_freq, n_heads,
                              n_kv_heads, head_dim, max_seq));
}

size_t pf_decode_attention_workspace_size(int n_heads, int head_dim, int max_seq) {
  if (n_heads <= 0 || head_dim <= 0 || max_seq <= 0) return 0;
  const size_t nchunk = ((size_t)max_seq + kAttnChunk - 1) / kAttnChunk;
  return (size_t)n_heads * nchunk * (head_dim + 2) * sizeof(float);
}

namespace {

bool kv_mode_ok(int mode) { return mode == PF_KV_INT8 || mode == PF_KV_2BIT || mode == PF_KV_2BIT_ASYM; }

int decode_attention(int mode, const float* q, KvView kc, KvView vc, const long long* pos, float* out, int n_heads,
                     int n_kv_heads, int head_dim, int max_seq, float scale, void* workspace, size_t workspace_bytes,
                     void* stream) {
  if (n_heads <= 0 || n_kv_heads <= 0 || n_heads % n_kv_heads || n_heads / n_kv_heads > kAttnG || head_dim <= 0 ||
      head_dim > 128 || (head_dim & 3) || max_seq <= 0 || max_seq > kDecodeMaxSeq)
    return PF_ERR_SHAPE;
  if (!al4(q) || !al4(out) || !al4(workspace) || (reinterpret_cast<uintptr_t>(pos) & 7u)) return PF_ERR_ALIGNMENT;
  // rows are read as float4 (fp32 cache) or 32-bit words (int8 codes)
  const uintptr_t need = mode == PF_KV_FP32 ? 15u : mode == PF_KV_INT8 ? 3u : 0u;
  if ((reinterpret_cast<uintptr_t>(kc.codes) | reinterpret_cast<uintptr_t>(vc.codes)) & need) return PF_ERR_ALIGNMENT;
  if (workspace_bytes < pf_decode_attention_workspace_size(n_heads, head_dim, max_seq)) return PF_ERR_WORKSPACE;
  const int nchunk = (max_seq + kAttnChunk - 1) / kAttnChunk;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  float* part = static_cast<float*>(workspace);
  const dim3 grid(n_kv_heads, nchunk);
  cudaError_t e;
  switch (mode) {
    case PF_KV_FP32:
      e = launch_pdl(attn_chunk_kernel<PF_KV_FP32>, grid, kAttnThreads, s, q, kc, vc, pos, part, n_heads, n_kv_heads,
                     head_dim, max_seq, nchunk, scale);
      break;
    case PF_KV_INT8:
      e = launch_pdl(attn_chunk_kernel<PF_KV_INT8>, grid, kAttnThreads, s, q, kc, vc, pos, part, n_heads, n_kv_heads,
                     head_dim, max_seq, nchunk, scale);
      break;
    case PF_KV_2BIT:
      e = launch_pdl(attn_chunk_kernel<PF_KV_2BIT>, grid, kAttnThreads, s, q, kc, vc, pos, part, n_heads, n_kv_heads,
                     head_dim, max_seq, nchunk, scale);
      break;
    default:
      e = launch_pdl(attn_chunk_kernel<PF_KV_2BIT_ASYM>, grid, kAttnThreads, s, q, kc, vc, pos, part, n_heads,
                     n_kv_heads, head_dim, max_seq, nchunk, scale);
  }
  if (e != cudaSuccess) return PF_ERR_CUDA;
  return status_of(launch_pdl(attn_combine_kernel, dim3(n_heads), kCombThreads, s, (const float*)part, pos, out,
                              head_dim, nchunk, max_seq));
}

}  // namespace

int pf_decode_attention(const float* q, const float* k_cache, const float* v_cache, const long long* pos, float* out,
                        int n_heads, int n_kv_heads, int head_dim, int max_seq, float scale, void* workspace,
                        size_t workspace_bytes, void* stream) {
  if (!q || !k_cache || !v_cache || !pos || !out || !workspace) return PF_ERR_INVALID_ARGUMENT;
  if (!al4(k_cache) || !al4(v_cache)) return PF_ERR_ALIGNMENT;
  return decode_attention(PF_KV_FP32, q, KvView{k_cache, nullptr, nullptr}, KvView{v_cache, nullptr, nullptr}, pos,
                          out, n_heads, n_kv_heads, head_dim, max_seq, scale, workspace, workspace_bytes, stream);
}

size_t pf_kv_row_bytes(int mode, int dim) {
  if (dim <= 0 || (mode != PF_KV_FP32 && !kv_mode_ok(mode))) return 0;
  return (size_t)kv_row_bytes(mode, dim);
}

int pf_kv_quantize(const float* x, long long rows, int dim, int mode, void* codes, float* scales, float* zeros,
                   void* stream) {
  if (!kv_mode_ok(mode) || !x || !codes || !scales || (mode == PF_KV_2BIT_ASYM && !zeros) || rows < 0)
    return PF_ERR_INVALID_ARGUMENT;
  if (dim <= 0 || rows > 0x7fffffffLL) return PF_ERR_SHAPE;
  if (!al4(x) || !al4(scales) || (zeros && !al4(zeros))) return PF_ERR_ALIGNMENT;
  if (rows == 0) return PF_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  uint8_t* c = static_cast<uint8_t*>(codes);
  float* z = mode == PF_KV_2BIT_ASYM ? zeros : nullptr;
  const dim3 grid((unsigned)rows);
  cudaError_t e;
  if (mode == PF_KV_INT8)
    e = launch_pdl(kv_quantize_kernel<PF_KV_INT8>, grid, kQuantThreads, s, x, dim, c, scales, z);
  else if (mode == PF_KV_2BIT)
    e = launch_pdl(kv_quantize_kernel<PF_KV_2BIT>, grid, kQuantThreads, s, x, dim, c, scales, z);
  else
    e = launch_pdl(kv_quantize_kernel<PF_KV_2BIT_ASYM>, grid, kQuantThreads, s, x, dim, c, scales, z);
  return status_of(e);
}

int pf_kv_dequantize(const void* codes, const float* scales, const float* zeros, long long rows, int dim, int mode,
                     float* out, void* stream) {
  if (!kv_mode_ok(mode) || !codes || !scales || !out || (mode == PF_KV_2BIT_ASYM && !zeros) || rows < 0)
    return PF_ERR_INVALID_ARGUMENT;
  if (dim <= 0) return PF_ERR_SHAPE;
  if (!al4(out) || !al4(scales) || (zeros && !al4(zeros))) return PF_ERR_ALIGNMENT;
  const long long n = rows * dim;
  if (n == 0) return PF_OK;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const uint8_t* c = static_cast<const uint8_t*>(codes);
  const long long blocks = (n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096;
  const dim3 grid((unsigned)blocks);
  cudaError_t e;
  if (mode == PF_KV_INT8)
    e = launch_pdl(kv_dequantize_kernel<PF_KV_INT8>, grid, 256, s, c, scales, zeros, rows, dim, out);
  else if (mode == PF_KV_2BIT)
    e = launch_pdl(kv_dequantize_kernel<PF_KV_2BIT>, grid, 256, s, c, scales, zeros, rows, dim, out);
  else
    e = launch_pdl(kv_dequantize_kernel<PF_KV_2BIT_ASYM>, grid, 256, s, c, scales, zeros, rows, dim, out);
  return status_of(e);
}

int pf_rope_kv_compressed(float* q, const float* k, const float* v, void* k_codes, float* k_scales, float* k_zeros,
                          void* v_codes, float* v_scales, float* v_zeros, const long long* pos, const float* inv_freq,
                          int n_heads, int n_kv_heads, int head_dim, int max_seq, int mode, void* stream) {
  if (!kv_mode_ok(mode) || !q || !k || !v || !k_codes || !k_scales || !v_codes || !v_scales || !pos || !inv_freq ||
      (mode == PF_KV_2BIT_ASYM && (!k_zeros || !v_zeros)))
    return PF_ERR_INVALID_ARGUMENT;
  if (n_heads <= 0 || n_kv_heads <= 0 || head_dim <= 0 || (head_dim & 1) || head_dim > kRopeMaxHd || max_seq <= 0)
    return PF_ERR_SHAPE;
  if (!al4(q) || !al4(k) || !al4(v) || !al4(k_scales) || !al4(v_scales) || !al4(inv_freq) ||
      (k_zeros && !al4(k_zeros)) || (v_zeros && !al4(v_zeros)) || (reinterpret_cast<uintptr_t>(pos) & 7u))
    return PF_ERR_ALIGNMENT;
  const bool asym = mode == PF_KV_2BIT_ASYM;
  const KvRows kc{static_cast<uint8_t*>(k_codes), k_scales, asym ? k_zeros : nullptr};
  const KvRows vc{static_cast<uint8_t*>(v_codes), v_scales, asym ? v_zeros : nullptr};
  const int threads = ((head_dim / 2 + 31) / 32) * 32;  // whole warps: the row reductions shuffle over full warps
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const dim3 grid(n_heads + n_kv_heads);
  cudaError_t e;
  if (mode == PF_KV_INT8)
    e = launch_pdl(rope_kvq_kernel<PF_KV_INT8>, grid, threads, s, q, k, v, kc, vc, pos, inv_freq, n_heads, n_kv_heads,
                   head_dim, max_seq);
  else if (mode == PF_KV_2BIT)
    e = launch_pdl(rope_kvq_kernel<PF_KV_2BIT>, grid, threads, s, q, k, v, kc, vc, pos, inv_freq, n_heads, n_kv_heads,
                   head_dim, max_seq);
  else
    e = launch_pdl(rope_kvq_kernel<PF_KV_2BIT_ASYM>, grid, threads, s, q, k, v, kc, vc, pos, inv_freq, n_heads,
                   n_kv_heads, head_dim, max_seq);
  return status_of(e);
}

int pf_decode_attention_compressed(const float* q, const void* k_codes, const float* k_scales, const float* k_zeros,
                                   const void* v_codes, const float* v_scales, const float* v_zeros,
                                   const long long* pos, float* out, int n_heads, int n_kv_heads, int head_dim,
                                   int max_seq, int mode, float scale, void* workspace, size_t workspace_bytes,
                                   void* stream) {
  if (!kv_mode_ok(mode) || !q || !k_codes || !k_scales || !v_codes || !v_scales || !pos || !out || !workspace ||
      (mode == PF_KV_2BIT_ASYM && (!k_zeros || !v_zeros)))
    return PF_ERR_INVALID_ARGUMENT;
  if (!al4(k_scales) || !al4(v_scales) || (k_zeros && !al4(k_zeros)) || (v_zeros && !al4(v_zeros)))
    return PF_ERR_ALIGNMENT;
  return decode_attention(mode, q, KvView{k_codes, k_scales, k_zeros}, KvView{v_codes, v_scales, v_zeros}, pos, out,
                          n_heads, n_kv_heads, head_dim, max_seq, scale, workspace, workspace_bytes, stream);
}

int pf_silu_mul(const float* g, const float* u, float* out, long long n, void* stream) {
  if (!g || !u || !out || n < 0) return PF_ERR_INVALID_ARGUMENT;
  if (!al4(g) || !al4(u) || !al4(out)) return PF_ERR_ALIGNMENT;
  if (n == 0) return PF_OK;
  const long long blocks = (n + 255) / 256 < 4096 ? (n + 255) / 256 : 4096;
  return status_of(launch_pdl(silu_mul_kernel, dim3((unsigned)blocks), 256, static_cast<cudaStream_t>(stream), g, u, out,
                              n));
}
