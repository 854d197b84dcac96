// x-preparation kernel: x' = forward block RWHT of x, written in the layout
// the GEMV kernels read.
//
// Fusion identity: the reference decodes W_hat = inverse_RWHT(Z) row by row
// (polarflash_quant/unified_quantizer.py:318-322, hadamard.py:146-169), with
// inverse(z) = D H z / sqrt(b).  H is symmetric and D diagonal, so
//   y = W_hat x = Z (H D x / sqrt(b)) = Z forward_RWHT(x)   (hadamard.py:119-144),
// i.e. one transform of the N x K activations replaces M x K weight work.
//
// Mode 0 writes x' as tensor-core B fragments (m16n8k16, fp16) in the
// permuted column order of frag_cols(), split into hi + lo fp16 parts so the
// product keeps ~fp32 accuracy: token t uses n-slots 2t (hi) and 2t+1 (lo).
// It also writes the per-group sums of every slot (sx), which the GEMV
// needs for the codes' zero offset.  Mode 1 writes plain fp32 x' [N][Kp].
#include "common.cuh"
#include "gemv.cuh"

namespace pfb {

namespace {

constexpr int kPrepThreads = 256;

__device__ __forceinline__ void block_of(const HadPlan& p, int k, int& off, int& size) {
  if (k < p.nfull * p.block) {
    off = (k / p.block) * p.block;
    size = p.block;
    return;
  }
  for (int i = 0; i < p.ncasc; ++i) {
    if (k >= p.casc_off[i] && k < p.casc_off[i] + p.casc_size[i]) {
      off = p.casc_off[i];
      size = p.casc_size[i];
      return;
    }
  }
  off = k;
  size = 1;
}

__global__ void __launch_bounds__(kPrepThreads) prep_kernel(PrepArgs a, int CH) {
  extern __shared__ float sm[];
  const int t = blockIdx.y;  // token slot
  const int k0 = blockIdx.x * CH;
  const int ncols = min(CH, a.Kp - k0);  // whole groups
  const bool live = t < a.N;
  const bool rotated = a.plan.block > 0;

  for (int j = threadIdx.x; j < ncols; j += blockDim.x) {
    int k = k0 + j;
    float v = 0.f;
    if (live && k < a.K) {
      v = load_x(a.x, a.x_dtype, (size_t)t * a.K + k);
      if (rotated && k < a.plan.rot_end) v = v * (float)a.signs[k];
    }
    sm[j] = v;
  }
  if (rotated) {
    // every block (full or cascade) has at most plan.block columns
    for (int h = 1; h < a.plan.block; h *= 2) {
      __syncthreads();
      for (int j = threadIdx.x; j < ncols; j += blockDim.x) {
        int k = k0 + j;
        if (k >= a.plan.rot_end) continue;
        int off, size;
        block_of(a.plan, k, off, size);
        if (h < size && ((k - off) & h) == 0) {
          float u = sm[j], w = sm[j + h];
          sm[j] = u + w;
          sm[j + h] = u - w;
        }
      }
    }
    __syncthreads();
    for (int j = threadIdx.x; j < ncols; j += blockDim.x) {
      int k = k0 + j;
      if (k >= a.plan.rot_end) continue;
      int off, size;
      block_of(a.plan, k, off, size);
      sm[j] = sm[j] / sqrtf((float)size);
    }
  }
  __syncthreads();

  const int g0 = k0 / kGroup;
  const int ngroups = ncols / kGroup;
  if (a.mode == 0) {
    // fragments: slot n = 2t (hi) and 2t+1 (lo); tile n/8, column-in-tile n%8
    const int tile = (2 * t) >> 3;
    const int nl_hi = (2 * t) & 7;
    const int Gp = a.Kp / kGroup;
    for (int it = threadIdx.x; it < ngroups * 32; it += blockDim.x) {
      int gi = it >> 5, j = (it >> 2) & 7, c = it & 3;
      const float* s = sm + gi * kGroup;
      int lo0, hi0, lo1, hi1;
      frag_cols(a.fmt, c, 2 * j, lo0, hi0);
      frag_cols(a.fmt, c, 2 * j + 1, lo1, hi1);
      float v[4] = {s[lo0], s[hi0], s[lo1], s[hi1]};
      __half h[4], l[4];
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        h[q] = __float2half_rn(v[q]);
        l[q] = __float2half_rn(v[q] - __half2float(h[q]));
      }
      __half2 bh0 = __halves2half2(h[0], h[1]), bh1 = __halves2half2(h[2], h[3]);
      __half2 bl0 = __halves2half2(l[0], l[1]), bl1 = __halves2half2(l[2], l[3]);
      size_t base = ((size_t)(tile * Gp + g0 + gi) * 8 + j) * 32;
      uint2 ph, pl;
      ph.x = *reinterpret_cast<uint32_t*>(&bh0);
      ph.y = *reinterpret_cast<uint32_t*>(&bh1);
      pl.x = *reinterpret_cast<uint32_t*>(&bl0);
      pl.y = *reinterpret_cast<uint32_t*>(&bl1);
      a.xfrag[base + 4 * nl_hi + c] = ph;
      a.xfrag[base + 4 * (nl_hi + 1) + c] = pl;
    }
    // group sums of the hi and lo parts
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int gi = warp; gi < ngroups; gi += kPrepThreads / 32) {
      float sh = 0.f, sl = 0.f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        float v = sm[gi * kGroup + lane + 32 * q];
        __half hv = __float2half_rn(v);
        __half lv = __float2half_rn(v - __half2float(hv));
        sh += __half2float(hv);
        sl += __half2float(lv);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        sh += __shfl_xor_sync(0xffffffffu, sh, o);
        sl += __shfl_xor_sync(0xffffffffu, sl, o);
      }
      if (lane == 0) {
        a.sx[(size_t)(g0 + gi) * (8 * a.NT) + 2 * t] = sh;
        a.sx[(size_t)(g0 + gi) * (8 * a.NT) + 2 * t + 1] = sl;
      }
    }
  } else if (live) {
    for (int j = threadIdx.x; j < ncols; j += blockDim.x) a.xplain[(size_t)t * a.Kp + k0 + j] = sm[j];
  }

  if (a.init_y && live) {
    int per = (a.M + gridDim.x - 1) / gridDim.x;
    int m0 = blockIdx.x * per, m1 = min(a.M, m0 + per);
    for (int m = m0 + threadIdx.x; m < m1; m += blockDim.x)
      a.y[(size_t)t * a.M + m] = a.bias ? a.bias[m] : 0.f;
  }
}

// x-prep for the TMA GEMV: one CTA per chunk of max(128, block) columns, all
// tokens in turn.  Per 128-column group and token it writes the B fragments
// of x' scaled by the group's power-of-two normaliser 2^-E (so |x'| <= 1) and
// by 2^(beta - p) for the mantissa position p at which the GEMV decodes each
// column's code, plus {Sx, 2^E, SB}.  Launched as a programmatic dependent:
// it waits for the preceding grid before reading x or writing the workspace.
constexpr int kPrep2Threads = 128;

__global__ void __launch_bounds__(kPrep2Threads) prep2_kernel(Prep2Args a, int CH) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  asm volatile("griddepcontrol.launch_dependents;");
  extern __shared__ float sm2[];
  const int k0 = blockIdx.x * CH;
  const int ncols = min(CH, a.G * kGroup - k0);
  const int g0 = k0 / kGroup, ngroups = ncols / kGroup;
  const bool rotated = a.plan.block > 0;
  const int Lp = tma_lanes(a.N, a.NT);
  const size_t rec_bytes = tma_record_bytes(a.N, a.NT);
  const int beta = a.subnormal ? 14 : 10;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  for (int t = 0; t < a.N; ++t) {
    for (int j = threadIdx.x; j < ncols; j += blockDim.x) {
      int k = k0 + j;
      float v = 0.f;
      if (k < a.K) {
        v = load_x(a.x, a.x_dtype, (size_t)t * a.K + k);
        if (rotated && k < a.plan.rot_end) v = v * (float)a.signs[k];
      }
      sm2[j] = v;
    }
    if (rotated) {
      for (int h = 1; h < a.plan.block; h *= 2) {
        __syncthreads();
        for (int j = threadIdx.x; j < ncols; j += blockDim.x) {
          int k = k0 + j;
          if (k >= a.plan.rot_end) continue;
          int off, size;
          block_of(a.plan, k, off, size);
          if (h < size && ((k - off) & h) == 0) {
            float u = sm2[j], w = sm2[j + h];
            sm2[j] = u + w;
            sm2[j + h] = u - w;
          }
        }
      }
      __syncthreads();
      for (int j = threadIdx.x; j < ncols; j += blockDim.x) {
        int k = k0 + j;
        if (k >= a.plan.rot_end) continue;
        int off, size;
        block_of(a.plan, k, off, size);
        sm2[j] = sm2[j] / sqrtf((float)size);
      }
    }
    __syncthreads();
    const int tile = (2 * t) >> 3, nl = (2 * t) & 7;
    for (int gi = warp; gi < ngroups; gi += kPrep2Threads / 32) {
      const float* xs = sm2 + gi * kGroup;
      float amax = 0.f, sx = 0.f;
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        float v = xs[4 * lane + e];
        amax = fmaxf(amax, fabsf(v));
        sx += v;
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) {
        amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
        sx += __shfl_xor_sync(0xffffffffu, sx, o);
      }
      int E = 0;
      if (amax > 0.f) frexpf(amax, &E);  // amax <= 2^E
      const int j8 = lane >> 2, c = lane & 3;
      int lo0, hi0, p0, lo1, hi1, p1;
      frag_cols2(a.fmt, c, 2 * j8, lo0, hi0, p0);
      frag_cols2(a.fmt, c, 2 * j8 + 1, lo1, hi1, p1);
      const float s0 = ldexpf(1.f, beta - p0 - E), s1 = ldexpf(1.f, beta - p1 - E);
      float v[4] = {xs[lo0] * s0, xs[hi0] * s0, xs[lo1] * s1, xs[hi1] * s1};
      __half h[4], l[4];
      float sb = 0.f;
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        h[q] = __float2half_rn(v[q]);
        l[q] = __float2half_rn(v[q] - __half2float(h[q]));
        sb += __half2float(h[q]) + __half2float(l[q]);
      }
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) sb += __shfl_xor_sync(0xffffffffu, sb, o);
      __half2 bh0 = __halves2half2(h[0], h[1]), bh1 = __halves2half2(h[2], h[3]);
      __half2 bl0 = __halves2half2(l[0], l[1]), bl1 = __halves2half2(l[2], l[3]);
      unsigned char* rec = a.rec + (size_t)(g0 + gi) * rec_bytes;
      uint2* fr = reinterpret_cast<uint2*>(rec) + (size_t)(tile * 8 + j8) * Lp;
      fr[4 * nl + c] = make_uint2(*reinterpret_cast<uint32_t*>(&bh0), *reinterpret_cast<uint32_t*>(&bh1));
      fr[4 * (nl + 1) + c] = make_uint2(*reinterpret_cast<uint32_t*>(&bl0), *reinterpret_cast<uint32_t*>(&bl1));
      if (lane == 0) {
        float4* gs = reinterpret_cast<float4*>(rec + (size_t)a.NT * 8 * Lp * 8);
        gs[t] = make_float4(sx, ldexpf(1.f, E), sb, 0.f);
      }
    }
    __syncthreads();
  }
}

}  // namespace

cudaError_t launch_prep2(const Prep2Args& a, cudaStream_t stream) {
  int CH = a.plan.block > kGroup ? a.plan.block : kGroup;
  size_t smem = (size_t)CH * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(prep2_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((a.G * kGroup + CH - 1) / CH);
  cfg.blockDim = dim3(kPrep2Threads);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, prep2_kernel, a, CH);
}

int prep_chunk_cols(const HadPlan& plan) {
  int ch = 1024;
  if (plan.block > ch) ch = plan.block;
  return ch;
}

cudaError_t launch_prep(const PrepArgs& a, cudaStream_t stream) {
  int CH = prep_chunk_cols(a.plan);
  dim3 grid((a.Kp + CH - 1) / CH, a.slots);
  size_t smem = (size_t)CH * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(prep_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  prep_kernel<<<grid, kPrepThreads, smem, stream>>>(a, CH);
  return cudaGetLastError();
}

}  // namespace pfb
