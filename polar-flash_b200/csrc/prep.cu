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

}  // namespace

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
  note_launch();
  return cudaGetLastError();
}

}  // namespace pfb
