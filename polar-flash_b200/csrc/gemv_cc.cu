// CUDA-core GEMV for the E8 residual-VQ and polar formats.
//
// One warp owns one weight row; lanes walk the row's 8-vectors (E8) or polar
// blocks, decode them in registers (E8 roots rebuilt from the index rule,
// polar angles from shared-memory cos/sin tables), and dot them with the
// rotated activations x' (fp32, from prep.cu).  A warp reduction finishes the
// row, so y is written once, with the bias, and needs no atomics.
#include "decode.cuh"
#include "gemv.cuh"

namespace pfb {

namespace {

constexpr int kWarpsCC = 8;

__global__ void __launch_bounds__(kWarpsCC * 32) gemv_e8_kernel(GemvCCArgs a) {
  __shared__ float roots[240][8];
  for (int k = threadIdx.x; k < 240; k += blockDim.x) {
    float r[8];
    e8_root(k, r);
#pragma unroll
    for (int q = 0; q < 8; ++q) roots[k][q] = r[q];
  }
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kWarpsCC + warp;
  if (row >= a.M) return;
  const int KO = a.K / 8, G = a.K / kGroup;
  const uint16_t* __restrict__ idx = static_cast<const uint16_t*>(a.codes) + (size_t)row * KO;
  const __half2* __restrict__ sc = static_cast<const __half2*>(a.scales) + (size_t)row * G;
  float acc[kMaxGemvTokens];
#pragma unroll
  for (int t = 0; t < kMaxGemvTokens; ++t) acc[t] = 0.f;
  for (int o = lane; o < KO; o += 32) {
    uint32_t pr = __ldg(idx + o);
    int i1 = pr & 0xff, i2 = pr >> 8;
    float2 s = __half22float2(sc[o / 16]);
    float w[8];
#pragma unroll
    for (int q = 0; q < 8; ++q) w[q] = __fadd_rn(__fmul_rn(s.x, roots[i1][q]), __fmul_rn(s.y, roots[i2][q]));
#pragma unroll
    for (int t = 0; t < kMaxGemvTokens; ++t) {
      if (t < a.N) {
        const float4* xv = reinterpret_cast<const float4*>(a.xplain + (size_t)t * a.Kp + 8 * o);
        float4 x0 = __ldg(xv), x1 = __ldg(xv + 1);
        acc[t] += w[0] * x0.x + w[1] * x0.y + w[2] * x0.z + w[3] * x0.w + w[4] * x1.x + w[5] * x1.y +
                  w[6] * x1.z + w[7] * x1.w;
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kMaxGemvTokens; ++t) {
    if (t < a.N) {
      float v = acc[t];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0) a.y[(size_t)t * a.M + row] = v + (a.bias ? a.bias[row] : 0.f);
    }
  }
}

__global__ void __launch_bounds__(kWarpsCC * 32) gemv_polar_kernel(GemvCCArgs a) {
  __shared__ float2 tab[15 * kPolarTabPerCol];
  __shared__ int alloc_s[17];
  if (threadIdx.x < 17) alloc_s[threadIdx.x] = a.alloc[threadIdx.x];
  polar_fill_tables(tab, a.d, a.alloc, a.angles);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int row = blockIdx.x * kWarpsCC + warp;
  if (row >= a.M) return;
  const int nblk = a.K / a.d;
  const uint8_t* __restrict__ rowp = static_cast<const uint8_t*>(a.codes) + (size_t)row * a.row_bytes;
  const long long avail = (long long)(a.M - row) * a.row_bytes;
  float acc[kMaxGemvTokens];
#pragma unroll
  for (int t = 0; t < kMaxGemvTokens; ++t) acc[t] = 0.f;
  for (int b = lane; b < nblk; b += 32) {
    uint32_t word = read_bits_msb(rowp, avail, (long long)b * a.tb, a.tb);
    float w[16];
    polar_block(word, a.d, alloc_s, a.r_scale, tab, a.zero_rule, w);
#pragma unroll
    for (int t = 0; t < kMaxGemvTokens; ++t) {
      if (t < a.N) {
        const float* xv = a.xplain + (size_t)t * a.Kp + (size_t)b * a.d;
        float s = 0.f;
        for (int q = 0; q < a.d; ++q) s += w[q] * __ldg(xv + q);
        acc[t] += s;
      }
    }
  }
#pragma unroll
  for (int t = 0; t < kMaxGemvTokens; ++t) {
    if (t < a.N) {
      float v = acc[t];
#pragma unroll
      for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane == 0) a.y[(size_t)t * a.M + row] = v + (a.bias ? a.bias[row] : 0.f);
    }
  }
}

}  // namespace

cudaError_t launch_gemv_cc(const GemvCCArgs& a, cudaStream_t s) {
  dim3 grid((a.M + kWarpsCC - 1) / kWarpsCC);
  if (a.fmt == PF_FMT_E8_RVQ2_G128)
    gemv_e8_kernel<<<grid, kWarpsCC * 32, 0, s>>>(a);
  else
    gemv_polar_kernel<<<grid, kWarpsCC * 32, 0, s>>>(a);
  note_launch();
  return cudaGetLastError();
}

}  // namespace pfb
