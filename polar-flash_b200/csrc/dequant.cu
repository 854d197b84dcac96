// Weight materialisation (pf_dequant), code unpacking (pf_unpack_codes) and the
// standalone block RWHT (pf_rwht).  These serve parity checks and the
// reference's dequantize API; the GEMV/GEMM never materialise weights.
#include "decode.cuh"
#include "gemv.cuh"

namespace pfb {

namespace {

// Code of column k in row `row` of an INT format.
__device__ __forceinline__ uint32_t int_code(const DequantArgs& a, int row, int k) {
  const uint32_t* rw = static_cast<const uint32_t*>(a.codes) + (size_t)row * a.row_words;
  switch (a.fmt) {
    case PF_FMT_INT4_G128:
    case PF_FMT_INT4: return (__ldg(rw + (k >> 3)) >> (4 * (k & 7))) & 0xfu;
    case PF_FMT_INT2_G128:
    case PF_FMT_INT2: return (__ldg(rw + (k >> 4)) >> (2 * (k & 15))) & 0x3u;
    case PF_FMT_INT3_G128: {
      int g = k >> 7, c = k & 127;
      return (__ldg(rw + g * 13 + c / 10) >> (3 * (c % 10))) & 0x7u;
    }
    default: {  // INT3 reference stream: code k at bit 3k of the row
      int bit = 3 * k, w = bit >> 5, s = bit & 31;
      uint32_t lo = __ldg(rw + w);
      uint32_t hi = (s > 29) ? __ldg(rw + w + 1) : 0u;
      return (uint32_t)((((unsigned long long)hi << 32) | lo) >> s) & 0x7u;
    }
  }
}

__global__ void dequant_int_kernel(DequantArgs a) {
  const int G = a.K / kGroup;
  const int bits = int_format_bits(a.fmt);
  const int off = is_group_int_format(a.fmt) ? 0 : (bits == 4 ? 8 : bits == 3 ? 4 : 2);
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < (long long)a.M * a.K;
       e += (long long)gridDim.x * blockDim.x) {
    int row = (int)(e / a.K), k = (int)(e % a.K);
    uint32_t q = int_code(a, row, k);
    if (a.codes_out) {
      a.codes_out[e] = (uint8_t)q;
      continue;
    }
    float w;
    if (is_group_int_format(a.fmt)) {
      size_t si = (size_t)row * G + (k >> 7);
      float s = __half2float(static_cast<const __half*>(a.scales)[si]);
      float m = __half2float(a.mins[si]);
      w = __fadd_rn(__fmul_rn((float)q, s), m);
    } else {
      float s = a.scales ? static_cast<const float*>(a.scales)[row] : a.tensor_scale;
      w = __fmul_rn((float)((int)q - off), s);
    }
    a.W[e] = w;
  }
}

__global__ void dequant_e8_kernel(DequantArgs a) {
  const int KO = a.K / 8, G = a.K / kGroup;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < (long long)a.M * KO;
       e += (long long)gridDim.x * blockDim.x) {
    int row = (int)(e / KO), o = (int)(e % KO);
    uint16_t pr = static_cast<const uint16_t*>(a.codes)[e];
    if (a.codes_out) {
      a.codes_out[2 * e] = (uint8_t)(pr & 0xff);
      a.codes_out[2 * e + 1] = (uint8_t)(pr >> 8);
      continue;
    }
    float2 s = __half22float2(static_cast<const __half2*>(a.scales)[(size_t)row * G + o / 16]);
    float r1[8], r2[8];
    e8_root(pr & 0xff, r1);
    e8_root(pr >> 8, r2);
#pragma unroll
    for (int q = 0; q < 8; ++q)
      a.W[(size_t)row * a.K + 8 * o + q] = __fadd_rn(__fmul_rn(s.x, r1[q]), __fmul_rn(s.y, r2[q]));
  }
}

__global__ void dequant_polar_kernel(DequantArgs a) {
  __shared__ float2 tab[15 * kPolarTabPerCol];
  __shared__ int alloc_s[17];
  if (threadIdx.x < 17) alloc_s[threadIdx.x] = a.alloc[threadIdx.x];
  polar_fill_tables(tab, a.d, a.alloc, a.angles);
  __syncthreads();
  const int nblk = a.K / a.d;
  const long long total = (long long)a.M * a.row_bytes;
  for (long long e = blockIdx.x * (long long)blockDim.x + threadIdx.x; e < (long long)a.M * nblk;
       e += (long long)gridDim.x * blockDim.x) {
    int row = (int)(e / nblk), b = (int)(e % nblk);
    const uint8_t* base = static_cast<const uint8_t*>(a.codes);
    uint32_t word = read_bits_msb(base, total, (long long)row * a.row_bytes * 8 + (long long)b * a.tb, a.tb);
    float w[16];
    polar_block(word, a.d, alloc_s, a.r_scale, tab, a.zero_rule, w);
    for (int q = 0; q < a.d; ++q) a.W[(size_t)row * a.K + (size_t)b * a.d + q] = w[q];
  }
}

__device__ __forceinline__ void plan_block(const HadPlan& p, int k, int& off, int& size) {
  if (k < p.nfull * p.block) {
    off = (k / p.block) * p.block;
    size = p.block;
    return;
  }
  for (int i = 0; i < p.ncasc; ++i)
    if (k >= p.casc_off[i] && k < p.casc_off[i] + p.casc_size[i]) {
      off = p.casc_off[i];
      size = p.casc_size[i];
      return;
    }
  off = k;
  size = 1;
}

// One CTA per (row, chunk of CH columns); CH is a multiple of the block size.
__global__ void rwht_rows_kernel(const float* in, float* out, int K, HadPlan plan, const int8_t* signs,
                                 int inverse, int CH) {
  extern __shared__ float sm[];
  const int row = blockIdx.y;
  const int k0 = blockIdx.x * CH;
  const int n = min(CH, K - k0);
  const float* src = in + (size_t)row * K + k0;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    int k = k0 + j;
    float v = src[j];
    if (!inverse && k < plan.rot_end) v = v * (float)signs[k];
    sm[j] = v;
  }
  for (int h = 1; h < plan.block; h *= 2) {
    __syncthreads();
    for (int j = threadIdx.x; j < n; j += blockDim.x) {
      int k = k0 + j;
      if (k >= plan.rot_end) continue;
      int off, size;
      plan_block(plan, k, off, size);
      if (h < size && ((k - off) & h) == 0) {
        float u = sm[j], w = sm[j + h];
        sm[j] = u + w;
        sm[j + h] = u - w;
      }
    }
  }
  __syncthreads();
  float* dst = out + (size_t)row * K + k0;
  for (int j = threadIdx.x; j < n; j += blockDim.x) {
    int k = k0 + j;
    float v = sm[j];
    if (k < plan.rot_end) {
      int off, size;
      plan_block(plan, k, off, size);
      v = v / sqrtf((float)size);
      if (inverse) v = v * (float)signs[k];
    }
    dst[j] = v;
  }
}

}  // namespace

cudaError_t launch_dequant(const DequantArgs& a, cudaStream_t s) {
  long long work = (long long)a.M * a.K;
  int blocks = (int)((work + 255) / 256);
  if (blocks > 148 * 32) blocks = 148 * 32;
  if (blocks < 1) blocks = 1;
  if (is_int_format(a.fmt))
    dequant_int_kernel<<<blocks, 256, 0, s>>>(a);
  else if (a.fmt == PF_FMT_E8_RVQ2_G128)
    dequant_e8_kernel<<<blocks, 256, 0, s>>>(a);
  else
    dequant_polar_kernel<<<blocks, 256, 0, s>>>(a);
  note_launch();
  return cudaGetLastError();
}

cudaError_t launch_unpack(const DequantArgs& a, cudaStream_t s) { return launch_dequant(a, s); }

cudaError_t launch_rwht_rows(const float* in, float* out, int rows, int K, const HadPlan& plan,
                             const int8_t* signs, int inverse, cudaStream_t s) {
  int CH = prep_chunk_cols(plan);
  size_t smem = (size_t)CH * sizeof(float);
  if (smem > 48 * 1024) {
    cudaError_t e = cudaFuncSetAttribute(rwht_rows_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
  }
  dim3 grid((K + CH - 1) / CH, rows);
  rwht_rows_kernel<<<grid, 256, smem, s>>>(in, out, K, plan, signs, inverse, CH);
  note_launch();
  return cudaGetLastError();
}

}  // namespace pfb
