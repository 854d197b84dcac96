// Device-side decoders shared by the CUDA-core GEMV and the dequant kernels.
#pragma once

#include "common.cuh"

namespace pfb {

// Root k of generate_e8_roots (polarflash_quant/lattice/e8_lattice.py:21-50):
// k < 112: pair p = k/4 of combinations(range(8), 2), signs (-,-),(-,+),(+,-),(+,+);
// k >= 112: the (k-112)-th even-popcount mask m = 2u + parity(u), bit set = -1/2.
__device__ __forceinline__ void e8_root(int k, float (&r)[8]) {
#pragma unroll
  for (int q = 0; q < 8; ++q) r[q] = 0.f;
  if (k < 112) {
    int p = k >> 2;
    int i = 0, rem = p;
    while (rem >= 7 - i) {
      rem -= 7 - i;
      ++i;
    }
    int j = i + 1 + rem;
    r[i] = (k & 2) ? 1.f : -1.f;
    r[j] = (k & 1) ? 1.f : -1.f;
  } else {
    int u = k - 112;
    int m = (u << 1) | (__popc(u) & 1);
#pragma unroll
    for (int q = 0; q < 8; ++q) r[q] = ((m >> q) & 1) ? -0.5f : 0.5f;
  }
}

// Reads `nbits` (<= 32) bits at bit offset `bit` of an MSB-first byte stream
// of `nbytes` bytes (bytes past the end read as 0).
__device__ __forceinline__ uint32_t read_bits_msb(const uint8_t* __restrict__ buf, long long nbytes,
                                                  long long bit, int nbits) {
  long long b0 = bit >> 3;
  unsigned long long v = 0;
#pragma unroll
  for (int q = 0; q < 5; ++q) {
    long long bi = b0 + q;
    unsigned long long byte = bi < nbytes ? (unsigned long long)__ldg(buf + bi) : 0ull;
    v = (v << 8) | byte;
  }
  int sh = 40 - (int)(bit & 7) - nbits;
  return (uint32_t)((v >> sh) & ((nbits == 32) ? 0xffffffffull : ((1ull << nbits) - 1ull)));
}

// Polar angle tables in shared memory: for angle column j (0..d-2, level 0
// first), entry c holds (cos th, sin th) of the reference's uniform
// reconstruction (polar_quant.py:540-559): level 0 th = ((c+.5)/2^b) 2pi - pi,
// upper levels th = ((c+.5)/2^b) pi/2; or, for a weight encoded with learned
// angle codebooks (polar_quant.py:552-554), th = angles[64 j + c] from the
// weight's fp32 angle table.
constexpr int kPolarTabPerCol = 64;  // angle codes up to 6 bits

__device__ __forceinline__ void polar_fill_tables(float2* tab, int d, const int* alloc,
                                                  const float* angles = nullptr) {
  const float kPi = 3.14159274101257324f, k2Pi = 6.28318548202514648f, kHalfPi = 1.57079637050628662f;
  for (int e = threadIdx.x; e < (d - 1) * kPolarTabPerCol; e += blockDim.x) {
    int j = e / kPolarTabPerCol, c = e % kPolarTabPerCol;
    int bits = alloc[1 + j];
    if (c >= (1 << bits)) continue;
    float L = (float)(1 << bits);
    float t = ((float)c + 0.5f) / L;
    float th = (j < d / 2) ? t * k2Pi - kPi : t * kHalfPi;
    if (angles) th = angles[e];
    tab[e] = make_float2(cosf(th), sinf(th));
  }
}

// inverse_recursive (polar_quant.py:252-272) of one block word.
__device__ __forceinline__ void polar_block(uint32_t word, int d, const int* alloc, float r_scale,
                                            const float2* tab, int zero_rule, float* out) {
  int codes[16];
  int shift = 0;
  for (int i = d - 1; i >= 0; --i) {
    codes[i] = (int)((word >> shift) & ((1u << alloc[i]) - 1u));
    shift += alloc[i];
  }
  float cur[16], nxt[16];
  cur[0] = (float)codes[0] * r_scale;
  int width = 1, base = d - 1;
  while (width < d) {
    base -= width;
    for (int j = 0; j < width; ++j) {
      float2 cs = tab[(base + j) * kPolarTabPerCol + codes[1 + base + j]];
      if (zero_rule && cur[j] <= 1e-12f) cs = make_float2(1.f, 0.f);
      nxt[2 * j] = cur[j] * cs.x;
      nxt[2 * j + 1] = cur[j] * cs.y;
    }
    width *= 2;
    for (int j = 0; j < width; ++j) cur[j] = nxt[j];
  }
  for (int i = 0; i < d; ++i) out[i] = cur[i];
}

}  // namespace pfb
