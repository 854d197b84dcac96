/*
 * pf_oracle.c -- CPU restatement of POLAR-FLASH's compressed-linear path.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the parity checker for the CUDA
 * library: only tests/, __graft_entry__.smoke() and bench.py's CPU-baseline
 * leg may load it.  The product path never calls into it.
 *
 * Each function restates one step of the reference algorithm (citations are
 * paths inside the ELANGKATHIR11/POLAR-FLASH project) or, for the formats the
 * reference lacks (group-128 asymmetric INT, INT3 10-per-word, E8 root
 * indices), defines the extension in the reference's own conventions.
 * Parity is pinned by the .npz fixtures in tests/golden, produced by importing the reference
 * Python package (tests/golden/make_golden.py).
 *
 * Floating point: compiled with -ffp-contract=off and without -ffast-math so
 * every fp32 operation rounds exactly once, in the order written.  Integer
 * and index outputs are bit-exact by construction.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>

#ifdef _OPENMP
#include <omp.h>
#endif

#define PFO_API __attribute__((visibility("default")))

/* ------------------------------------------------------------------ */
/* IEEE half <-> float, round to nearest even (numpy / CUDA __float2half_rn) */
/* ------------------------------------------------------------------ */
PFO_API uint16_t pfo_f32_to_f16(float f) {
  uint32_t x;
  memcpy(&x, &f, 4);
  uint32_t sign = (x >> 16) & 0x8000u;
  uint32_t absx = x & 0x7fffffffu;
  if (absx >= 0x7f800000u) { /* inf / nan */
    return (uint16_t)(sign | 0x7c00u | (absx > 0x7f800000u ? 0x200u : 0u));
  }
  if (absx >= 0x477ff000u) { /* rounds to >= 65520 -> inf */
    return (uint16_t)(sign | 0x7c00u);
  }
  if (absx < 0x38800000u) { /* result is subnormal or zero */
    if (absx < 0x33000000u) return (uint16_t)sign; /* < 2^-25 -> 0 */
    uint32_t e = absx >> 23;
    uint32_t m = (absx & 0x7fffffu) | 0x800000u;
    /* value = m * 2^(e-150); in half subnormal units of 2^-24: m * 2^(e-126) */
    uint32_t shift = 126u - e;
    uint32_t q = m >> shift;
    uint32_t rem = m & ((1u << shift) - 1u);
    uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (q & 1u))) q++;
    return (uint16_t)(sign | q);
  }
  uint32_t e = (absx >> 23) - 112u; /* rebias 127 -> 15 */
  uint32_t m = absx & 0x7fffffu;
  uint32_t q = (e << 10) | (m >> 13);
  uint32_t rem = m & 0x1fffu;
  if (rem > 0x1000u || (rem == 0x1000u && (q & 1u))) q++;
  return (uint16_t)(sign | q);
}

PFO_API float pfo_f16_to_f32(uint16_t h) {
  uint32_t sign = ((uint32_t)h & 0x8000u) << 16;
  uint32_t e = (h >> 10) & 0x1fu;
  uint32_t m = h & 0x3ffu;
  uint32_t x;
  if (e == 0) {
    if (m == 0) {
      x = sign;
    } else { /* subnormal: m * 2^-24 */
      float v = (float)m * 5.9604644775390625e-08f;
      memcpy(&x, &v, 4);
      x |= sign;
    }
  } else if (e == 31) {
    x = sign | 0x7f800000u | (m << 13);
  } else {
    x = sign | ((e + 112u) << 23) | (m << 13);
  }
  float f;
  memcpy(&f, &x, 4);
  return f;
}

/* ------------------------------------------------------------------ */
/* Reference bit packing (polarflash_quant/bitpacking.py)               */
/* ------------------------------------------------------------------ */

/* unpack_int4 (bitpacking.py:34-46): low nibble = element 2i, value - 8. */
PFO_API void pfo_unpack_int4(const uint8_t* packed, int64_t n, int8_t* out) {
  for (int64_t i = 0; i < n; ++i) {
    uint8_t b = packed[i >> 1];
    int v = (i & 1) ? (b >> 4) : (b & 0xf);
    out[i] = (int8_t)(v - 8);
  }
}

/* pack_int4 (bitpacking.py:16-31): (v + 8) & 0xf, even element low; an odd
 * length is padded with the value 0 (code 8), as the reference pads. */
PFO_API void pfo_pack_int4(const int8_t* v, int64_t n, uint8_t* packed) {
  int64_t nb = (n + 1) / 2;
  memset(packed, 0, (size_t)nb);
  for (int64_t i = 0; i < 2 * nb; ++i) {
    int val = i < n ? v[i] : 0;
    uint8_t u = (uint8_t)((val + 8) & 0xf);
    packed[i >> 1] |= (uint8_t)((i & 1) ? (u << 4) : u);
  }
}

/* unpack_int2 (bitpacking.py:68-85): 4 codes per byte LSB first, [0,3]. */
PFO_API void pfo_unpack_int2(const uint8_t* packed, int64_t n, uint8_t* out) {
  for (int64_t i = 0; i < n; ++i) out[i] = (uint8_t)((packed[i >> 2] >> (2 * (i & 3))) & 3);
}

/* pack_int2 (bitpacking.py:49-65). */
PFO_API void pfo_pack_int2(const uint8_t* v, int64_t n, uint8_t* packed) {
  int64_t nb = (n + 3) / 4;
  memset(packed, 0, (size_t)nb);
  for (int64_t i = 0; i < n; ++i) packed[i >> 2] |= (uint8_t)((v[i] & 3) << (2 * (i & 3)));
}

/* unpack_int3 (bitpacking.py:126-156): 8 codes per 3 bytes; as a 24-bit
 * little-endian chunk, code i sits at bits 3i (b0 | b1<<8 | b2<<16). */
PFO_API void pfo_unpack_int3(const uint8_t* packed, int64_t n, uint8_t* out) {
  for (int64_t i = 0; i < n; ++i) {
    int64_t g = i >> 3;
    uint32_t chunk = (uint32_t)packed[3 * g] | ((uint32_t)packed[3 * g + 1] << 8) |
                     ((uint32_t)packed[3 * g + 2] << 16);
    out[i] = (uint8_t)((chunk >> (3 * (i & 7))) & 7);
  }
}

/* pack_int3 (bitpacking.py:88-123). */
PFO_API void pfo_pack_int3(const uint8_t* v, int64_t n, uint8_t* packed) {
  int64_t ng = (n + 7) / 8;
  for (int64_t g = 0; g < ng; ++g) {
    uint32_t chunk = 0;
    for (int j = 0; j < 8; ++j) {
      int64_t i = 8 * g + j;
      uint32_t c = i < n ? (uint32_t)(v[i] & 7) : 0u;
      chunk |= c << (3 * j);
    }
    packed[3 * g] = (uint8_t)(chunk & 0xff);
    packed[3 * g + 1] = (uint8_t)((chunk >> 8) & 0xff);
    packed[3 * g + 2] = (uint8_t)((chunk >> 16) & 0xff);
  }
}

/* ------------------------------------------------------------------ */
/* Group-128 word layouts (extension; codes in the reference bit order)  */
/* ------------------------------------------------------------------ */
/* words per 128-column group: INT4 16 (8/u32), INT2 8 (16/u32),
 * INT3 13 (10/u32, bits 30-31 zero, slots 8..9 of word 12 unused). */
PFO_API int pfo_g128_words(int bits) {
  return bits == 4 ? 16 : bits == 2 ? 8 : bits == 3 ? 13 : -1;
}

PFO_API int pfo_pack_g128(int bits, const uint8_t* q, int64_t M, int64_t K, uint32_t* words) {
  int wpg = pfo_g128_words(bits);
  if (wpg < 0 || K % 128) return -1;
  int64_t G = K / 128;
  int per = bits == 3 ? 10 : 32 / bits;
  uint32_t mask = (1u << bits) - 1u;
  memset(words, 0, (size_t)(M * G * wpg) * 4);
  for (int64_t m = 0; m < M; ++m)
    for (int64_t k = 0; k < K; ++k) {
      int64_t g = k / 128, c = k % 128;
      int64_t w = (m * G + g) * wpg + c / per;
      words[w] |= ((uint32_t)q[m * K + k] & mask) << (bits * (c % per));
    }
  return 0;
}

PFO_API int pfo_unpack_g128(int bits, const uint32_t* words, int64_t M, int64_t K, uint8_t* q) {
  int wpg = pfo_g128_words(bits);
  if (wpg < 0 || K % 128) return -1;
  int64_t G = K / 128;
  int per = bits == 3 ? 10 : 32 / bits;
  uint32_t mask = (1u << bits) - 1u;
  for (int64_t m = 0; m < M; ++m)
    for (int64_t k = 0; k < K; ++k) {
      int64_t g = k / 128, c = k % 128;
      uint32_t w = words[(m * G + g) * wpg + c / per];
      q[m * K + k] = (uint8_t)((w >> (bits * (c % per))) & mask);
    }
  return 0;
}

/* Group-128 asymmetric quantizer, following the reference's asymmetric
 * convention (polarflash_rt/kv_cache/compressed_kv.py:115-146):
 *   s = clamp((max - min) / (2^b - 1), 1e-8), q = clamp(round((w - min) / s)),
 *   w_hat = q * s + min.
 * Extension detail: s and min are stored as fp16 and q is computed against
 * the stored (fp16-rounded) values; an s that rounds to 0 becomes 2^-24. */
PFO_API int pfo_quant_g128_asym(int bits, const float* w, int64_t M, int64_t K, uint8_t* q,
                                uint16_t* s_h, uint16_t* m_h) {
  if (K % 128) return -1;
  int64_t G = K / 128;
  float L = (float)((1 << bits) - 1);
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; ++m) {
    for (int64_t g = 0; g < G; ++g) {
      const float* row = w + m * K + g * 128;
      float mn = row[0], mx = row[0];
      for (int c = 1; c < 128; ++c) {
        if (row[c] < mn) mn = row[c];
        if (row[c] > mx) mx = row[c];
      }
      float s = (mx - mn) / L;
      if (s < 1e-8f) s = 1e-8f;
      uint16_t sh = pfo_f32_to_f16(s);
      if ((sh & 0x7fffu) == 0) sh = 1;
      uint16_t mh = pfo_f32_to_f16(mn);
      float sf = pfo_f16_to_f32(sh), mf = pfo_f16_to_f32(mh);
      s_h[m * G + g] = sh;
      m_h[m * G + g] = mh;
      for (int c = 0; c < 128; ++c) {
        float t = nearbyintf((row[c] - mf) / sf);
        if (t < 0.f) t = 0.f;
        if (t > L) t = L;
        q[m * K + g * 128 + c] = (uint8_t)t;
      }
    }
  }
  return 0;
}

/* w_hat = q * s + m (two fp32 roundings, as compressed_kv.py:145). */
PFO_API void pfo_dequant_g128_asym(const uint8_t* q, const uint16_t* s_h, const uint16_t* m_h,
                                   int64_t M, int64_t K, float* w) {
  int64_t G = K / 128;
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; ++m)
    for (int64_t k = 0; k < K; ++k) {
      float s = pfo_f16_to_f32(s_h[m * G + k / 128]);
      float mn = pfo_f16_to_f32(m_h[m * G + k / 128]);
      float p = (float)q[m * K + k] * s;
      w[m * K + k] = p + mn;
    }
}

/* ------------------------------------------------------------------ */
/* Block randomized Walsh-Hadamard (polarflash_quant/transforms/hadamard.py) */
/* ------------------------------------------------------------------ */

/* BlockHadamardTransform._init_dims (hadamard.py:93-99): block = largest power of
 * two <= min(requested, K), at least 2. */
PFO_API int pfo_hadamard_block(int req, int64_t K) {
  int64_t lim = (int64_t)req < K ? (int64_t)req : K;
  int64_t bs = 1;
  while (bs * 2 <= lim) bs *= 2;
  return (int)(bs < 2 ? 2 : bs);
}

/* Block plan (hadamard.py:100-116): full blocks of `block`, then a cascade of the
 * largest powers of two of the remainder while it exceeds 1; a final single
 * column stays unrotated.  Writes (offset, size) pairs; returns the count. */
PFO_API int pfo_hadamard_plan(int block, int64_t K, int64_t* offs, int64_t* sizes, int cap) {
  int n = 0;
  int64_t nfull = K / block;
  for (int64_t b = 0; b < nfull; ++b) {
    if (n < cap) { offs[n] = b * block; sizes[n] = block; }
    n++;
  }
  int64_t off = nfull * block, rem = K - off;
  while (rem > 1) {
    int64_t p2 = 1;
    while (p2 * 2 <= rem) p2 *= 2;
    if (n < cap) { offs[n] = off; sizes[n] = p2; }
    n++;
    off += p2;
    rem -= p2;
  }
  return n;
}

/* fast_walsh_hadamard_transform (hadamard.py:18-46): butterflies at distance
 * h = 1, 2, 4, ... (u+v, u-v), then / sqrt(d). */
static void fwht_f32(float* x, int64_t d) {
  for (int64_t h = 1; h < d; h *= 2)
    for (int64_t i = 0; i < d; i += 2 * h)
      for (int64_t j = i; j < i + h; ++j) {
        float u = x[j], v = x[j + h];
        x[j] = u + v;
        x[j + h] = u - v;
      }
  float sq = (float)sqrt((double)d);
  for (int64_t i = 0; i < d; ++i) x[i] = x[i] / sq;
}

/* Forward (hadamard.py:119-144): z = H(D x)/sqrt(b) per block.
 * Inverse (hadamard.py:146-169): x = D (H z)/sqrt(b) per block.
 * `signs` holds one +-1 per column (full-block signs repeated, then the
 * remainder signs); columns outside the plan (a last single column) pass
 * through unchanged. */
PFO_API void pfo_rwht(const float* in, int64_t rows, int64_t K, int block, const float* signs,
                      int inverse, float* out) {
  int64_t offs[64], sizes[64];
  int64_t nfull = K / block;
  /* remainder cascade (full blocks are handled in the loop below) */
  int nr = 0;
  {
    int64_t off = nfull * block, rem = K - off;
    while (rem > 1 && nr < 64) {
      int64_t p2 = 1;
      while (p2 * 2 <= rem) p2 *= 2;
      offs[nr] = off;
      sizes[nr] = p2;
      nr++;
      off += p2;
      rem -= p2;
    }
  }
#pragma omp parallel
  {
    float* buf = (float*)malloc(sizeof(float) * (size_t)(block > 1 ? block : 2));
#pragma omp for schedule(static)
    for (int64_t r = 0; r < rows; ++r) {
      const float* xi = in + r * K;
      float* yo = out + r * K;
      memcpy(yo, xi, sizeof(float) * (size_t)K);
      for (int64_t b = 0; b < nfull + nr; ++b) {
        int64_t off = b < nfull ? b * block : offs[b - nfull];
        int64_t d = b < nfull ? block : sizes[b - nfull];
        if (!inverse) {
          for (int64_t j = 0; j < d; ++j) buf[j] = xi[off + j] * signs[off + j];
          fwht_f32(buf, d);
          for (int64_t j = 0; j < d; ++j) yo[off + j] = buf[j];
        } else {
          for (int64_t j = 0; j < d; ++j) buf[j] = xi[off + j];
          fwht_f32(buf, d);
          for (int64_t j = 0; j < d; ++j) yo[off + j] = buf[j] * signs[off + j];
        }
      }
    }
    free(buf);
  }
}

/* ------------------------------------------------------------------ */
/* E8 roots and the 2-stage root residual VQ (extension)                */
/* ------------------------------------------------------------------ */

/* generate_e8_roots (polarflash_quant/lattice/e8_lattice.py:21-50), index =
 * position in the list: 112 (+-1,+-1) roots over combinations(range(8), 2) with
 * s1, s2 in (-1, +1), then 128 half-integer roots for mask 0..255 with even
 * popcount, bit set meaning -0.5. */
PFO_API void pfo_e8_roots(float* roots /* 240 x 8 */) {
  int n = 0;
  for (int i = 0; i < 8; ++i)
    for (int j = i + 1; j < 8; ++j)
      for (int a = 0; a < 2; ++a)
        for (int b = 0; b < 2; ++b) {
          for (int k = 0; k < 8; ++k) roots[n * 8 + k] = 0.f;
          roots[n * 8 + i] = a ? 1.f : -1.f;
          roots[n * 8 + j] = b ? 1.f : -1.f;
          n++;
        }
  for (int mask = 0; mask < 256; ++mask) {
    if (__builtin_popcount((unsigned)mask) & 1) continue;
    for (int k = 0; k < 8; ++k) roots[n * 8 + k] = ((mask >> k) & 1) ? -0.5f : 0.5f;
    n++;
  }
}

/* <r_k, e> in a fixed fp32 order.  A (+-1,+-1) root: one add of the two
 * signed coordinates (lower coordinate first).  A half-integer root: the
 * signed coordinates t_k = +-e_k summed as the pairwise tree
 * ((t0+t1)+(t2+t3)) + ((t4+t5)+(t6+t7)), then * 0.5 (exact). */
static float e8_dot(const float* r, const float* e) {
  if (r[0] == 0.5f || r[0] == -0.5f) {
    float t[8];
    for (int k = 0; k < 8; ++k) t[k] = r[k] > 0.f ? e[k] : -e[k];
    float a = (t[0] + t[1]) + (t[2] + t[3]);
    float b = (t[4] + t[5]) + (t[6] + t[7]);
    return (a + b) * 0.5f;
  }
  float v[2];
  int n = 0;
  for (int k = 0; k < 8 && n < 2; ++k)
    if (r[k] != 0.f) v[n++] = r[k] > 0.f ? e[k] : -e[k];
  return v[0] + v[1];
}

/* sum of 16 values as the pairwise tree (0+1)+(2+3) ... level by level. */
static float tree16(const float* v) {
  float a[8], b[4], c[2];
  for (int i = 0; i < 8; ++i) a[i] = v[2 * i] + v[2 * i + 1];
  for (int i = 0; i < 4; ++i) b[i] = a[2 * i] + a[2 * i + 1];
  for (int i = 0; i < 2; ++i) c[i] = b[2 * i] + b[2 * i + 1];
  return c[0] + c[1];
}

/* Extension "E8 2-stage RVQ, group 128" encoder.  For every 8-vector e of a
 * (row, 128-column group) and stage t = 1, 2:
 *   idx = argmax_k <r_k, e>  (ties -> lowest k; equals argmin ||e/s - r_k|| for
 *         any s > 0 because every root has |r|^2 = 2, e8_lattice.py:46-49),
 *   s_t = fp16( tree16(<r_idx, e> over the group's 16 vectors) / 32 )
 *         (least squares for the fixed indices; pairwise-tree sum),
 *   e  <- e - s_t * r_idx   (s_t * r is exact, one rounding).
 * idx layout [M][K/8][2] (stage-interleaved), scales [M][K/128][2] fp16. */
PFO_API int pfo_e8_encode(const float* w, int64_t M, int64_t K, uint8_t* idx, uint16_t* scales) {
  if (K % 128) return -1;
  float roots[240 * 8];
  pfo_e8_roots(roots);
  int64_t G = K / 128;
#pragma omp parallel for schedule(dynamic, 4)
  for (int64_t m = 0; m < M; ++m) {
    float e[128];
    for (int64_t g = 0; g < G; ++g) {
      memcpy(e, w + m * K + g * 128, sizeof(e));
      for (int t = 0; t < 2; ++t) {
        int best[16];
        float bestv[16];
        for (int o = 0; o < 16; ++o) {
          int bi = 0;
          float bv = e8_dot(roots, e + 8 * o);
          for (int k = 1; k < 240; ++k) {
            float v = e8_dot(roots + 8 * k, e + 8 * o);
            if (v > bv) { bv = v; bi = k; }
          }
          best[o] = bi;
          bestv[o] = bv;
        }
        uint16_t sh = pfo_f32_to_f16(tree16(bestv) / 32.f);
        float s = pfo_f16_to_f32(sh);
        scales[(m * G + g) * 2 + t] = sh;
        for (int o = 0; o < 16; ++o) {
          idx[(m * (K / 8) + g * 16 + o) * 2 + t] = (uint8_t)best[o];
          for (int k = 0; k < 8; ++k) e[8 * o + k] = e[8 * o + k] - s * roots[best[o] * 8 + k];
        }
      }
    }
  }
  return 0;
}

/* w_hat = s1 * r[i1] + s2 * r[i2] (products exact, one rounding). */
PFO_API void pfo_e8_decode(const uint8_t* idx, const uint16_t* scales, int64_t M, int64_t K, float* w) {
  float roots[240 * 8];
  pfo_e8_roots(roots);
  int64_t G = K / 128;
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; ++m)
    for (int64_t o = 0; o < K / 8; ++o) {
      int64_t g = o / 16;
      float s1 = pfo_f16_to_f32(scales[(m * G + g) * 2]);
      float s2 = pfo_f16_to_f32(scales[(m * G + g) * 2 + 1]);
      int i1 = idx[(m * (K / 8) + o) * 2], i2 = idx[(m * (K / 8) + o) * 2 + 1];
      for (int k = 0; k < 8; ++k) {
        float a = s1 * roots[i1 * 8 + k];
        float b = s2 * roots[i2 * 8 + k];
        w[m * K + o * 8 + k] = a + b;
      }
    }
}

/* ------------------------------------------------------------------ */
/* Recursive PolarQuant (polarflash_quant/polar/polar_quant.py)          */
/* ------------------------------------------------------------------ */
#define PFO_PI_F 3.14159274101257324f /* float32(math.pi) */
#define PFO_2PI_F 6.28318548202514648f
#define PFO_HALFPI_F 1.57079637050628662f

/* compute_adaptive_bit_allocation (polar_quant.py:352-379). */
PFO_API int pfo_polar_alloc(int d, double target_bpw, int* alloc) {
  int total = (int)llround(d * target_bpw);
  if (d == 2) {
    int rb = total / 2 > 2 ? total / 2 : 2;
    int tb = total - rb > 1 ? total - rb : 1;
    alloc[0] = rb;
    alloc[1] = tb;
    return 2;
  }
  long rr = lround(target_bpw + 1.0);
  /* python round() is half-to-even */
  {
    double v = target_bpw + 1.0, fl = floor(v);
    if (v - fl == 0.5) rr = ((long)fl % 2 == 0) ? (long)fl : (long)fl + 1;
  }
  int r_bits = (int)(rr < 4 ? rr : 4);
  if (r_bits < 2) r_bits = 2;
  int rem_bits = total - r_bits > d - 1 ? total - r_bits : d - 1;
  alloc[0] = r_bits;
  int na = d - 1, base = rem_bits / na, rem = rem_bits % na;
  for (int i = 0; i < na; ++i) {
    int b = base + (i < rem ? 1 : 0);
    alloc[1 + i] = b > 1 ? b : 1;
  }
  int sum = 0;
  for (int i = 0; i < d; ++i) sum += alloc[i];
  while (sum < total) { alloc[1] += 1; sum++; }
  while (sum > total && alloc[d - 1] > 1) { alloc[d - 1] -= 1; sum--; }
  return d;
}

/* MSB-first continuous bitstream (polar_quant.py:463-473; identical to the
 * big-endian word path at :448-461 for 8/16/32/64-bit blocks). */
static uint64_t get_bits_msb(const uint8_t* buf, int64_t bit, int n) {
  uint64_t v = 0;
  for (int i = 0; i < n; ++i) {
    int64_t b = bit + i;
    v = (v << 1) | ((buf[b >> 3] >> (7 - (b & 7))) & 1u);
  }
  return v;
}
static void put_bits_msb(uint8_t* buf, int64_t bit, int n, uint64_t v) {
  for (int i = 0; i < n; ++i) {
    int64_t b = bit + i;
    if ((v >> (n - 1 - i)) & 1u) buf[b >> 3] |= (uint8_t)(1u << (7 - (b & 7)));
  }
}

/* Bit packing half of encode_packed (polar_quant.py:440-473): the block words
 * (radius code most significant, then the angle codes level by level) written
 * as one MSB-first stream of `total_bits` per block.  The float half of the
 * encoder (forward_recursive and the code quantisation) runs on torch in
 * oracle/__init__.py, because its results depend on torch's own sqrt/atan2. */
PFO_API void pfo_pack_bits_msb(const uint64_t* words, int64_t nblk, int total_bits, uint8_t* out) {
  memset(out, 0, (size_t)((nblk * total_bits + 7) / 8));
  for (int64_t b = 0; b < nblk; ++b) put_bits_msb(out, b * total_bits, total_bits, words[b]);
}

PFO_API void pfo_unpack_bits_msb(const uint8_t* buf, int64_t nblk, int total_bits, uint64_t* words) {
  for (int64_t b = 0; b < nblk; ++b) words[b] = get_bits_msb(buf, b * total_bits, total_bits);
}

/* decode_packed + inverse_recursive (polar_quant.py:489-575, 252-272), fp32.
 * Blocks start at bit b * total_bits of the stream.  With learned angle
 * codebooks (n_cb levels, level l holding cb_len[l] floats from cb +
 * sum(cb_len[0..l-1]); polar_quant.py:552-554) an angle of level l < n_cb is
 * cb[l][clamp(code, 0, cb_len[l] - 1)]; other levels use the uniform grid. */
PFO_API void pfo_polar_decode_cb(const uint8_t* packed, int64_t nblk, int d, const int* alloc, double r_scale,
                                 const float* cb, const int* cb_len, int n_cb, float* out) {
  int total_bits = 0;
  for (int i = 0; i < d; ++i) total_bits += alloc[i];
  float rs = (float)r_scale;
#pragma omp parallel for schedule(static)
  for (int64_t b = 0; b < nblk; ++b) {
    uint64_t word = get_bits_msb(packed, b * total_bits, total_bits);
    int codes[64];
    int shift = 0;
    for (int i = d - 1; i >= 0; --i) {
      codes[i] = (int)((word >> shift) & ((1u << alloc[i]) - 1u));
      shift += alloc[i];
    }
    float th[64];
    int col = 0, dd = d;
    for (int lvl = 0; dd > 1; ++lvl) {
      int cb_off = 0;
      for (int l = 0; l < lvl && l < n_cb; ++l) cb_off += cb_len[l];
      for (int j = 0; j < dd / 2; ++j) {
        int c = codes[1 + col + j];
        if (lvl < n_cb) {
          int cc = c < cb_len[lvl] - 1 ? c : cb_len[lvl] - 1;
          th[col + j] = cb[cb_off + cc];
          continue;
        }
        float L = (float)(1 << alloc[1 + col + j]);
        float t = ((float)c + 0.5f) / L;
        th[col + j] = lvl == 0 ? t * PFO_2PI_F - PFO_PI_F : t * PFO_HALFPI_F;
      }
      col += dd / 2;
      dd /= 2;
    }
    /* top-down: level L-1 has 1 angle at column d-2 */
    float cur[64], nxt[64];
    cur[0] = (float)codes[0] * rs;
    int width = 1;
    int base = d - 1; /* start column index past the last level */
    while (width < d) {
      base -= width;
      for (int j = 0; j < width; ++j) {
        float t = th[base + j];
        nxt[2 * j] = cur[j] * cosf(t);
        nxt[2 * j + 1] = cur[j] * sinf(t);
      }
      width *= 2;
      for (int j = 0; j < width; ++j) cur[j] = nxt[j];
    }
    for (int i = 0; i < d; ++i) out[b * d + i] = cur[i];
  }
}

PFO_API void pfo_polar_decode(const uint8_t* packed, int64_t nblk, int d, const int* alloc,
                              double r_scale, float* out) {
  pfo_polar_decode_cb(packed, nblk, d, alloc, r_scale, 0, 0, 0, out);
}

/* 2-D polar payload (polar_quant.py:18-73, unified_quantizer.py:288-312):
 * (r << theta_bits | theta) MSB-first per pair; r_hat = r * r_scale,
 * theta = ((c + 0.5) / 2^tb) * 2pi - pi, theta = 0 where r_hat <= 1e-12. */
PFO_API void pfo_polar2d_decode(const uint8_t* packed, int64_t npairs, int r_bits, int th_bits,
                                double r_scale, float* out) {
  int pb = r_bits + th_bits;
  float rs = (float)r_scale;
  float L = (float)(1 << th_bits);
#pragma omp parallel for schedule(static)
  for (int64_t i = 0; i < npairs; ++i) {
    uint64_t v = get_bits_msb(packed, i * pb, pb);
    int th = (int)(v & ((1u << th_bits) - 1u));
    int r = (int)((v >> th_bits) & ((1u << r_bits) - 1u));
    float rh = (float)r * rs;
    float t = (((float)th + 0.5f) / L) * PFO_2PI_F - PFO_PI_F;
    if (rh <= 1e-12f) t = 0.f;
    out[2 * i] = rh * cosf(t);
    out[2 * i + 1] = rh * sinf(t);
  }
}

/* ------------------------------------------------------------------ */
/* Dense products                                                      */
/* ------------------------------------------------------------------ */
/* y[n][m] = sum_k W[m][k] x[n][k], accumulated in double (the oracle is more
 * exact than the reference's fp32 matmul, cpu/engine.py:93). */
PFO_API void pfo_matvec(const float* W, int64_t M, int64_t K, const float* x, int64_t N, float* y) {
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; ++m) {
    const float* wr = W + m * K;
    for (int64_t n = 0; n < N; ++n) {
      const float* xr = x + n * K;
      double acc = 0.0;
      for (int64_t k = 0; k < K; ++k) acc += (double)wr[k] * (double)xr[k];
      y[n * M + m] = (float)acc;
    }
  }
}

/* Same product in fp32 with a vectorisable inner loop: the CPU baseline's
 * matvec (what the reference's torch.matmul does on the host). */
PFO_API void pfo_matvec_f32(const float* W, int64_t M, int64_t K, const float* x, int64_t N,
                            float* y) {
#pragma omp parallel for schedule(static)
  for (int64_t m = 0; m < M; ++m) {
    const float* wr = W + m * K;
    for (int64_t n = 0; n < N; ++n) {
      const float* xr = x + n * K;
      float acc[16] = {0};
      int64_t k = 0;
      for (; k + 16 <= K; k += 16)
        for (int j = 0; j < 16; ++j) acc[j] += wr[k + j] * xr[k + j];
      float s = 0.f;
      for (int j = 0; j < 16; ++j) s += acc[j];
      for (; k < K; ++k) s += wr[k] * xr[k];
      y[n * M + m] = s;
    }
  }
}

PFO_API int pfo_num_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}

PFO_API void pfo_set_num_threads(int n) {
#ifdef _OPENMP
  if (n > 0) omp_set_num_threads(n);
#else
  (void)n;
#endif
}
