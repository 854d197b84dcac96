// Shared definitions for the sm_100a compressed-linear kernels.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "polarflash_b200.h"

namespace pfb {

constexpr int kGroup = 128;          // columns per scale group (and per GEMV k-step)
constexpr int kMaxGemvTokens = 16;   // N handled by the register-decode GEMV
constexpr int kMaxHadBlock = 8192;   // largest RWHT block the x-prep kernel stages
constexpr int kMaxCascade = 16;

// Block plan of BlockHadamardTransform (polarflash_quant/transforms/hadamard.py:93-116):
// `nfull` blocks of `block` columns, then a cascade of smaller power-of-two blocks;
// columns at or past `rot_end` (a trailing single column) are not rotated.
struct HadPlan {
  int block;  // 0 = the weight is not rotated
  int nfull;
  int ncasc;
  int rot_end;
  int casc_off[kMaxCascade];
  int casc_size[kMaxCascade];
};

// Scale handling of the INT formats.
enum ScaleMode : int { kScaleGroup = 0, kScaleRow = 1, kScaleTensor = 2 };

// Format traits used by the integer GEMV.
template <int FMT>
struct IntFmt;
template <>
struct IntFmt<PF_FMT_INT4_G128> {
  static constexpr int kBits = 4, kWordsPerGroup = 16, kOffset = 0;
};
template <>
struct IntFmt<PF_FMT_INT3_G128> {
  static constexpr int kBits = 3, kWordsPerGroup = 13, kOffset = 0;
};
template <>
struct IntFmt<PF_FMT_INT2_G128> {
  static constexpr int kBits = 2, kWordsPerGroup = 8, kOffset = 0;
};
template <>
struct IntFmt<PF_FMT_INT4> {
  static constexpr int kBits = 4, kWordsPerGroup = 16, kOffset = 8;
};
template <>
struct IntFmt<PF_FMT_INT3> {
  static constexpr int kBits = 3, kWordsPerGroup = 12, kOffset = 4;
};
template <>
struct IntFmt<PF_FMT_INT2> {
  static constexpr int kBits = 2, kWordsPerGroup = 8, kOffset = 2;
};

__host__ __device__ inline bool is_int_format(int f) { return f >= PF_FMT_INT4_G128 && f <= PF_FMT_INT2; }
__host__ __device__ inline bool is_group_int_format(int f) {
  return f >= PF_FMT_INT4_G128 && f <= PF_FMT_INT2_G128;
}
__host__ __device__ inline int int_format_bits(int f) {
  return (f == PF_FMT_INT4_G128 || f == PF_FMT_INT4) ? 4 : (f == PF_FMT_INT3_G128 || f == PF_FMT_INT3) ? 3 : 2;
}

// Column pair (lo, hi), inside a 128-column group, that a GEMV thread with
// quad index `c` (lane & 3) holds in its i-th packed half2 (i = 0..15).  The
// tensor-core k-slots of the thread are bound to these columns, and the
// x-prep kernel writes x in the same permuted order, so the codes never move.
//   INT4: thread c owns words 4c..4c+3; half2 i = codes (p, p+4) of word i/4.
//   INT2: words 2c, 2c+1; half2 i = codes (p, p+8) of word i/8.
//   INT3 g128 (10 codes/word, 13 words): words c, c+4, c+8 give codes (p, p+5),
//         and word 12 gives codes (2c, 2c+1).
//   INT3 reference stream: words 3c..3c+2 hold codes 32c..32c+31; three 10-code
//         windows give (p, p+5), the last two codes form half2 15.
__device__ __forceinline__ void frag_cols(int fmt, int c, int i, int& lo, int& hi) {
  switch (fmt) {
    case PF_FMT_INT4_G128:
    case PF_FMT_INT4: {
      int w = 4 * c + (i >> 2), p = i & 3;
      lo = 8 * w + p;
      hi = lo + 4;
      break;
    }
    case PF_FMT_INT2_G128:
    case PF_FMT_INT2: {
      int w = 2 * c + (i >> 3), p = i & 7;
      lo = 16 * w + p;
      hi = lo + 8;
      break;
    }
    case PF_FMT_INT3_G128: {
      if (i < 15) {
        int t = i / 5, p = i % 5, w = c + 4 * t;
        lo = 10 * w + p;
        hi = lo + 5;
      } else {
        lo = 120 + 2 * c;
        hi = lo + 1;
      }
      break;
    }
    default: {  // PF_FMT_INT3
      if (i < 15) {
        int t = i / 5, p = i % 5;
        lo = 32 * c + 10 * t + p;
        hi = lo + 5;
      } else {
        lo = 32 * c + 30;
        hi = lo + 1;
      }
      break;
    }
  }
}

// In-place decode map of the TMA GEMV (gemv_tma.cu): the thread's i-th half2
// holds the codes of columns (lo, hi) at mantissa bit position p, extracted
// with one AND/OR and no shift where the code already sits below bit 10.
//   INT4 (words 4c..4c+3, word t = i/4): (0,4)@0 (1,5)@4, then >>8: (2,6)@0 (3,7)@4
//   INT2 (words 2c, 2c+1, word t = i/8): (k, k+8)@2k for k < 5, then >>10:
//        (5+k, 13+k)@2k for k < 3
//   INT3 g128 (words c, c+4, c+8 merged with <<1 halves): (0,5)@0 (1,6)@3 (2,7)@6,
//        then >>9: (3,8)@0 (4,9)@3; half2 15 = word 12 codes (2c, 2c+1)@0
__device__ __forceinline__ void frag_cols2(int fmt, int c, int i, int& lo, int& hi, int& p) {
  switch (fmt) {
    case PF_FMT_INT4_G128:
    case PF_FMT_INT4: {
      int w = 4 * c + (i >> 2), sub = i & 3;
      lo = 8 * w + sub;
      hi = lo + 4;
      p = (sub & 1) ? 4 : 0;
      break;
    }
    case PF_FMT_INT2_G128:
    case PF_FMT_INT2: {
      int w = 2 * c + (i >> 3), sub = i & 7;
      lo = 16 * w + sub;
      hi = lo + 8;
      p = sub < 5 ? 2 * sub : 2 * (sub - 5);
      break;
    }
    default: {  // PF_FMT_INT3_G128
      if (i < 15) {
        int t = i / 5, sub = i % 5, w = c + 4 * t;
        lo = 10 * w + sub;
        hi = lo + 5;
        p = (sub == 1 || sub == 4) ? 3 : (sub == 2 ? 6 : 0);
      } else {
        lo = 120 + 2 * c;
        hi = lo + 1;
        p = 0;
      }
      break;
    }
  }
}

__device__ __forceinline__ float load_x(const void* x, int dtype, size_t idx) {
  if (dtype == PF_DTYPE_F16) return __half2float(static_cast<const __half*>(x)[idx]);
  if (dtype == PF_DTYPE_BF16) return __bfloat162float(static_cast<const __nv_bfloat16*>(x)[idx]);
  return static_cast<const float*>(x)[idx];
}

// Host-side launch helpers (prep.cu).
struct PrepArgs {
  const void* x;
  int x_dtype;
  int N;       // real tokens
  int slots;   // token slots written (>= N; padded slots are zero)
  int K;
  int Kp;      // K rounded up to a whole group
  HadPlan plan;
  const int8_t* signs;
  int mode;    // 0: tensor-core fragments, 1: plain fp32 x'
  int fmt;
  int NT;      // n8 tiles of the fragment layout
  uint2* xfrag;
  float* sx;
  float* xplain;
  float* y;    // initialised to bias (or 0) when init_y
  const float* bias;
  int M;
  int init_y;
};

cudaError_t launch_prep(const PrepArgs& a, cudaStream_t stream);
int prep_chunk_cols(const HadPlan& plan);

}  // namespace pfb
