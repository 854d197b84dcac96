// Launch interfaces of the GEMV / dequant kernels (host side).
#pragma once

#include "common.cuh"

namespace pfb {

struct GemvIntArgs {
  const void* codes;
  const void* scales;  // fp16 [M][G] (group) or fp32 [M] (row)
  const __half* mins;  // fp16 [M][G] (group)
  float tensor_scale;
  int M, K, N;
  int G;          // groups per row (partial last group included)
  int Gp;         // groups in the fragment buffer
  int row_words;  // u32 words per row
  int NT;
  int CG;         // groups per work item
  int n_row_items;
  int n_items;
  int n_chunks;
  const uint2* xfrag;
  const float* sx;
  const float* bias;
  float* y;
  float* partials;     // [n_chunks][N][M] when n_chunks > 1
  unsigned* counters;  // [n_row_items], zero on entry, left zero on exit
};

int gemv_int_rows_per_item(int NT);
cudaError_t launch_gemv_int(int fmt, const GemvIntArgs& a, int smode, cudaStream_t s);

struct GemvCCArgs {
  int fmt;
  const void* codes;
  const void* scales;
  int M, K, N;
  int Kp;
  const float* xplain;  // [N][Kp]
  const float* bias;
  float* y;
  // polar
  int d;
  int tb;          // bits per block
  int row_bytes;
  int alloc[17];
  float r_scale;
  int zero_rule;   // 2-D polar: theta = 0 where r_hat <= 1e-12
};

cudaError_t launch_gemv_cc(const GemvCCArgs& a, cudaStream_t s);

struct DequantArgs {
  int fmt;
  const void* codes;
  const void* scales;
  const __half* mins;
  float tensor_scale;
  int M, K;
  int row_words;
  int d, tb, row_bytes, zero_rule;
  int alloc[17];
  float r_scale;
  float* W;        // [M][K] fp32, or nullptr
  uint8_t* codes_out;  // unpack mode
};

cudaError_t launch_dequant(const DequantArgs& a, cudaStream_t s);
cudaError_t launch_unpack(const DequantArgs& a, cudaStream_t s);
cudaError_t launch_rwht_rows(const float* in, float* out, int rows, int K, const HadPlan& plan,
                             const int8_t* signs, int inverse, cudaStream_t s);

}  // namespace pfb
