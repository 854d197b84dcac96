// Launch interfaces of the GEMV / dequant kernels (host side).
#pragma once

#include "common.cuh"

namespace pfb {

// Workspace head: split-K arrival counters (zero-filled once by the owner of
// the workspace, left zero by every call); the last slot records a device
// status word (PF_ERR_TIMEOUT when a bounded pipeline wait gave up).
constexpr size_t kWsCounterSlots = 16384;
constexpr size_t kWsCounterBytes = kWsCounterSlots * sizeof(unsigned);
constexpr size_t kWsStatusSlot = kWsCounterSlots - 1;

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

// ---- TMA-pipelined integer GEMV (gemv_tma.cu) and its x-prep (prep.cu) ----
// x' record per 128-column group: [NT tiles][8 k-steps][Lp lanes] uint2 B
// fragments (Lp = 8 for N = 1, else 32), then float4 {Sx, f, SB, 0} per
// token slot (4 * NT).  Sx = sum of x' over the group, f = 2^E the group's
// power-of-two normaliser, SB = sum of the B values (normal-magic decode).
__host__ __device__ inline int tma_lanes(int N, int NT) { return (NT == 1 && N == 1) ? 8 : 32; }
__host__ __device__ inline size_t tma_record_bytes(int N, int NT) {
  return (size_t)NT * 8 * tma_lanes(N, NT) * 8 + (size_t)64 * NT;
}

struct Prep2Args {
  const void* x;
  int x_dtype;
  int N, NT, K, G;
  HadPlan plan;
  const int8_t* signs;
  int fmt;
  int subnormal;  // B scale 2^(14-p) (subnormal codes) or 2^(10-p) (1 + q 2^(p-10) codes)
  unsigned char* rec;
};
cudaError_t launch_prep2(const Prep2Args& a, cudaStream_t s);

struct TmaArgs {
  const void* codes;
  const void* scales;
  const __half* mins;
  float tensor_scale;
  int M, K, N, NT, G;
  int row_words;
  int n_rb, spb, n_units;  // row blocks, stages per row block, units
  int rows;                // rows per row block
  const unsigned char* rec;  // x' records
  int rec_bytes;
  const float* bias;
  float* y;
  float* partials;         // [2 * grid][rows][N]
  unsigned* counters;      // per (row block, consumer warp); status word at kWsStatusSlot
};
bool tma_eligible(int fmt, int M, int K, const void* codes);
int tma_grid(int fmt, int NT, int n_units);
int tma_block_rows();
cudaError_t launch_gemv_tma(int fmt, const TmaArgs& a, int smode, int subnormal, cudaStream_t s);
int tma_stage_groups(int fmt);

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
