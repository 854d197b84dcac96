// Launch interfaces of the GEMV / dequant kernels (host side).
#pragma once

#include "common.cuh"

namespace pfb {

// Adds one to the library's count of kernel launches (read by
// pf_kernel_launches); called after every launch this library makes.
void note_launch();
// PF_OK, or PF_ERR_CUDA with `e` kept for pf_last_cuda_error.
int report_cuda(cudaError_t e);
// The workspace head after the stream's work: the status word (PF_OK or the
// PF_ERR_* a kernel recorded), optionally the number of non-zero arrival
// counters, then optionally zeroed again (pf_workspace_status).
int read_workspace_head(void* ws, int reset, int* status, int* busy_counters, cudaStream_t s);

// The least workspace pf_qlinear accepts for (w, N) (pf_qlinear_workspace_size
// reports the size for the fastest paths, which can be larger).
size_t min_workspace_bytes(const pf_qweight* w, int N);

// Workspace head: split-K arrival counters (zero-filled once by the owner of
// the workspace, left zero by every call); the last slot records a device
// status word (PF_ERR_TIMEOUT when a bounded pipeline wait gave up).
constexpr size_t kWsCounterSlots = 16384;
constexpr size_t kWsCounterBytes = kWsCounterSlots * sizeof(unsigned);
constexpr size_t kWsStatusSlot = kWsCounterSlots - 1;
// CTAs of a gathering GEMV launch that have finished (zero, left zero)
constexpr size_t kWsDoneSlot = kWsStatusSlot - 1;

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
  const float* angles;  // recursive polar: learned angle table [d-1][64], or nullptr
};

cudaError_t launch_gemv_cc(const GemvCCArgs& a, cudaStream_t s);

// ---- streaming integer GEMV (gemv_tma.cu): up to kTmaMaxJobs weights of one
// format per launch, each with its own input.  The forward RWHT of every
// input is prepared once, by launch_xprep_frag, as tensor-core B-fragment
// records in the workspace; the GEMV streams them with the weights.
constexpr int kTmaMaxJobs = 16;
constexpr int kLutGroupJobs = 4;  // weights per table-GEMV launch (gemv_lut.cu)

struct TmaJob {  // device view of one weight of a launch
  const void* scales;         // fp16 [M][G] (group) or fp32 [M] (row)
  const __half* mins;         // fp16 [M][G] (group)
  const unsigned char* xq;    // x' records of the job's input, [G][record bytes]
  const float* bias;
  float* y;                   // [N][M] fp32
  float* partials;            // [n_rb][spb][128][N] partial sums of split row blocks (spb > 1)
  float tensor_scale;
  int M, K, G, n_rb, spb;
  int unit0;                  // first unit of the job
  int tile0;                  // first 16-row arrival counter of the job
  int fsel;                   // 0: the launch's first format, 1: its second
  // gathering launches: y of the whole linear at byte offset yoff of every
  // rank's peer buffer, [N][m_full], this rank's rows from row0
  unsigned long long yoff;
  int m_full, row0;
};

// Peer buffers of a gathering launch (pf_peers): world ranks' buffers, each
// mapped in this process; the first kPeerHeader bytes hold the rank's epoch
// (offset 0) and one flag per source rank (offset 16 + 4 q).
constexpr int kMaxPeers = 8;
constexpr size_t kPeerHeader = 256;

struct TmaArgs {
  TmaJob job[kTmaMaxJobs];
  unsigned* counters;   // workspace head: 16-row arrival counters (zero, left zero)
  unsigned* status;     // workspace status word
  unsigned* done;       // gathering launches: finished-CTA counter (zero, left zero)
  unsigned char* peer[kMaxPeers];  // gathering launches: every rank's peer buffer
  int world, rank;      // world 0: y goes to job.y (no gathering)
  int n_jobs, n_units, N;
  int NS, XS;           // ring stages of the CTA (XS unused)
  unsigned xstage;      // bytes of one stage of x' records (a multiple of 128)
};

struct TmaWeight {  // host view of one weight
  int format, M, K, had_block;
  const void* codes;
  const void* scales;
  const void* mins;
  const int8_t* signs;
  float tensor_scale;
};
struct TmaIO {
  const void* x;
  const float* bias;
  float* y;
  const unsigned char* xq;  // the job's x' records (from launch_xprep_frag)
  unsigned long long yoff;  // gathering launches: the job's y in the peer buffers
  int m_full, row0;
};

// One input of launch_xprep_frag: x' records of x [N][K] for weights of
// format `fmt` rotated with `had_block` (0: none) and `signs`.
struct XPrepJob {
  const void* x;
  const int8_t* signs;
  unsigned char* xq;  // out: [K/128][tma_xrec_bytes(N)]
  float had_rscale;
  int had_block;
  int K;
  int fmt;
  int blk0;           // first prep block of this input (set by launch_xprep_frag)
};
constexpr int kXPrepMaxJobs = 2 * kTmaMaxJobs;

bool tma_eligible(const TmaWeight& w);
// Bytes of one 128-column group of x' records for N tokens.
size_t tma_xrec_bytes(int N);
// Workspace bytes of a job's split row-block partial sums.
size_t tma_partial_bytes(const TmaWeight& w, int N);
// 16-row arrival counters one weight uses.
int tma_tiles(const TmaWeight& w);
int tma_block_rows();
int tma_stage_groups(int fmt);
int row_words_of_tma(int fmt, int K);
// x' records of `count` inputs (any streaming formats) in one launch.
int launch_xprep_frag(XPrepJob* xj, int count, int N, int x_dtype, cudaStream_t s, cudaError_t* err);
// One GEMV launch for `count` weights (of one format, or of INT3 and INT2
// group-128 together; each with its x' records in io[k].xq) and N <= 16
// tokens; split row blocks are reduced inside the launch.  `workspace` holds the counter/status head; every job's partial
// sums follow one another from `partials` (tma_partial_bytes each, in job
// order).  Returns a pf_status; *err receives a CUDA error.
// `peers` (nullable): a gathering launch, each job's rows stored into every
// rank's peer buffer, then the rank's flag raised in every buffer.
int launch_gemv_tma(const TmaWeight* ws, const TmaIO* io, int count, int N, void* workspace, char* partials,
                    const pf_peers* peers, cudaStream_t s, cudaError_t* err);

// ---- streaming lookup-table GEMVs at batch 1 (gemv_lut.cu): E8 RVQ2, and
// recursive polar with block 8 and allocation [3 | 2 2 2 2 | 1 1 | 1]
struct E8In {
  const void* codes;     // uint16 [M][K/8]: stage-1 root index (low byte), stage-2 (high byte)
  const void* scales;    // half2 [M][K/128]: (stage-1, stage-2) scale per 128-column group
  const void* x;         // [K] activations (x_dtype)
  int x_dtype;
  const int8_t* signs;   // RWHT column signs (had_block > 0)
  int had_block;         // 0 or a power of two <= 512 dividing K
  const float* bias;
  float* y;              // [M] fp32
  int M, K;
};
// Shapes, alignments and rotation blocks the kernel takes (else the GEMM serves E8).
bool e8_lut_eligible(const E8In& in);
// Workspace bytes after the counter/status head: the stage partial sums.
size_t e8_lut_partial_bytes(int M, int K);
// One GEMV launch over `count` <= 4 weights that share x, K and the rotation
// (+ one partial-sum combine launch when K spans several 256-column stages);
// the workspace holds the status word in its head, then every weight's stage
// partial sums.  Returns a pf_status.
int launch_e8_lut(const E8In* in, int count, void* workspace, cudaStream_t s, cudaError_t* err);

struct Polar8In {
  const void* codes;     // rows of K/8 14-bit MSB-first block codes (K * 7 / 32 bytes per row)
  int alloc[8];          // the block allocation (must be 3 2 2 2 2 1 1 1)
  float r_scale;
  const float* angles;   // learned angle table [7][64], or nullptr (uniform angles)
  const void* x;
  int x_dtype;
  const int8_t* signs;
  int had_block;
  const float* bias;
  float* y;
  int M, K;
};
bool polar8_lut_eligible(const Polar8In& in);
size_t polar8_lut_partial_bytes(int M, int K);
int launch_polar8_lut(const Polar8In* in, int count, void* workspace, cudaStream_t s, cudaError_t* err);

// ---- tensor-core dequant-GEMM (gemm_tc.cu) for N > 16 tokens
struct GemmIn {
  int fmt;
  const void* codes;
  const __half* scales;
  const __half* mins;
  int M, K, Kp, N, row_words;
  const float* xplain;  // [N][Kp] fp32 x' (prep_kernel, plain mode), or nullptr: x' made from x here
  const void* x;        // [N][K] activations (when xplain == nullptr)
  int x_dtype;
  const int8_t* signs;  // RWHT column signs (block > 1)
  int block;            // rotation block tiling K (0 / 1: none)
  float rscale;         // 1/sqrt(block)
  __half* x16;          // [N][K] fp16 x' scaled per token (written here)
  float* tok_scale;     // [N]
  const float* bias;
  float* y;
  unsigned* status;
  unsigned* counters;  // workspace arrival counters (zero; left zero)
  float* partials;     // gemm_partial_bytes() of split-tile partial sums
  float r_scale;        // recursive polar: radius scale
  const float* angles;  // recursive polar: learned angle table [7][64], or nullptr
};
constexpr int kGemmPrepMaxK = 49152;  // K of the one-kernel x' preparation (K floats of smem)
constexpr int kGemmCounterSlots = (int)kWsStatusSlot;  // tiles one GEMM launch may split
bool gemm_eligible(int fmt, int K);
size_t gemm_x16_bytes(int N, int K);
size_t gemm_partial_bytes();
cudaError_t launch_gemm(const GemmIn& in, cudaStream_t s);

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
  const float* angles;  // recursive polar: learned angle table [d-1][64], or nullptr
  float* W;        // [M][K] fp32, or nullptr
  uint8_t* codes_out;  // unpack mode
};

cudaError_t launch_dequant(const DequantArgs& a, cudaStream_t s);
cudaError_t launch_unpack(const DequantArgs& a, cudaStream_t s);
cudaError_t launch_rwht_rows(const float* in, float* out, int rows, int K, const HadPlan& plan,
                             const int8_t* signs, int inverse, cudaStream_t s);

}  // namespace pfb
