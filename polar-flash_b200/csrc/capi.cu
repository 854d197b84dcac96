// C ABI entry points: argument validation on the host, then the launch
// sequence (x-prep, GEMV) on the caller's stream.  Nothing here allocates.
#include <stdlib.h>
#include <atomic>
#include <string.h>

#include "gemv.cuh"

using namespace pfb;

namespace {

thread_local int g_last_cuda_error = 0;

int cuda_status(cudaError_t e) {
  if (e == cudaSuccess) return PF_OK;
  g_last_cuda_error = (int)e;
  return PF_ERR_CUDA;
}

bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }
bool pow2(int v) { return v > 0 && (v & (v - 1)) == 0; }
size_t round_up(size_t v, size_t a) { return (v + a - 1) / a * a; }

// Block plan of BlockHadamardTransform._init_dims (hadamard.py:93-116).
int make_plan(int K, int block, HadPlan* p) {
  memset(p, 0, sizeof(*p));
  if (block == 0) return PF_OK;
  if (!pow2(block) || block < 2 || block > kMaxHadBlock || block > K) return PF_ERR_UNSUPPORTED;
  p->block = block;
  p->nfull = K / block;
  int off = p->nfull * block, rem = K - off;
  while (rem > 1) {
    int p2 = 1;
    while (p2 * 2 <= rem) p2 *= 2;
    if (p->ncasc >= kMaxCascade) return PF_ERR_UNSUPPORTED;
    p->casc_off[p->ncasc] = off;
    p->casc_size[p->ncasc] = p2;
    p->ncasc++;
    off += p2;
    rem -= p2;
  }
  p->rot_end = off;
  return PF_OK;
}

int row_words_of(int fmt, int K) { return row_words_of_tma(fmt, K); }

struct PolarShape {
  int d, tb, row_bytes;
  int alloc[17];
};

int polar_shape(const pf_qweight* w, PolarShape* ps) {
  memset(ps, 0, sizeof(*ps));
  if (w->format == PF_FMT_POLAR_RECURSIVE) {
    int d = w->params[0];
    if (d != 2 && d != 4 && d != 8 && d != 16) return PF_ERR_UNSUPPORTED;
    ps->d = d;
    for (int i = 0; i < d; ++i) {
      int b = w->params[1 + i];
      if (b < 1 || (i > 0 && b > 6) || (i == 0 && b > 16)) return PF_ERR_UNSUPPORTED;
      ps->alloc[i] = b;
      ps->tb += b;
    }
  } else {
    int rb = w->params[0], thb = w->params[1];
    if (rb < 1 || rb > 16 || thb < 1 || thb > 6) return PF_ERR_UNSUPPORTED;
    ps->d = 2;
    ps->alloc[0] = rb;
    ps->alloc[1] = thb;
    ps->tb = rb + thb;
  }
  if (ps->tb > 32) return PF_ERR_UNSUPPORTED;
  if (w->K % ps->d) return PF_ERR_SHAPE;
  long long bits = (long long)(w->K / ps->d) * ps->tb;
  if (bits % 8) return PF_ERR_SHAPE;
  ps->row_bytes = (int)(bits / 8);
  return PF_OK;
}

int check(const pf_qweight* w) {
  if (!w) return PF_ERR_INVALID_ARGUMENT;
  if (w->M <= 0 || w->K <= 0) return PF_ERR_SHAPE;
  if (!w->codes) return PF_ERR_INVALID_ARGUMENT;
  if (w->had_block != 0) {
    if (!w->had_signs) return PF_ERR_INVALID_ARGUMENT;
    HadPlan p;
    int st = make_plan(w->K, w->had_block, &p);
    if (st) return st;
  }
  switch (w->format) {
    case PF_FMT_INT4_G128:
    case PF_FMT_INT3_G128:
    case PF_FMT_INT2_G128: {
      if (w->K % 128) return PF_ERR_SHAPE;
      if (!w->scales || !w->mins) return PF_ERR_INVALID_ARGUMENT;
      size_t al = w->format == PF_FMT_INT4_G128 ? 16 : w->format == PF_FMT_INT2_G128 ? 8 : 4;
      if (!aligned(w->codes, al) || !aligned(w->scales, 2) || !aligned(w->mins, 2)) return PF_ERR_ALIGNMENT;
      return PF_OK;
    }
    case PF_FMT_INT4:
    case PF_FMT_INT3:
    case PF_FMT_INT2: {
      if (w->K % 32) return PF_ERR_SHAPE;
      size_t al = w->format == PF_FMT_INT4 ? 16 : w->format == PF_FMT_INT2 ? 8 : 4;
      if (!aligned(w->codes, al)) return PF_ERR_ALIGNMENT;
      if (w->scales && !aligned(w->scales, 4)) return PF_ERR_ALIGNMENT;
      return PF_OK;
    }
    case PF_FMT_E8_RVQ2_G128: {
      if (w->K % 128) return PF_ERR_SHAPE;
      if (!w->scales) return PF_ERR_INVALID_ARGUMENT;
      if (!aligned(w->codes, 2) || !aligned(w->scales, 4)) return PF_ERR_ALIGNMENT;
      return PF_OK;
    }
    case PF_FMT_POLAR_RECURSIVE:
    case PF_FMT_POLAR2D: {
      PolarShape ps;
      const int st = polar_shape(w, &ps);
      if (st) return st;
      // recursive polar: optional learned angle table (fp32 [d-1][64]); 2-D polar: none
      if (w->scales && (w->format == PF_FMT_POLAR2D || !aligned(w->scales, 4)))
        return w->format == PF_FMT_POLAR2D ? PF_ERR_INVALID_ARGUMENT : PF_ERR_ALIGNMENT;
      return PF_OK;
    }
    default: return PF_ERR_INVALID_ARGUMENT;
  }
}

int tokens_per_pass(int N) { return N < kMaxGemvTokens ? N : kMaxGemvTokens; }
int nt_of(int np) { return np <= 4 ? 1 : np <= 8 ? 2 : 4; }

// Workspace layout (every part 256-byte aligned):
//   [split-K counters + status word: kWsCounterBytes, zero-filled once, left zero]
//   [x' region: fragments + group sums (INT) or plain fp32 x' (E8 / polar)]
//   [split-K partials]
// The x' region sits at a fixed offset for a given (format family, K, N), so
// one prepare can serve several runs over weights of different M.
constexpr size_t kCounterBytes = kWsCounterBytes;

TmaWeight tma_weight(const pf_qweight* w) {
  TmaWeight t;
  t.format = w->format;
  t.M = w->M;
  t.K = w->K;
  t.had_block = w->had_block;
  t.codes = w->codes;
  t.scales = w->scales;
  t.mins = w->mins;
  t.signs = w->had_signs;
  t.tensor_scale = (float)w->tensor_scale;
  return t;
}

// The streaming GEMV (gemv_tma.cu) serves INT4/INT3/INT2 group-128 and the
// INT4/INT2 reference streams when K % 512 == 0 and the rotation block is at
// most 512; PF_GEMV_PATH=ldg forces the register-prefetch GEMV.
bool use_tma(const pf_qweight* w) {
  static int mode = -1;
  if (mode < 0) {
    const char* e = getenv("PF_GEMV_PATH");
    mode = (e && strcmp(e, "ldg") == 0) ? 0 : 1;
  }
  if (!mode) return false;
  return tma_eligible(tma_weight(w));
}

// x alignment of the streaming GEMV's vector loads (else the other path runs)
bool x_tma_aligned(const void* x, int x_dtype) { return aligned(x, x_dtype == PF_DTYPE_F32 ? 16 : 8); }

struct IntPlan {
  int NT, rpi, n_row_items, CG, n_chunks, Gp;
};

IntPlan plan_int(const pf_qweight* w, int np) {
  IntPlan p;
  p.NT = nt_of(np);
  p.rpi = gemv_int_rows_per_item(p.NT);
  p.Gp = (w->K + 127) / 128;
  p.n_row_items = (w->M + p.rpi - 1) / p.rpi;
  const long long target = 148LL * 16;  // warps resident across the 148 SMs
  long long cg = ((long long)p.Gp * p.n_row_items + target - 1) / target;
  if (cg < 1) cg = 1;
  if (cg > p.Gp) cg = p.Gp;
  if ((size_t)p.n_row_items >= kWsStatusSlot) cg = p.Gp;  // enough rows: no split
  p.CG = (int)cg;
  p.n_chunks = (p.Gp + p.CG - 1) / p.CG;
  return p;
}

size_t xprep_bytes(const pf_qweight* w, int np) {
  size_t Gp = (size_t)(w->K + 127) / 128;
  if (is_int_format(w->format)) {
    int NT = nt_of(np);
    return round_up((size_t)NT * Gp * 2048, 256) + round_up(Gp * 8 * NT * sizeof(float), 256);
  }
  return round_up((size_t)np * Gp * 128 * sizeof(float), 256);
}

// One pass of the register-prefetch / CUDA-core path.
size_t ldg_pass_bytes(const pf_qweight* w, int np) {
  size_t b = kCounterBytes + xprep_bytes(w, np);
  if (is_int_format(w->format)) {
    IntPlan p = plan_int(w, np);
    if (p.n_chunks > 1) b += round_up((size_t)p.n_chunks * np * w->M * sizeof(float), 256);
  }
  return b;
}

// The streaming GEMV's workspace for one weight: its input's x' records,
// then its split row blocks' partial sums.
size_t tma_xq_bytes(const pf_qweight* w, int np) { return round_up((size_t)(w->K / 128) * tma_xrec_bytes(np), 256); }
size_t tma_member_bytes(const pf_qweight* w, int np) {
  return tma_xq_bytes(w, np) + tma_partial_bytes(tma_weight(w), np);
}

// Streaming-GEMV weights also fit the other path (taken for misaligned x).
size_t pass_bytes(const pf_qweight* w, int np) {
  size_t b = ldg_pass_bytes(w, np);
  if (use_tma(w)) {
    size_t t = kCounterBytes + tma_member_bytes(w, np);
    if (t > b) b = t;
  }
  return b;
}

// Batches of more than 16 tokens of the group-128 INT and E8 formats run on
// the tensor-core dequant-GEMM, kGemmChunk tokens per launch; its workspace
// holds fp32 x' and the per-token-scaled fp16 copy the GEMM reads.
constexpr int kGemmChunk = 512;
// Recursive polar with block 8 and allocation [3 | 2 2 2 2 | 1 1 | 1] (1.75 bpw).
bool is_polar8_175(const pf_qweight* w) {
  static const int32_t k[9] = {8, 3, 2, 2, 2, 2, 1, 1, 1};
  return w->format == PF_FMT_POLAR_RECURSIVE && memcmp(w->params, k, sizeof(k)) == 0;
}
bool use_gemm(const pf_qweight* w, int N) {
  static int mode = -1;
  if (mode < 0) {
    const char* e = getenv("PF_GEMM");
    mode = (e && strcmp(e, "0") == 0) ? 0 : 1;
  }
  if (w->format == PF_FMT_POLAR_RECURSIVE)  // above batch 1 (the table GEMV's), on the persistent kernel
    return mode && N >= 2 && is_polar8_175(w) && gemm_eligible(w->format, w->K) && aligned(w->codes, 16);
  // E8 decodes through a shared-memory root table: the tensor-core kernel
  // serves it at every batch size; the INT formats use it above 16 tokens
  const int min_tokens = w->format == PF_FMT_E8_RVQ2_G128 ? 1 : kMaxGemvTokens + 1;
  if (!mode || N < min_tokens || !gemm_eligible(w->format, w->K)) return false;
  // the GEMM reads packed rows with 16-byte loads (INT3: 4-byte), E8 scales as fp16 pairs
  if (w->format != PF_FMT_INT3_G128 && !aligned(w->codes, 16)) return false;
  return w->format != PF_FMT_E8_RVQ2_G128 || aligned(w->scales, 4);
}
// `partials`: room for the stream-K kernel's split-tile partial sums; a
// workspace without it runs the GEMM on the non-persistent kernel.
size_t gemm_bytes(const pf_qweight* w, int N, bool partials = true) {
  const int nc = N < kGemmChunk ? N : kGemmChunk;
  const size_t Kp = (size_t)((w->K + 127) / 128) * 128;
  return kCounterBytes + round_up((size_t)nc * Kp * sizeof(float), 256) + gemm_x16_bytes(nc, w->K) +
         (partials ? gemm_partial_bytes() : 0);
}

// Batch-1 E8 runs on the lookup-table GEMV when its shapes and alignments
// allow (PF_E8_LUT=0 keeps it on the GEMM).
bool e8_lut_enabled() {
  static int mode = -1;
  if (mode < 0) {
    const char* e = getenv("PF_E8_LUT");
    mode = (e && strcmp(e, "0") == 0) ? 0 : 1;
  }
  return mode == 1;
}
E8In e8_in(const pf_qweight* w, const HadPlan& plan, const void* x, int x_dtype, const float* bias, float* y) {
  E8In e;
  e.codes = w->codes;
  e.scales = w->scales;
  e.x = x;
  e.x_dtype = x_dtype;
  e.signs = w->had_signs;
  e.had_block = plan.block > 1 ? plan.block : 0;
  e.bias = bias;
  e.y = y;
  e.M = w->M;
  e.K = w->K;
  return e;
}
bool use_e8_lut(const pf_qweight* w, int N, const HadPlan& plan, const void* x, int x_dtype) {
  if (N != 1 || w->format != PF_FMT_E8_RVQ2_G128 || !e8_lut_enabled()) return false;
  if (plan.ncasc != 0 || (plan.block > 1 && plan.rot_end != w->K)) return false;
  return e8_lut_eligible(e8_in(w, plan, x, x_dtype, nullptr, nullptr));
}
// Batch-1 recursive polar with 8-column blocks at 1.75 bpw likewise runs on a
// lookup-table GEMV (PF_POLAR_LUT=0 keeps it on the CUDA-core kernel).
bool polar_lut_enabled() {
  static int mode = -1;
  if (mode < 0) {
    const char* e = getenv("PF_POLAR_LUT");
    mode = (e && strcmp(e, "0") == 0) ? 0 : 1;
  }
  return mode == 1;
}
Polar8In polar8_in(const pf_qweight* w, const HadPlan& plan, const void* x, int x_dtype, const float* bias, float* y) {
  Polar8In p;
  memset(&p, 0, sizeof(p));
  p.codes = w->codes;
  for (int i = 0; i < 8; ++i) p.alloc[i] = w->params[1 + i];
  p.r_scale = (float)w->tensor_scale;
  p.angles = static_cast<const float*>(w->scales);
  p.x = x;
  p.x_dtype = x_dtype;
  p.signs = w->had_signs;
  p.had_block = plan.block > 1 ? plan.block : 0;
  p.bias = bias;
  p.y = y;
  p.M = w->M;
  p.K = w->K;
  return p;
}
bool use_polar_lut(const pf_qweight* w, int N, const HadPlan& plan, const void* x, int x_dtype) {
  if (N != 1 || w->format != PF_FMT_POLAR_RECURSIVE || w->params[0] != 8 || !polar_lut_enabled()) return false;
  if (plan.ncasc != 0 || (plan.block > 1 && plan.rot_end != w->K)) return false;
  return polar8_lut_eligible(polar8_in(w, plan, x, x_dtype, nullptr, nullptr));
}

// full: the size pf_qlinear_workspace_size reports (fastest paths); without
// it, the least pf_qlinear accepts.
size_t workspace_bytes(const pf_qweight* w, int N, bool full = true) {
  if (N < 1) N = 1;
  if ((w->format == PF_FMT_E8_RVQ2_G128 || (w->format == PF_FMT_POLAR_RECURSIVE && w->params[0] == 8)) && N == 1) {
    // either path, depending on the input's alignment
    const size_t part = w->format == PF_FMT_E8_RVQ2_G128 ? e8_lut_partial_bytes(w->M, w->K)
                                                         : polar8_lut_partial_bytes(w->M, w->K);
    const size_t lut = kCounterBytes + part;
    const size_t other = use_gemm(w, N) ? gemm_bytes(w, N, full) : pass_bytes(w, 1);
    return lut > other ? lut : other;
  }
  size_t b = pass_bytes(w, tokens_per_pass(N));
  int tail = N % kMaxGemvTokens;
  if (N > kMaxGemvTokens && tail) {
    size_t t = pass_bytes(w, tail);
    if (t > b) b = t;
  }
  if (use_gemm(w, N)) {
    const size_t g = gemm_bytes(w, N, full);
    if (w->format != PF_FMT_POLAR_RECURSIVE) return g;
    // polar takes the GEMM only with room for its partial tiles, else the CUDA-core passes
    return full ? (g > b ? g : b) : b;
  }
  return b;
}

size_t dtype_size(int dt) { return dt == PF_DTYPE_F32 ? 4 : 2; }

int do_prepare(const pf_qweight* w, const HadPlan& plan, const void* x, int x_dtype, int N, void* ws,
               cudaStream_t s) {
  const int Gp = (w->K + 127) / 128;
  char* base = static_cast<char*>(ws) + kCounterBytes;
  PrepArgs pa;
  memset(&pa, 0, sizeof(pa));
  pa.x = x;
  pa.x_dtype = x_dtype;
  pa.N = N;
  pa.K = w->K;
  pa.Kp = Gp * 128;
  pa.plan = plan;
  pa.signs = w->had_signs;
  pa.fmt = w->format;
  pa.M = w->M;
  pa.init_y = 0;
  if (is_int_format(w->format)) {
    const int NT = nt_of(N);
    pa.mode = 0;
    pa.NT = NT;
    pa.slots = 4 * NT;
    pa.xfrag = reinterpret_cast<uint2*>(base);
    pa.sx = reinterpret_cast<float*>(base + round_up((size_t)NT * Gp * 2048, 256));
  } else {
    pa.mode = 1;
    pa.slots = N;
    pa.xplain = reinterpret_cast<float*>(base);
  }
  return cuda_status(launch_prep(pa, s));
}

int do_run(const pf_qweight* w, int N, const float* bias, float* y, void* ws, cudaStream_t s) {
  const int K = w->K, M = w->M;
  const int Gp = (K + 127) / 128;
  char* base = static_cast<char*>(ws) + kCounterBytes;
  if (is_int_format(w->format)) {
    IntPlan p = plan_int(w, N);
    GemvIntArgs ga;
    memset(&ga, 0, sizeof(ga));
    ga.codes = w->codes;
    ga.scales = w->scales;
    ga.mins = static_cast<const __half*>(w->mins);
    ga.tensor_scale = (float)w->tensor_scale;
    ga.M = M;
    ga.K = K;
    ga.N = N;
    ga.G = Gp;
    ga.Gp = Gp;
    ga.row_words = row_words_of(w->format, K);
    ga.NT = p.NT;
    ga.CG = p.CG;
    ga.n_row_items = p.n_row_items;
    ga.n_chunks = p.n_chunks;
    ga.n_items = p.n_row_items * p.n_chunks;
    ga.xfrag = reinterpret_cast<const uint2*>(base);
    ga.sx = reinterpret_cast<const float*>(base + round_up((size_t)p.NT * Gp * 2048, 256));
    ga.bias = bias;
    ga.y = y;
    ga.partials = reinterpret_cast<float*>(base + xprep_bytes(w, N));
    ga.counters = static_cast<unsigned*>(ws);
    int smode = is_group_int_format(w->format) ? kScaleGroup : (w->scales ? kScaleRow : kScaleTensor);
    return cuda_status(launch_gemv_int(w->format, ga, smode, s));
  }
  GemvCCArgs ca;
  memset(&ca, 0, sizeof(ca));
  ca.fmt = w->format;
  ca.codes = w->codes;
  ca.scales = w->scales;
  ca.M = M;
  ca.K = K;
  ca.N = N;
  ca.Kp = Gp * 128;
  ca.xplain = reinterpret_cast<const float*>(base);
  ca.bias = bias;
  ca.y = y;
  if (w->format != PF_FMT_E8_RVQ2_G128) {
    PolarShape ps;
    polar_shape(w, &ps);
    ca.d = ps.d;
    ca.tb = ps.tb;
    ca.row_bytes = ps.row_bytes;
    memcpy(ca.alloc, ps.alloc, sizeof(ca.alloc));
    ca.r_scale = (float)w->tensor_scale;
    ca.zero_rule = w->format == PF_FMT_POLAR2D;
    ca.angles = w->format == PF_FMT_POLAR_RECURSIVE ? static_cast<const float*>(w->scales) : nullptr;
  }
  return cuda_status(launch_gemv_cc(ca, s));
}

}  // namespace

size_t pfb::min_workspace_bytes(const pf_qweight* w, int N) { return workspace_bytes(w, N, false); }
int pfb::report_cuda(cudaError_t e) { return cuda_status(e); }

static std::atomic<unsigned long long> g_launches{0};
void pfb::note_launch() { g_launches.fetch_add(1, std::memory_order_relaxed); }

extern "C" {

unsigned long long pf_kernel_launches(void) { return g_launches.load(std::memory_order_relaxed); }

const char* pf_version(void) { return "polarflash_b200 0.1.0 (sm_100a)"; }

const char* pf_status_string(int status) {
  switch (status) {
    case PF_OK: return "ok";
    case PF_ERR_INVALID_ARGUMENT: return "invalid argument";
    case PF_ERR_SHAPE: return "unsupported shape";
    case PF_ERR_ALIGNMENT: return "misaligned device pointer";
    case PF_ERR_UNSUPPORTED: return "unsupported format parameters";
    case PF_ERR_WORKSPACE: return "workspace missing or too small";
    case PF_ERR_CUDA: return "CUDA error";
    case PF_ERR_TIMEOUT: return "device wait timed out";
    default: return "unknown status";
  }
}

int pf_last_cuda_error(void) { return g_last_cuda_error; }

int pf_qweight_check(const pf_qweight* w) { return check(w); }

int pf_qlinear_workspace_size(const pf_qweight* w, int N, size_t* bytes) {
  int st = check(w);
  if (st) return st;
  if (!bytes || N < 0) return PF_ERR_INVALID_ARGUMENT;
  *bytes = workspace_bytes(w, N);
  return PF_OK;
}

static int common_args(const pf_qweight* w, int N, void* ws, size_t ws_bytes) {
  int st = check(w);
  if (st) return st;
  if (N < 0) return PF_ERR_INVALID_ARGUMENT;
  if (N == 0) return PF_OK;
  if (!ws || ws_bytes < workspace_bytes(w, N, false)) return PF_ERR_WORKSPACE;
  if (!aligned(ws, 256)) return PF_ERR_ALIGNMENT;
  return PF_OK;
}

// Most members one pf_qlinear_group call passes to the streaming GEMV.
constexpr int kStreamMaxMembers = 1024;

// One streaming-GEMV pass (np <= 16 tokens) over `count` weights: one x'
// preparation launch for the distinct inputs (an input read by several
// weights of one format is prepared once), then one GEMV launch per format
// and scale mode (INT3 and INT2 group-128 share one), up to kTmaMaxJobs
// weights each.  Workspace: counters, then
// x' records, then partial sums (at most tma_member_bytes per weight).
static int stream_pass(int count, const pf_qweight* const* ws, const void* const* xs, int x_dtype, int np,
                       const float* const* biases, float* const* ys, size_t t0, void* workspace, cudaStream_t s,
                       const pf_peers* peers = nullptr, const size_t* y_offsets = nullptr,
                       const int* m_full = nullptr) {
  if (count < 1 || count > kStreamMaxMembers) return PF_ERR_INVALID_ARGUMENT;
  const size_t xsz = dtype_size(x_dtype);
  char* cursor = static_cast<char*>(workspace) + kCounterBytes;
  XPrepJob xj[kXPrepMaxJobs];
  int nxj = 0;
  const unsigned char* xq_of[kStreamMaxMembers];
  cudaError_t e = cudaSuccess;
  for (int i = 0; i < count; ++i) {
    const pf_qweight* w = ws[i];
    const void* x = static_cast<const char*>(xs[i]) + t0 * w->K * xsz;
    const int8_t* sg = w->had_block ? w->had_signs : nullptr;
    int found = -1;
    for (int k = 0; k < nxj; ++k)
      if (xj[k].x == x && xj[k].fmt == w->format && xj[k].K == w->K && xj[k].had_block == w->had_block &&
          xj[k].signs == sg)
        found = k;
    if (found < 0) {
      if (nxj == kXPrepMaxJobs) {  // a full preparation launch
        int st = launch_xprep_frag(xj, nxj, np, x_dtype, s, &e);
        if (st == PF_ERR_CUDA) return cuda_status(e);
        if (st) return st;
        nxj = 0;
      }
      XPrepJob& p = xj[nxj];
      memset(&p, 0, sizeof(p));
      p.x = x;
      p.signs = sg;
      p.xq = reinterpret_cast<unsigned char*>(cursor);
      p.had_block = w->had_block;
      p.had_rscale = w->had_block ? 1.f / sqrtf((float)w->had_block) : 1.f;
      p.K = w->K;
      p.fmt = w->format;
      cursor += tma_xq_bytes(w, np);
      found = nxj++;
    }
    xq_of[i] = xj[found].xq;
  }
  if (nxj) {
    int st = launch_xprep_frag(xj, nxj, np, x_dtype, s, &e);
    if (st == PF_ERR_CUDA) return cuda_status(e);
    if (st) return st;
  }
  // GEMV launches: members of one format and scale mode together, and the
  // group-128 INT3 and INT2 members in one launch
  auto joins = [&](int f, int g) {
    const bool pair = (f == PF_FMT_INT3_G128 || f == PF_FMT_INT2_G128) && (g == PF_FMT_INT3_G128 || g == PF_FMT_INT2_G128);
    return f == g || pair;
  };
  bool done[kStreamMaxMembers] = {false};
  char* part = cursor;
  for (int i0 = 0; i0 < count; ++i0) {
    if (done[i0]) continue;
    TmaWeight tw[kTmaMaxJobs];
    TmaIO io[kTmaMaxJobs];
    int n = 0, tiles = 0;
    char* part0 = part;
    for (int i = i0; i < count && n < kTmaMaxJobs; ++i) {
      if (done[i] || !joins(ws[i]->format, ws[i0]->format) || (ws[i]->scales != nullptr) != (ws[i0]->scales != nullptr))
        continue;
      const TmaWeight t = tma_weight(ws[i]);
      if (n > 0 && (size_t)(tiles + tma_tiles(t)) > kWsDoneSlot) continue;
      tw[n] = t;
      io[n].x = nullptr;
      io[n].bias = biases ? biases[i] : nullptr;
      io[n].y = ys ? ys[i] + t0 * ws[i]->M : nullptr;
      io[n].xq = xq_of[i];
      if (peers) {  // tokens t0.. of linear i's gathered y, this rank's rows
        io[n].yoff = y_offsets[i] + t0 * (size_t)m_full[i] * sizeof(float);
        io[n].m_full = m_full[i];
        io[n].row0 = peers->rank * ws[i]->M;
      } else {
        io[n].yoff = 0;
        io[n].m_full = 0;
        io[n].row0 = 0;
      }
      tiles += tma_tiles(t);
      part += tma_partial_bytes(t, np);
      done[i] = true;
      ++n;
    }
    int st = launch_gemv_tma(tw, io, n, np, workspace, part0, peers, s, &e);
    if (st == PF_ERR_CUDA) return cuda_status(e);
    if (st) return st;
  }
  return PF_OK;
}

// One pass (N <= 16 tokens) of pf_qlinear.
static int qlinear_pass(const pf_qweight* w, const HadPlan& plan, const void* x, int x_dtype, int np,
                        const float* bias, float* y, void* ws, cudaStream_t s) {
  if (use_tma(w) && x_tma_aligned(x, x_dtype)) {
    const void* xs[1] = {x};
    const float* bs[1] = {bias};
    float* yv[1] = {y};
    return stream_pass(1, &w, xs, x_dtype, np, bs, yv, 0, ws, s);
  }
  int st = do_prepare(w, plan, x, x_dtype, np, ws, s);
  if (st) return st;
  return do_run(w, np, bias, y, ws, s);
}

// Tokens [0, N) through the tensor-core GEMM, kGemmChunk at a time.
static int qlinear_gemm(const pf_qweight* w, const HadPlan& plan, const void* x, int x_dtype, int N,
                        const float* bias, float* y, void* ws, bool with_partials, cudaStream_t s) {
  const int K = w->K, Kp = ((K + 127) / 128) * 128;
  const size_t xs = dtype_size(x_dtype);
  char* base = static_cast<char*>(ws) + kCounterBytes;
  const int cmax = N < kGemmChunk ? N : kGemmChunk;
  float* xplain = reinterpret_cast<float*>(base);
  __half* x16 = reinterpret_cast<__half*>(base + round_up((size_t)cmax * Kp * sizeof(float), 256));
  float* tsc = reinterpret_cast<float*>(reinterpret_cast<char*>(x16) + round_up((size_t)cmax * K * 2, 256));
  // no room for partial tiles: the non-persistent GEMM kernel runs
  float* partials =
      with_partials ? reinterpret_cast<float*>(reinterpret_cast<char*>(x16) + gemm_x16_bytes(cmax, K)) : nullptr;
  // rotation blocks that tile K: x' straight from x in the GEMM's own prep
  const bool direct = plan.ncasc == 0 && (plan.block == 0 || plan.rot_end == K) && K <= kGemmPrepMaxK;
  const bool pol = w->format == PF_FMT_POLAR_RECURSIVE;
  for (int t0 = 0; t0 < N; t0 += kGemmChunk) {
    const int nc = N - t0 < kGemmChunk ? N - t0 : kGemmChunk;
    if (direct) {
      GemmIn g;
      memset(&g, 0, sizeof(g));
      g.fmt = w->format;
      g.codes = w->codes;
      g.scales = pol ? nullptr : static_cast<const __half*>(w->scales);
      g.mins = static_cast<const __half*>(w->mins);
      g.r_scale = (float)w->tensor_scale;
      g.angles = pol ? static_cast<const float*>(w->scales) : nullptr;
      g.M = w->M;
      g.K = K;
      g.Kp = Kp;
      g.N = nc;
      g.row_words = row_words_of(w->format, K);
      g.xplain = nullptr;
      g.x = static_cast<const char*>(x) + (size_t)t0 * K * xs;
      g.x_dtype = x_dtype;
      g.signs = w->had_signs;
      g.block = plan.block;
      g.rscale = plan.block > 1 ? 1.f / sqrtf((float)plan.block) : 1.f;
      g.x16 = x16;
      g.tok_scale = tsc;
      g.bias = bias;
      g.y = y + (size_t)t0 * w->M;
      g.status = static_cast<unsigned*>(ws) + kWsStatusSlot;
      g.counters = static_cast<unsigned*>(ws);
      g.partials = partials;
      int st = cuda_status(launch_gemm(g, s));
      if (st) return st;
      continue;
    }
    PrepArgs pa;
    memset(&pa, 0, sizeof(pa));
    pa.x = static_cast<const char*>(x) + (size_t)t0 * K * xs;
    pa.x_dtype = x_dtype;
    pa.N = nc;
    pa.K = K;
    pa.Kp = Kp;
    pa.plan = plan;
    pa.signs = w->had_signs;
    pa.fmt = w->format;
    pa.M = w->M;
    pa.mode = 1;
    pa.slots = nc;
    pa.xplain = xplain;
    int st = cuda_status(launch_prep(pa, s));
    if (st) return st;
    GemmIn g;
    memset(&g, 0, sizeof(g));
    g.fmt = w->format;
    g.codes = w->codes;
    g.scales = pol ? nullptr : static_cast<const __half*>(w->scales);
    g.mins = static_cast<const __half*>(w->mins);
    g.r_scale = (float)w->tensor_scale;
    g.angles = pol ? static_cast<const float*>(w->scales) : nullptr;
    g.M = w->M;
    g.K = K;
    g.Kp = Kp;
    g.N = nc;
    g.row_words = row_words_of(w->format, K);
    g.xplain = xplain;
    g.x16 = x16;
    g.tok_scale = tsc;
    g.bias = bias;
    g.y = y + (size_t)t0 * w->M;
    g.status = static_cast<unsigned*>(ws) + kWsStatusSlot;
    g.counters = static_cast<unsigned*>(ws);
    g.partials = partials;
    st = cuda_status(launch_gemm(g, s));
    if (st) return st;
  }
  return PF_OK;
}

int pf_qlinear(const pf_qweight* w, const void* x, int x_dtype, int N, const float* bias, float* y,
               void* workspace, size_t ws_bytes, void* stream) {
  int st = common_args(w, N, workspace, ws_bytes);
  if (st || N == 0) return st;
  if (x_dtype < PF_DTYPE_F32 || x_dtype > PF_DTYPE_BF16) return PF_ERR_INVALID_ARGUMENT;
  if (!x || !y) return PF_ERR_INVALID_ARGUMENT;
  if (!aligned(x, dtype_size(x_dtype)) || !aligned(y, 4) || (bias && !aligned(bias, 4))) return PF_ERR_ALIGNMENT;
  HadPlan plan;
  st = make_plan(w->K, w->had_block, &plan);
  if (st) return st;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (use_e8_lut(w, N, plan, x, x_dtype)) {
    cudaError_t e = cudaSuccess;
    const E8In in = e8_in(w, plan, x, x_dtype, bias, y);
    st = launch_e8_lut(&in, 1, workspace, s, &e);
    return st == PF_ERR_CUDA ? cuda_status(e) : st;
  }
  if (use_polar_lut(w, N, plan, x, x_dtype)) {
    cudaError_t e = cudaSuccess;
    const Polar8In in = polar8_in(w, plan, x, x_dtype, bias, y);
    st = launch_polar8_lut(&in, 1, workspace, s, &e);
    return st == PF_ERR_CUDA ? cuda_status(e) : st;
  }
  if (use_gemm(w, N)) {
    const bool full = ws_bytes >= workspace_bytes(w, N);
    if (full || w->format != PF_FMT_POLAR_RECURSIVE)
      return qlinear_gemm(w, plan, x, x_dtype, N, bias, y, workspace, full, s);
  }
  const size_t xs = dtype_size(x_dtype);
  for (int t0 = 0; t0 < N; t0 += kMaxGemvTokens) {
    int np = N - t0 < kMaxGemvTokens ? N - t0 : kMaxGemvTokens;
    st = qlinear_pass(w, plan, static_cast<const char*>(x) + (size_t)t0 * w->K * xs, x_dtype, np, bias,
                      y + (size_t)t0 * w->M, workspace, s);
    if (st) return st;
  }
  return PF_OK;
}

// ---- grouped linears: every member that takes the streaming GEMV (any INT
// format it serves) shares one x' preparation launch and one GEMV launch per
// format, up to kTmaMaxJobs members each.
static bool group_streams(int count, const pf_qweight* const* ws) {
  if (count < 1 || count > kStreamMaxMembers) return false;
  for (int i = 0; i < count; ++i)
    if (!use_tma(ws[i])) return false;
  return true;
}

// Batch-1 groups of E8 or block-8 polar weights that read one x share a
// table-GEMV launch (tables depend on x only), four weights at a time.
static int group_lut_kind(int count, const pf_qweight* const* ws, int N) {
  if (count < 2 || N != 1) return 0;
  const int f = ws[0]->format;
  const bool e8 = f == PF_FMT_E8_RVQ2_G128 && e8_lut_enabled();
  const bool pol = f == PF_FMT_POLAR_RECURSIVE && ws[0]->params[0] == 8 && polar_lut_enabled();
  if (!e8 && !pol) return 0;
  for (int i = 1; i < count; ++i) {
    const pf_qweight* w = ws[i];
    if (w->format != f || w->K != ws[0]->K || w->had_block != ws[0]->had_block || w->had_signs != ws[0]->had_signs)
      return 0;
    if (pol && (memcmp(w->params, ws[0]->params, 9 * sizeof(int32_t)) != 0 || w->scales != ws[0]->scales)) return 0;
  }
  return e8 ? 1 : 2;
}

static size_t group_bytes(int count, const pf_qweight* const* ws, int N) {
  size_t b = 0;
  for (int i = 0; i < count; ++i) {
    size_t t = workspace_bytes(ws[i], N);
    if (t > b) b = t;
  }
  if (const int kind = group_lut_kind(count, ws, N)) {
    for (int c0 = 0; c0 < count; c0 += kLutGroupJobs) {
      size_t t = kCounterBytes;
      for (int i = c0; i < count && i < c0 + kLutGroupJobs; ++i)
        t += kind == 1 ? e8_lut_partial_bytes(ws[i]->M, ws[i]->K) : polar8_lut_partial_bytes(ws[i]->M, ws[i]->K);
      if (t > b) b = t;
    }
  }
  if (N <= kMaxGemvTokens && group_streams(count, ws)) {
    const int np = tokens_per_pass(N < 1 ? 1 : N);
    size_t t = kCounterBytes;
    for (int i = 0; i < count; ++i) t += tma_member_bytes(ws[i], np);
    if (t > b) b = t;
  }
  return b;
}

int pf_qlinear_group_workspace_size(int count, const pf_qweight* const* ws, int N, size_t* bytes) {
  if (count < 1 || !ws || !bytes || N < 0) return PF_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < count; ++i) {
    int st = check(ws[i]);
    if (st) return st;
  }
  *bytes = group_bytes(count, ws, N);
  return PF_OK;
}

int pf_qlinear_group(int count, const pf_qweight* const* ws, const void* const* xs, int x_dtype, int N,
                     const float* const* biases, float* const* ys, void* workspace, size_t ws_bytes, void* stream) {
  if (count < 1 || !ws || !xs || !ys || N < 0) return PF_ERR_INVALID_ARGUMENT;
  if (x_dtype < PF_DTYPE_F32 || x_dtype > PF_DTYPE_BF16) return PF_ERR_INVALID_ARGUMENT;
  for (int i = 0; i < count; ++i) {
    int st = check(ws[i]);
    if (st) return st;
    if (!xs[i] || !ys[i]) return PF_ERR_INVALID_ARGUMENT;
    const float* b = biases ? biases[i] : nullptr;
    if (!aligned(xs[i], dtype_size(x_dtype)) || !aligned(ys[i], 4) || (b && !aligned(b, 4)))
      return PF_ERR_ALIGNMENT;
  }
  if (N == 0) return PF_OK;
  if (!workspace || ws_bytes < group_bytes(count, ws, N)) return PF_ERR_WORKSPACE;
  if (!aligned(workspace, 256)) return PF_ERR_ALIGNMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  if (const int kind = group_lut_kind(count, ws, N)) {
    // every member eligible and reading the same x: table-GEMV launches of up to four
    HadPlan plan;
    bool ok = make_plan(ws[0]->K, ws[0]->had_block, &plan) == PF_OK &&
              (kind == 1 ? use_e8_lut(ws[0], 1, plan, xs[0], x_dtype) : use_polar_lut(ws[0], 1, plan, xs[0], x_dtype));
    for (int i = 1; i < count && ok; ++i) ok = xs[i] == xs[0];
    for (int c0 = 0; ok && c0 < count; c0 += kLutGroupJobs) {
      const int n = count - c0 < kLutGroupJobs ? count - c0 : kLutGroupJobs;
      cudaError_t e = cudaSuccess;
      int st;
      if (kind == 1) {
        E8In in[kLutGroupJobs];
        for (int k = 0; k < n; ++k)
          in[k] = e8_in(ws[c0 + k], plan, xs[0], x_dtype, biases ? biases[c0 + k] : nullptr, ys[c0 + k]);
        st = launch_e8_lut(in, n, workspace, s, &e);
      } else {
        Polar8In in[kLutGroupJobs];
        for (int k = 0; k < n; ++k)
          in[k] = polar8_in(ws[c0 + k], plan, xs[0], x_dtype, biases ? biases[c0 + k] : nullptr, ys[c0 + k]);
        st = launch_polar8_lut(in, n, workspace, s, &e);
      }
      if (st == PF_ERR_CUDA) return cuda_status(e);
      if (st) return st;
    }
    if (ok) return PF_OK;
  }
  bool grouped = N <= kMaxGemvTokens && group_streams(count, ws);
  for (int i = 0; i < count && grouped; ++i) grouped = x_tma_aligned(xs[i], x_dtype);
  if (!grouped) {
    for (int i = 0; i < count; ++i) {
      int st = pf_qlinear(ws[i], xs[i], x_dtype, N, biases ? biases[i] : nullptr, ys[i], workspace, ws_bytes,
                          stream);
      if (st) return st;
    }
    return PF_OK;
  }
  for (int t0 = 0; t0 < N; t0 += kMaxGemvTokens) {
    const int np = N - t0 < kMaxGemvTokens ? N - t0 : kMaxGemvTokens;
    int st = stream_pass(count, ws, xs, x_dtype, np, biases, ys, (size_t)t0, workspace, s);
    if (st) return st;
  }
  return PF_OK;
}

int pf_qlinear_group_gather(int count, const pf_qweight* const* ws, const void* const* xs, int x_dtype, int N,
                            const float* const* biases, const size_t* y_offsets, const int* m_full,
                            const pf_peers* peers, void* workspace, size_t ws_bytes, void* stream) {
  if (count < 1 || !ws || !xs || !y_offsets || !m_full || !peers || N < 0) return PF_ERR_INVALID_ARGUMENT;
  if (x_dtype < PF_DTYPE_F32 || x_dtype > PF_DTYPE_BF16) return PF_ERR_INVALID_ARGUMENT;
  if (peers->world < 1 || peers->world > kMaxPeers || peers->rank < 0 || peers->rank >= peers->world)
    return PF_ERR_INVALID_ARGUMENT;
  for (int p = 0; p < peers->world; ++p)
    if (!peers->bases[p] || !aligned(peers->bases[p], 256)) return PF_ERR_ALIGNMENT;
  for (int i = 0; i < count; ++i) {
    int st = check(ws[i]);
    if (st) return st;
    if (!xs[i]) return PF_ERR_INVALID_ARGUMENT;
    const float* b = biases ? biases[i] : nullptr;
    if ((b && !aligned(b, 4)) || !aligned(xs[i], dtype_size(x_dtype))) return PF_ERR_ALIGNMENT;
    if ((long long)m_full[i] != (long long)peers->world * ws[i]->M) return PF_ERR_SHAPE;
    if (y_offsets[i] < kPeerHeader || y_offsets[i] % 16) return PF_ERR_ALIGNMENT;
    if (y_offsets[i] + (size_t)N * m_full[i] * sizeof(float) > peers->bytes) return PF_ERR_SHAPE;
  }
  if (N == 0) return PF_OK;
  if (N > kMaxGemvTokens || !group_streams(count, ws)) return PF_ERR_UNSUPPORTED;
  for (int i = 0; i < count; ++i)
    if (!x_tma_aligned(xs[i], x_dtype)) return PF_ERR_UNSUPPORTED;
  if (!workspace || ws_bytes < group_bytes(count, ws, N)) return PF_ERR_WORKSPACE;
  if (!aligned(workspace, 256)) return PF_ERR_ALIGNMENT;
  return stream_pass(count, ws, xs, x_dtype, N, biases, nullptr, 0, workspace, static_cast<cudaStream_t>(stream),
                     peers, y_offsets, m_full);
}

int pf_dequant(const pf_qweight* w, float* W_out, int inverse_rwht, void* stream) {
  int st = check(w);
  if (st) return st;
  if (!W_out) return PF_ERR_INVALID_ARGUMENT;
  DequantArgs a;
  memset(&a, 0, sizeof(a));
  a.fmt = w->format;
  a.codes = w->codes;
  a.scales = w->scales;
  a.mins = static_cast<const __half*>(w->mins);
  a.tensor_scale = (float)w->tensor_scale;
  a.M = w->M;
  a.K = w->K;
  a.row_words = row_words_of(w->format, w->K);
  a.W = W_out;
  if (w->format == PF_FMT_POLAR_RECURSIVE || w->format == PF_FMT_POLAR2D) {
    PolarShape ps;
    polar_shape(w, &ps);
    a.d = ps.d;
    a.tb = ps.tb;
    a.row_bytes = ps.row_bytes;
    memcpy(a.alloc, ps.alloc, sizeof(a.alloc));
    a.r_scale = (float)w->tensor_scale;
    a.zero_rule = w->format == PF_FMT_POLAR2D;
    a.angles = w->format == PF_FMT_POLAR_RECURSIVE ? static_cast<const float*>(w->scales) : nullptr;
  }
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  st = cuda_status(launch_dequant(a, s));
  if (st) return st;
  if (inverse_rwht && w->had_block) {
    HadPlan plan;
    make_plan(w->K, w->had_block, &plan);
    for (int r0 = 0; r0 < w->M; r0 += 65535) {
      int rows = w->M - r0 < 65535 ? w->M - r0 : 65535;
      float* p = W_out + (size_t)r0 * w->K;
      st = cuda_status(launch_rwht_rows(p, p, rows, w->K, plan, w->had_signs, 1, s));
      if (st) return st;
    }
  }
  return PF_OK;
}

int pf_unpack_codes(const pf_qweight* w, uint8_t* codes_out, void* stream) {
  int st = check(w);
  if (st) return st;
  if (!codes_out) return PF_ERR_INVALID_ARGUMENT;
  if (!is_int_format(w->format) && w->format != PF_FMT_E8_RVQ2_G128) return PF_ERR_UNSUPPORTED;
  DequantArgs a;
  memset(&a, 0, sizeof(a));
  a.fmt = w->format;
  a.codes = w->codes;
  a.scales = w->scales;
  a.M = w->M;
  a.K = w->K;
  a.row_words = row_words_of(w->format, w->K);
  a.codes_out = codes_out;
  return cuda_status(launch_unpack(a, static_cast<cudaStream_t>(stream)));
}

int pf_rwht(const float* in, float* out, int rows, int K, int block, const int8_t* signs, int inverse,
            void* stream) {
  if (!in || !out || !signs || rows < 0 || K <= 0) return PF_ERR_INVALID_ARGUMENT;
  HadPlan plan;
  int st = make_plan(K, block, &plan);
  if (st) return st;
  if (block == 0) return PF_ERR_INVALID_ARGUMENT;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  for (int r0 = 0; r0 < rows; r0 += 65535) {
    int n = rows - r0 < 65535 ? rows - r0 : 65535;
    st = cuda_status(launch_rwht_rows(in + (size_t)r0 * K, out + (size_t)r0 * K, n, K, plan, signs, inverse, s));
    if (st) return st;
  }
  return PF_OK;
}

static int native_gemv(int fmt, const float* x, const uint8_t* packed, const float* scales, int N, int M,
                       int K, float* y, void* ws, size_t ws_bytes, void* stream) {
  if (!scales) return PF_ERR_INVALID_ARGUMENT;
  pf_qweight w;
  memset(&w, 0, sizeof(w));
  w.format = fmt;
  w.M = M;
  w.K = K;
  w.codes = packed;
  w.scales = scales;
  return pf_qlinear(&w, x, PF_DTYPE_F32, N, nullptr, y, ws, ws_bytes, stream);
}

int pf_native_gemv_int4(const float* x, const uint8_t* packed, const float* scales, int M, int K, float* y,
                        void* ws, size_t ws_bytes, void* stream) {
  return native_gemv(PF_FMT_INT4, x, packed, scales, 1, M, K, y, ws, ws_bytes, stream);
}

int pf_native_gemv_int2(const float* x, const uint8_t* packed, const float* scales, int M, int K, float* y,
                        void* ws, size_t ws_bytes, void* stream) {
  return native_gemv(PF_FMT_INT2, x, packed, scales, 1, M, K, y, ws, ws_bytes, stream);
}

int pf_native_gemm_int4(const float* X, const uint8_t* packed, const float* scales, int N, int M, int K,
                        float* Y, void* ws, size_t ws_bytes, void* stream) {
  return native_gemv(PF_FMT_INT4, X, packed, scales, N, M, K, Y, ws, ws_bytes, stream);
}

}  // extern "C"
