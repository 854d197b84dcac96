// C ABI entry points: argument validation on the host, then the launch
// sequence (x-prep, GEMV) on the caller's stream.  Nothing here allocates.
#include <stdlib.h>
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

int row_words_of(int fmt, int K) {
  switch (fmt) {
    case PF_FMT_INT4_G128: return (K / 128) * 16;
    case PF_FMT_INT3_G128: return (K / 128) * 13;
    case PF_FMT_INT2_G128: return (K / 128) * 8;
    case PF_FMT_INT4: return K / 8;
    case PF_FMT_INT3: return 3 * K / 32;
    case PF_FMT_INT2: return K / 16;
    default: return 0;
  }
}

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
      return polar_shape(w, &ps);
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

// TMA-pipelined GEMV for INT4/INT3/INT2 group-128 and the INT4/INT2 reference
// streams when K % 512 == 0; chosen from format and K only, so a prepare and
// every run that shares it take the same path.  PF_GEMV_PATH=ldg forces the
// register-prefetch GEMV.
bool use_tma(const pf_qweight* w) {
  static int mode = -1;
  if (mode < 0) {
    const char* e = getenv("PF_GEMV_PATH");
    mode = (e && strcmp(e, "ldg") == 0) ? 0 : 1;
  }
  if (!mode) return false;
  return tma_eligible(w->format, 1, w->K, reinterpret_cast<const void*>(16));
}

// The TMA GEMV decodes codes to exact subnormal fp16 (q * 2^(p-24)).
int tma_subnormal() { return 1; }

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

size_t tma_partials_bytes(const pf_qweight* w, int np) {
  const int rows = tma_block_rows();
  const int spb = (w->K / 128) / tma_stage_groups(w->format);
  const int n_units = ((w->M + rows - 1) / rows) * spb;
  return round_up((size_t)2 * tma_grid(w->format, nt_of(np), n_units) * rows * np * sizeof(float), 256);
}

size_t xprep_bytes(const pf_qweight* w, int np) {
  size_t Gp = (size_t)(w->K + 127) / 128;
  if (use_tma(w)) return round_up(Gp * tma_record_bytes(np, nt_of(np)), 256);
  if (is_int_format(w->format)) {
    int NT = nt_of(np);
    return round_up((size_t)NT * Gp * 2048, 256) + round_up(Gp * 8 * NT * sizeof(float), 256);
  }
  return round_up((size_t)np * Gp * 128 * sizeof(float), 256);
}

size_t pass_bytes(const pf_qweight* w, int np) {
  size_t b = kCounterBytes + xprep_bytes(w, np);
  if (use_tma(w)) return b + tma_partials_bytes(w, np);
  if (is_int_format(w->format)) {
    IntPlan p = plan_int(w, np);
    if (p.n_chunks > 1) b += round_up((size_t)p.n_chunks * np * w->M * sizeof(float), 256);
  }
  return b;
}

size_t workspace_bytes(const pf_qweight* w, int N) {
  if (N < 1) N = 1;
  size_t b = pass_bytes(w, tokens_per_pass(N));
  int tail = N % kMaxGemvTokens;
  if (N > kMaxGemvTokens && tail) {
    size_t t = pass_bytes(w, tail);
    if (t > b) b = t;
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
  if (use_tma(w)) {
    Prep2Args p2;
    memset(&p2, 0, sizeof(p2));
    p2.x = x;
    p2.x_dtype = x_dtype;
    p2.N = N;
    p2.NT = nt_of(N);
    p2.K = w->K;
    p2.G = Gp;
    p2.plan = plan;
    p2.signs = w->had_signs;
    p2.fmt = w->format;
    p2.subnormal = tma_subnormal();
    p2.rec = reinterpret_cast<unsigned char*>(base);
    return cuda_status(launch_prep2(p2, s));
  }
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
  if (use_tma(w)) {
    if (!tma_eligible(w->format, M, K, w->codes)) return PF_ERR_ALIGNMENT;
    TmaArgs ta;
    memset(&ta, 0, sizeof(ta));
    ta.codes = w->codes;
    ta.scales = w->scales;
    ta.mins = static_cast<const __half*>(w->mins);
    ta.tensor_scale = (float)w->tensor_scale;
    ta.M = M;
    ta.K = K;
    ta.N = N;
    ta.NT = nt_of(N);
    ta.G = Gp;
    ta.row_words = row_words_of(w->format, K);
    ta.rows = tma_block_rows();
    ta.n_rb = (M + ta.rows - 1) / ta.rows;
    ta.spb = Gp / tma_stage_groups(w->format);
    ta.n_units = ta.n_rb * ta.spb;
    ta.rec = reinterpret_cast<const unsigned char*>(base);
    ta.rec_bytes = (int)tma_record_bytes(N, ta.NT);
    ta.bias = bias;
    ta.y = y;
    ta.partials = reinterpret_cast<float*>(base + xprep_bytes(w, N));
    ta.counters = static_cast<unsigned*>(ws);
    int smode = is_group_int_format(w->format) ? kScaleGroup : (w->scales ? kScaleRow : kScaleTensor);
    return cuda_status(launch_gemv_tma(w->format, ta, smode, tma_subnormal(), s));
  }
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
  }
  return cuda_status(launch_gemv_cc(ca, s));
}

}  // namespace

extern "C" {

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
  if (!ws || ws_bytes < workspace_bytes(w, N)) return PF_ERR_WORKSPACE;
  if (!aligned(ws, 256)) return PF_ERR_ALIGNMENT;
  return PF_OK;
}

int pf_qlinear_prepare(const pf_qweight* w, const void* x, int x_dtype, int N, void* workspace,
                       size_t ws_bytes, void* stream) {
  int st = common_args(w, N, workspace, ws_bytes);
  if (st || N == 0) return st;
  if (N > kMaxGemvTokens) return PF_ERR_SHAPE;
  if (x_dtype < PF_DTYPE_F32 || x_dtype > PF_DTYPE_BF16) return PF_ERR_INVALID_ARGUMENT;
  if (!x) return PF_ERR_INVALID_ARGUMENT;
  if (!aligned(x, dtype_size(x_dtype))) return PF_ERR_ALIGNMENT;
  HadPlan plan;
  st = make_plan(w->K, w->had_block, &plan);
  if (st) return st;
  return do_prepare(w, plan, x, x_dtype, N, workspace, static_cast<cudaStream_t>(stream));
}

int pf_qlinear_run(const pf_qweight* w, int N, const float* bias, float* y, void* workspace, size_t ws_bytes,
                   void* stream) {
  int st = common_args(w, N, workspace, ws_bytes);
  if (st || N == 0) return st;
  if (N > kMaxGemvTokens) return PF_ERR_SHAPE;
  if (!y) return PF_ERR_INVALID_ARGUMENT;
  if (!aligned(y, 4) || (bias && !aligned(bias, 4))) return PF_ERR_ALIGNMENT;
  return do_run(w, N, bias, y, workspace, static_cast<cudaStream_t>(stream));
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
  const size_t xs = dtype_size(x_dtype);
  for (int t0 = 0; t0 < N; t0 += kMaxGemvTokens) {
    int np = N - t0 < kMaxGemvTokens ? N - t0 : kMaxGemvTokens;
    st = do_prepare(w, plan, static_cast<const char*>(x) + (size_t)t0 * w->K * xs, x_dtype, np, workspace, s);
    if (st) return st;
    st = do_run(w, np, bias, y + (size_t)t0 * w->M, workspace, s);
    if (st) return st;
  }
  return PF_OK;
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
