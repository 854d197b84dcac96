// Streaming lookup-table GEMVs at batch 1 for the two codebook formats whose
// every weight vector is one of a few shapes:
//
//  * E8 RVQ2: row m, 8-vector v = s1(m, g) r[i1] + s2(m, g) r[i2] (r = the 240
//    E8 roots in generate_e8_roots order, g = v's 128-column group), so
//      y_m = sum_g [ s1 sum_{v in g} T[v][i1] + s2 sum_{v in g} T[v][i2] ]
//    with the table T[v][k] = <r_k, x'_v> (256 entries per vector, 240..255
//    zero).
//  * Recursive polar, block 8, allocation [3 | 2 2 2 2 | 1 1 | 1] (1.75 bpw):
//    a block is R = r r_scale times a tree of cos / sin factors (polar_quant.py
//    inverse_recursive: psi splits the radius between the two halves, phi_h
//    each half between its two pairs, theta_j each pair), so
//      <w, x'_v> = r (Q0[th0 th1 phi0 psi] + Q1[th2 th3 phi1 psi])
//    with Q_h = (cos | sin psi)(cos phi_h P_2h[th] + sin phi_h P_2h+1[th'])
//    and P_j[c] = cos th_j(c) x'_2j + sin th_j(c) x'_2j+1: two 64-entry
//    tables per vector (r_scale multiplies the row sums).
//
// The weight's block RWHT is folded into x (x' = forward RWHT of x).  A CTA
// builds the tables of a column stage in shared memory from x' (fp32), then
// a weight vector costs two table reads and two adds: no weight is decoded.
//
// A launch serves up to four weights ("jobs") that read the same x (q|k|v,
// gate|up): the tables depend on x and the stage only, so the jobs share
// them.  Work unit = (stage, block of 512 rows of one job), dealt to the CTAs
// stream-K style in stage-major order (every job's row blocks of a stage, then
// the next stage), so a CTA's consecutive units share a stage and its tables.  One 16-warp CTA per SM; every warp owns 32 rows of a unit and
// streams them through its own ring of shared-memory slots: lane 0 issues the
// TMA copy of the 32-row code tile (L2 evict-first), E8 lanes copy their row's
// group scales with cp.async, and the copies arrive on the slot's mbarrier.
// The first two slots are requested before the kernel waits for the
// preceding grid (weights and scales are never written by it); x' and the
// tables are built after the wait.  A lane reads a quarter of a row's stage
// codes; four lanes finish a row with two shuffles.  Each unit's row sums go
// to the workspace, and lut_combine_kernel (a programmatic dependent) adds a
// row's stage sums in stage order and writes y: deterministic.
// Every wait is bounded (%globaltimer); on expiry the kernel records
// PF_ERR_TIMEOUT in the workspace status word and finishes.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <string.h>

#include <mutex>

#include "common.cuh"
#include "decode.cuh"
#include "gemv.cuh"
#include "tma.cuh"

namespace pfb {

namespace {

constexpr int kLW = 16;                // warps per CTA
constexpr int kLT = kLW * 32;          // threads per CTA
constexpr int kLRowsW = 32;            // rows per warp and unit
constexpr int kLRows = kLW * kLRowsW;  // rows per unit
constexpr int kLMaxStages = 8;
constexpr int kLMaxTabs = 3;
constexpr int kLSmemBudget = 216 * 1024;

constexpr int kLutMaxJobs = 4;

struct LutJob {  // one weight of a launch
  const uint32_t* scales;  // E8: half2 [M][G] as words
  const float* bias;
  float* y;
  float* partials;  // [n_rb][spb][kLRows] stage row sums (spb > 1)
  float out_scale;  // polar r_scale (1 for E8)
  int M, n_rb, rb0;  // rows, row blocks, first row block of the launch's block list
};

struct LutArgs {
  LutJob job[kLutMaxJobs];
  const void* x;  // shared by the jobs
  const int8_t* signs;
  const float* angles;  // polar: learned angle table shared by the jobs, or nullptr
  unsigned* status;
  float had_rscale;
  int n_jobs, had_block, x_dtype, K, G, n_rb, spb, n_units, NS, XS;
};

__device__ __forceinline__ const LutJob& lut_job(const LutArgs& a, int j) {
  return j == 0 ? a.job[0] : j == 1 ? a.job[1] : j == 2 ? a.job[2] : a.job[3];
}
// Job holding row block `grb` of the launch's block list.
__device__ __forceinline__ int lut_job_of(const LutArgs& a, int grb) {
  int j = 0;
#pragma unroll
  for (int k = 1; k < kLutMaxJobs; ++k)
    if (k < a.n_jobs && grb >= a.job[k].rb0) j = k;
  return j;
}

// Table entry `idx` of the table row at shared address `row` (a constant
// offset from the lane's row block, which folds into the load's immediate).
__device__ __forceinline__ float tab_read(uint32_t row, uint32_t idx) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(row + (idx << 2)));
  return v;
}

// ---- E8 RVQ2 (256-column stages: 32 vectors, 64 code bytes per row)
struct E8Pol {
  static constexpr int kCols = 256;
  static constexpr uint32_t kRowCode = 64;                // code bytes per row and stage
  static constexpr uint32_t kCodes = kLRowsW * kRowCode;  // per warp tile
  static constexpr uint32_t kScales = kLRowsW * 8;        // two half2 group scales per row
  static constexpr int kTabFloats = (kCols / 8) * 256;
  static constexpr int kAuxFloat2 = 1;
  struct State {
    float root[8];  // root k = threadIdx.x mod 256 (zero past 239)
  };
  __device__ static void init(State& s, float2*, const LutArgs&) {
    const int k = threadIdx.x & 255;
    if (k < 240) {
      e8_root(k, s.root);
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) s.root[q] = 0.f;
    }
  }
  // T[v][k] = <r_k, x'[8v, 8v + 8)>: thread (k, half) fills 16 vectors
  __device__ static void build(const State& s, const LutArgs&, const float* xs, float* tab, const float2*) {
    const int k = threadIdx.x & 255, v0 = (threadIdx.x >> 8) * (kCols / 16);
    for (int v = v0; v < v0 + kCols / 16; ++v) {
      const float4 p0 = *reinterpret_cast<const float4*>(xs + 8 * v);
      const float4 p1 = *reinterpret_cast<const float4*>(xs + 8 * v + 4);
      float d = s.root[0] * p0.x;
      d = fmaf(s.root[1], p0.y, d);
      d = fmaf(s.root[2], p0.z, d);
      d = fmaf(s.root[3], p0.w, d);
      d = fmaf(s.root[4], p1.x, d);
      d = fmaf(s.root[5], p1.y, d);
      d = fmaf(s.root[6], p1.z, d);
      d = fmaf(s.root[7], p1.w, d);
      tab[v * 256 + k] = d;
    }
  }
  // the sum over the lane's 8 vectors (8q .. 8q + 7) of row r, scaled
  __device__ static float part(const unsigned char* tile, int r, int q, uint32_t tab) {
    const uint4 cw = lds<uint4>(tile + r * kRowCode + q * 16);
    const uint32_t sw = lds<uint32_t>(tile + kCodes + r * 8 + (q >> 1) * 4);
    const float2 s = __half22float2(*reinterpret_cast<const __half2*>(&sw));
    const uint32_t w[4] = {cw.x, cw.y, cw.z, cw.w};
    const uint32_t t0 = tab + (uint32_t)(8 * q) * 1024u;  // table rows 1 KB apart
    float A1 = 0.f, A2 = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j)
#pragma unroll
      for (int h = 0; h < 2; ++h) {
        // index bytes 2h (stage 1) and 2h + 1 (stage 2) of word j: vector 2j + h
        const uint32_t row = t0 + (uint32_t)(2 * j + h) * 1024u;
        A1 += tab_read(row, __byte_perm(w[j], 0u, 0x4440u + 2 * h));
        A2 += tab_read(row, __byte_perm(w[j], 0u, 0x4441u + 2 * h));
      }
    return fmaf(s.x, A1, s.y * A2);
  }
};

// ---- recursive polar, d = 8, allocation [3 | 2 2 2 2 | 1 1 | 1], 14-bit
// MSB-first codes (512-column stages: 64 vectors, 112 code bytes per row).
// Code bits (LSB first): psi 0, phi1 1, phi0 2, th3 3-4, th2 5-6, th1 7-8,
// th0 9-10, r 11-13.  Table of vector v: Q0 at [128 v, +64), Q1 at +64, entry
// (th_a << 4 | th_b << 2 | phi << 1 | psi).
struct Polar8Pol {
  static constexpr int kCols = 512;
  static constexpr uint32_t kRowCode = 112;
  static constexpr uint32_t kCodes = kLRowsW * kRowCode;
  static constexpr uint32_t kScales = 0;
  static constexpr int kTabFloats = (kCols / 8) * 128;
  static constexpr int kAuxFloat2 = 7 * kPolarTabPerCol;  // cos / sin of every angle column and code
  struct State {};
  __device__ static void init(State&, float2* aux, const LutArgs& a) {
    const int alloc[8] = {3, 2, 2, 2, 2, 1, 1, 1};
    polar_fill_tables(aux, 8, alloc, a.angles);
  }
  // thread t: vector t / 8, half (t / 4) % 2, entries 16 (t % 4) .. + 16
  __device__ static void build(const State&, const LutArgs& a, const float* xs, float* tab, const float2* cs) {
    const int v = threadIdx.x >> 3, h = (threadIdx.x >> 2) & 1, e0 = (threadIdx.x & 3) * 16;
    const float* xv = xs + 8 * v + 4 * h;  // pairs 2h and 2h + 1 of the vector
    float Pa[4], Pb[4];
#pragma unroll
    for (int c = 0; c < 4; ++c) {
      const float2 ta = cs[(2 * h) * kPolarTabPerCol + c], tb = cs[(2 * h + 1) * kPolarTabPerCol + c];
      Pa[c] = fmaf(ta.x, xv[0], ta.y * xv[1]);
      Pb[c] = fmaf(tb.x, xv[2], tb.y * xv[3]);
    }
    float* out = tab + v * 128 + h * 64;
#pragma unroll
    for (int i = 0; i < 16; ++i) {
      const int e = e0 + i;
      const int ta = e >> 4, tb = (e >> 2) & 3, ph = (e >> 1) & 1, ps = e & 1;
      const float2 fph = cs[(4 + h) * kPolarTabPerCol + ph], fps = cs[6 * kPolarTabPerCol + ps];
      const float half = fmaf(fph.x, Pa[ta], fph.y * Pb[tb]);
      out[e] = (h == 0 ? fps.x : fps.y) * half;
    }
  }
  __device__ static float part(const unsigned char* tile, int r, int q, uint32_t tab) {
    // the lane's 16 codes: 28 bytes at 28 q, big-endian bit order
    const unsigned char* p = tile + r * kRowCode + q * 28;
    uint32_t be[7];
#pragma unroll
    for (int i = 0; i < 7; ++i) be[i] = __byte_perm(lds<uint32_t>(p + 4 * i), 0u, 0x0123u);
    const uint32_t t0 = tab + (uint32_t)(16 * q) * 512u;  // vector tables 512 bytes apart
    float acc = 0.f;
#pragma unroll
    for (int k = 0; k < 16; ++k) {
      const int bit = 14 * k, w = bit >> 5, off = bit & 31;
      const uint32_t code =
          off <= 18 ? (be[w] >> (18 - off)) & 0x3FFFu : __funnelshift_l(be[w + 1], be[w], off) >> 18;
      const uint32_t i0 = ((code >> 5) & 0x3Cu) | ((code >> 1) & 2u) | (code & 1u);
      const uint32_t i1 = ((code >> 1) & 0x3Cu) | (code & 3u);
      const uint32_t row = t0 + (uint32_t)k * 512u;
      const float qs = tab_read(row, i0) + tab_read(row + 256u, i1);
      acc = fmaf((float)(code >> 11), qs, acc);
    }
    return acc;
  }
};

// x' of columns [col0, col0 + 32 E) restricted to [c0, c0 + cols), into
// xs[col - c0]: forward block RWHT of x (signs, Walsh-Hadamard butterflies in
// registers and across lanes, 1/sqrt(b)) for rotation blocks b <= 32 E.
template <int E>
__device__ __forceinline__ void xprime_chunk(const LutArgs& a, int col0, int c0, int cols, float* xs, int lane) {
  const int b = a.had_block;
  float v[E];
  const int base = col0 + E * lane;
  int s4[E / 4];
  const int* sp = reinterpret_cast<const int*>(a.signs + base);
#pragma unroll
  for (int q = 0; q < E / 4; ++q) s4[q] = __ldg(sp + q);
  if (a.x_dtype == PF_DTYPE_F32) {
    const float4* xp = reinterpret_cast<const float4*>(static_cast<const float*>(a.x) + base);
    float4 f[E / 4];
#pragma unroll
    for (int q = 0; q < E / 4; ++q) f[q] = __ldg(xp + q);
#pragma unroll
    for (int q = 0; q < E / 4; ++q) {
      v[4 * q] = f[q].x; v[4 * q + 1] = f[q].y; v[4 * q + 2] = f[q].z; v[4 * q + 3] = f[q].w;
    }
  } else {
    const uint2* xp = reinterpret_cast<const uint2*>(static_cast<const uint16_t*>(a.x) + base);
    uint2 r[E / 4];
#pragma unroll
    for (int q = 0; q < E / 4; ++q) r[q] = __ldg(xp + q);
#pragma unroll
    for (int q = 0; q < E / 4; ++q) {
      if (a.x_dtype == PF_DTYPE_F16) {
        const float2 f0 = __half22float2(*reinterpret_cast<const __half2*>(&r[q].x));
        const float2 f1 = __half22float2(*reinterpret_cast<const __half2*>(&r[q].y));
        v[4 * q] = f0.x; v[4 * q + 1] = f0.y; v[4 * q + 2] = f1.x; v[4 * q + 3] = f1.y;
      } else {  // bf16: the upper half of an fp32
        v[4 * q] = __uint_as_float(r[q].x << 16);
        v[4 * q + 1] = __uint_as_float(r[q].x & 0xFFFF0000u);
        v[4 * q + 2] = __uint_as_float(r[q].y << 16);
        v[4 * q + 3] = __uint_as_float(r[q].y & 0xFFFF0000u);
      }
    }
  }
#pragma unroll
  for (int q = 0; q < E / 4; ++q)
#pragma unroll
    for (int e = 0; e < 4; ++e)  // sign bit of the int8 column sign
      v[4 * q + e] = __uint_as_float(__float_as_uint(v[4 * q + e]) ^ (((uint32_t)s4[q] << (24 - 8 * e)) & 0x80000000u));
#pragma unroll
  for (int h = 1; h < E; h *= 2) {
    if (h < b) {
#pragma unroll
      for (int e = 0; e < E; ++e)
        if (!(e & h)) {
          const float u = v[e], w = v[e + h];
          v[e] = u + w;
          v[e + h] = u - w;
        }
    }
  }
#pragma unroll
  for (int m = 1; m < 32; m *= 2) {
    if (m * E < b) {
      const float sg = (lane & m) ? -1.f : 1.f;
#pragma unroll
      for (int e = 0; e < E; ++e) {
        const float p = __shfl_xor_sync(0xffffffffu, v[e], m);
        v[e] = fmaf(sg, v[e], p);
      }
    }
  }
#pragma unroll
  for (int e = 0; e < E; ++e) {
    const int col = base + e - c0;
    if (col >= 0 && col < cols) xs[col] = v[e] * a.had_rscale;
  }
}

// x' of the stage's columns [c0, c0 + cols) into xs[0, cols).
__device__ __forceinline__ void stage_xprime(const LutArgs& a, int c0, int cols, float* xs, int warp, int lane) {
  const int b = a.had_block;
  if (b == 0) {
    for (int i = threadIdx.x; i < cols; i += kLT) {
      float v;
      if (a.x_dtype == PF_DTYPE_F32)
        v = static_cast<const float*>(a.x)[c0 + i];
      else if (a.x_dtype == PF_DTYPE_F16)
        v = __half2float(static_cast<const __half*>(a.x)[c0 + i]);
      else
        v = __uint_as_float((uint32_t)static_cast<const uint16_t*>(a.x)[c0 + i] << 16);
      xs[i] = v;
    }
    return;
  }
  const int C = b > 256 ? 512 : (b > 128 ? 256 : 128);  // chunk columns: whole rotation blocks
  const int first = (c0 / C) * C;
  const int col0 = first + warp * C;
  if (col0 >= c0 + cols) return;
  if (C == 512)
    xprime_chunk<16>(a, col0, c0, cols, xs, lane);
  else if (C == 256)
    xprime_chunk<8>(a, col0, c0, cols, xs, lane);
  else
    xprime_chunk<4>(a, col0, c0, cols, xs, lane);
}

template <class Pol>
__global__ void __launch_bounds__(kLT, 1)
    lut_gemv_kernel(const __grid_constant__ CUtensorMap map0, const __grid_constant__ CUtensorMap map1,
                    const __grid_constant__ CUtensorMap map2, const __grid_constant__ CUtensorMap map3,
                    const __grid_constant__ LutArgs a) {
  constexpr uint32_t kSlot = Pol::kCodes + Pol::kScales;
  constexpr uint32_t kTab = Pol::kTabFloats * 4;
  asm volatile("griddepcontrol.launch_dependents;");
  if (threadIdx.x >= 32 && threadIdx.x < 32 + kLutMaxJobs) {
    const int k = threadIdx.x - 32;
    const CUtensorMap* m = k == 0 ? &map0 : k == 1 ? &map1 : k == 2 ? &map2 : &map3;
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
  }

  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ int abort_flag;
  __shared__ __align__(16) float xs[Pol::kCols];
  __shared__ float2 aux[Pol::kAuxFloat2];
  unsigned char* const base = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  const int NS = a.NS, XS = a.XS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* const tabs = reinterpret_cast<float*>(base);
  unsigned char* const ring = base + (size_t)XS * kTab + (size_t)warp * NS * kSlot;
  const uint32_t full0 = smem_u32(base + (size_t)XS * kTab + (size_t)kLW * NS * kSlot) + warp * NS * 8;

  typename Pol::State pst;
  Pol::init(pst, aux, a);
  if (threadIdx.x == 0) abort_flag = 0;
  if (lane == 0) {
    // arrivals per slot: the copy's expect_tx, plus every lane's cp.async of scales
    const uint32_t count = Pol::kScales ? 33u : 1u;
    for (int s = 0; s < NS; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(full0 + 8 * s), "r"(count));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  const unsigned U = (unsigned)a.n_units, P = gridDim.x, cta = blockIdx.x;
  const int u0 = (int)(cta * U / P), u1 = (int)((cta + 1) * U / P);  // U * P < 2^32 (host-checked)
  const int nunits = u1 - u0;
  if (nunits <= 0) return;

  // ---- load side: this warp's next unit to request (stage, block of the list)
  int fst = u0 / a.n_rb, fgrb = u0 - fst * a.n_rb;
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  const uint32_t ring_s = smem_u32(ring);
  auto request = [&](int slot) {
    const int fj = lut_job_of(a, fgrb);
    const LutJob& jb = lut_job(a, fj);
    const CUtensorMap* map = fj == 0 ? &map0 : fj == 1 ? &map1 : fj == 2 ? &map2 : &map3;
    const uint32_t sb = ring_s + slot * kSlot, bar = full0 + 8 * slot;
    const int row0 = (fgrb - jb.rb0) * kLRows + warp * kLRowsW;
    __syncwarp();
    if (lane == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_expect(bar, Pol::kCodes);
      tma_2d(sb, map, fst * (int)(Pol::kRowCode / 4), row0, bar, policy);
    }
    if constexpr (Pol::kScales > 0) {
      const int grow = row0 + lane;
      const bool ok = grow < jb.M;
      cp_async8(sb + Pol::kCodes + lane * 8, jb.scales + (ok ? (size_t)grow * a.G + 2 * fst : 0), ok ? 8u : 0u);
      cp_async_arrive(bar);
    }
    if (++fgrb == a.n_rb) {
      fgrb = 0;
      ++fst;
    }
  };
  int requested = 0;
  for (; requested < 2 && requested < NS && requested < nunits; ++requested) request(requested);

  // ---- tables of the CTA's stages ("runs"), XS resident, run r in slot r % XS
  const int st_first = u0 / a.n_rb;
  const int nruns = (u1 - 1) / a.n_rb - st_first + 1;
  int win_end = 0;
  auto build_window = [&](int r0) {
    const int r1 = r0 + XS < nruns ? r0 + XS : nruns;
    for (int r = r0; r < r1; ++r) {
      stage_xprime(a, (st_first + r) * Pol::kCols, Pol::kCols, xs, warp, lane);
      __syncthreads();
      Pol::build(pst, a, xs, tabs + (size_t)(r % XS) * Pol::kTabFloats, aux);
      __syncthreads();  // tables written, xs free for the next run
    }
    win_end = r1;
  };

  // x may be written by the preceding grid, and so may the workspace and y
  asm volatile("griddepcontrol.wait;" ::: "memory");
  build_window(0);
  for (; requested < NS && requested < nunits; ++requested) request(requested);

  const int r8 = lane >> 2, q = lane & 3;
  int st = st_first, grb = u0 - st_first * a.n_rb, run = 0, slot = 0;
  uint32_t phase = 0;
  bool live = true;
  for (int it = 0; it < nunits; ++it) {
    if (run >= win_end) {  // same decision in every warp of the CTA
      __syncthreads();
      build_window(win_end);
    }
    if (live && !mbar_wait(full0 + 8 * slot, phase, &abort_flag)) {
      live = false;
      if (lane == 0) {
        abort_flag = 1;
        atomicExch(a.status, (unsigned)PF_ERR_TIMEOUT);
      }
    }
    if (live) {
      const unsigned char* tile = ring + slot * kSlot;
      const uint32_t tab = smem_u32(tabs) + (uint32_t)(run % XS) * kTab;
      float rs[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        float v = Pol::part(tile, 8 * p + r8, q, tab);
        v += __shfl_xor_sync(0xffffffffu, v, 1);
        v += __shfl_xor_sync(0xffffffffu, v, 2);
        rs[p] = v;
      }
      if (q == 0) {
        const LutJob& jb = lut_job(a, lut_job_of(a, grb));
        const int rb = grb - jb.rb0;
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const int rl = warp * kLRowsW + 8 * p + r8;
          const int row = rb * kLRows + rl;
          const float v = rs[p] * jb.out_scale;
          if (a.spb == 1) {
            if (row < jb.M) jb.y[row] = v + (jb.bias ? jb.bias[row] : 0.f);
          } else {
            __stcg(jb.partials + ((size_t)rb * a.spb + st) * kLRows + rl, v);
          }
        }
      }
    }
    if (live && requested < nunits) {  // refill the slot just consumed
      request(slot);
      ++requested;
    }
    if (++slot == NS) {
      slot = 0;
      phase ^= 1u;
    }
    if (++grb == a.n_rb) {
      grb = 0;
      ++st;
      ++run;
    }
  }
  if (!live && lane == 0) {
    // after a timeout: bounded waits on this warp's tiles that may still be in flight
    volatile int keep_waiting = 0;
    for (int k = requested > NS ? requested - NS : 0; k < requested; ++k)
      mbar_wait(full0 + 8 * (k % NS), (k / NS) & 1, &keep_waiting);
  }
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// y = the sum of a row's stage sums in stage order (+ bias).  Block b of the
// grid covers 256 rows of one job (jobs start on a new block).
__global__ void __launch_bounds__(256) lut_combine_kernel(const __grid_constant__ LutArgs a) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  int blk = blockIdx.x, j = 0;
  for (; j < a.n_jobs; ++j) {
    const int nb = (lut_job(a, j).M + 255) / 256;
    if (blk < nb) break;
    blk -= nb;
  }
  if (j >= a.n_jobs) return;
  const LutJob& jb = lut_job(a, j);
  const int row = blk * 256 + threadIdx.x;
  if (row >= jb.M) return;
  const int rb = row / kLRows, r = row - rb * kLRows;
  const float* p = jb.partials + (size_t)rb * a.spb * kLRows + r;
  float sum = 0.f;
  int st = 0;
  for (; st + 8 <= a.spb; st += 8) {
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = __ldcg(p + (size_t)(st + k) * kLRows);
#pragma unroll
    for (int k = 0; k < 8; ++k) sum += v[k];
  }
  for (; st < a.spb; ++st) sum += __ldcg(p + (size_t)st * kLRows);
  jb.y[row] = sum + (jb.bias ? jb.bias[row] : 0.f);
}

int lut_sm_count() {
  static int n = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  });
  return n;
}

PFN_cuTensorMapEncodeTiled_v12000 lut_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// Rotation block, activations and code tile alignment the kernels take.
bool lut_common_eligible(int M, int K, int cols, int had_block, const int8_t* signs, const void* codes,
                         const void* x, int x_dtype) {
  if (M <= 0 || K <= 0 || K % cols) return false;
  if (had_block != 0) {
    if (had_block > 512 || (had_block & (had_block - 1)) || had_block < 4 || K % had_block) return false;
    if (!signs || reinterpret_cast<uintptr_t>(signs) % 4) return false;
  }
  if (reinterpret_cast<uintptr_t>(codes) % 16) return false;
  const uintptr_t xa = x_dtype == PF_DTYPE_F32 ? 16 : 8;
  if (reinterpret_cast<uintptr_t>(x) % xa) return false;
  return lut_encode_fn() != nullptr;
}

size_t lut_partial_bytes(int M, int K, int cols) {
  const size_t n_rb = (M + kLRows - 1) / kLRows, spb = K / cols;
  if (spb <= 1) return 0;
  return (n_rb * spb * kLRows * sizeof(float) + 255) / 256 * 256;
}

// One launch over a.n_jobs weights sharing x, K and the rotation (the jobs'
// scales, bias, y, out_scale and M set by the caller).
template <class Pol>
int launch_lut(LutArgs& a, const void* const* codes, void* workspace, cudaStream_t s, cudaError_t* err) {
  constexpr uint32_t kSlot = Pol::kCodes + Pol::kScales;
  constexpr size_t kTab = (size_t)Pol::kTabFloats * 4;
  auto fn = lut_encode_fn();
  a.G = a.K / 128;
  a.spb = a.K / Pol::kCols;
  a.status = static_cast<unsigned*>(workspace) + kWsStatusSlot;
  const size_t row_bytes = (size_t)(a.K / Pol::kCols) * Pol::kRowCode;
  char* part = static_cast<char*>(workspace) + kWsCounterBytes;
  int rb0 = 0;
  CUtensorMap maps[kLutMaxJobs];
  for (int k = 0; k < a.n_jobs; ++k) {
    LutJob& jb = a.job[k];
    jb.n_rb = (jb.M + kLRows - 1) / kLRows;
    jb.rb0 = rb0;
    rb0 += jb.n_rb;
    jb.partials = reinterpret_cast<float*>(part);
    part += lut_partial_bytes(jb.M, a.K, Pol::kCols);
    cuuint64_t dims[2] = {(cuuint64_t)(row_bytes / 4), (cuuint64_t)jb.M};
    cuuint64_t strides[1] = {(cuuint64_t)row_bytes};
    cuuint32_t box[2] = {(cuuint32_t)(Pol::kRowCode / 4), (cuuint32_t)kLRowsW};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(&maps[k], CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(codes[k]), dims, strides, box,
                    estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                    CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return PF_ERR_UNSUPPORTED;
  }
  for (int k = a.n_jobs; k < kLutMaxJobs; ++k) maps[k] = maps[0];
  a.n_rb = rb0;
  a.n_units = a.n_rb * a.spb;
  int P = lut_sm_count();
  if (P > a.n_units) P = a.n_units;
  if ((unsigned long long)a.n_units * (unsigned long long)(P + 1) >= (1ull << 32)) return PF_ERR_SHAPE;
  int max_runs = 1;
  for (int cta = 0; cta < P; ++cta) {
    const int u0 = (int)((long long)cta * a.n_units / P), u1 = (int)((long long)(cta + 1) * a.n_units / P);
    if (u1 <= u0) continue;
    const int r = (u1 - 1) / a.n_rb - u0 / a.n_rb + 1;
    if (r > max_runs) max_runs = r;
  }
  const size_t per_stage = (size_t)kLW * (kSlot + 8);
  int XS = max_runs < kLMaxTabs ? max_runs : kLMaxTabs;
  while (XS > 1 && 128 + (size_t)XS * kTab + 3 * per_stage > (size_t)kLSmemBudget) --XS;
  int NS = (int)(((size_t)kLSmemBudget - 128 - (size_t)XS * kTab) / per_stage);
  if (NS > kLMaxStages) NS = kLMaxStages;
  if (NS < 2) return PF_ERR_UNSUPPORTED;
  a.NS = NS;
  a.XS = XS;
  const size_t smem = 128 + (size_t)XS * kTab + (size_t)NS * per_stage;
  auto kern = lut_gemv_kernel<Pol>;
  {
    // the shared-memory opt-in is per device
    static std::mutex mu;
    static bool done[64] = {false};
    int dev = 0;
    cudaError_t e = cudaGetDevice(&dev);
    if (e != cudaSuccess) {
      *err = e;
      return PF_ERR_CUDA;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (dev < 0 || dev >= 64 || !done[dev]) {
      e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kLSmemBudget);
      if (e != cudaSuccess) {
        *err = e;
        return PF_ERR_CUDA;
      }
      if (dev >= 0 && dev < 64) done[dev] = true;
    }
  }
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(P);
  cfg.blockDim = dim3(kLT);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, maps[0], maps[1], maps[2], maps[3], (const LutArgs)a);
  if (e != cudaSuccess) {
    *err = e;
    return PF_ERR_CUDA;
  }
  note_launch();
  if (a.spb > 1) {
    int blocks = 0;
    for (int k = 0; k < a.n_jobs; ++k) blocks += (a.job[k].M + 255) / 256;
    cudaLaunchConfig_t cc = {};
    cc.gridDim = dim3(blocks);
    cc.blockDim = dim3(256);
    cc.stream = s;
    cc.attrs = attr;
    cc.numAttrs = 1;
    e = cudaLaunchKernelEx(&cc, lut_combine_kernel, (const LutArgs)a);
    if (e != cudaSuccess) {
      *err = e;
      return PF_ERR_CUDA;
    }
    note_launch();
  }
  return PF_OK;
}

LutArgs lut_args(const void* x, int x_dtype, const int8_t* signs, int had_block, int K) {
  LutArgs a;
  memset(&a, 0, sizeof(a));
  a.x = x;
  a.x_dtype = x_dtype;
  a.signs = had_block ? signs : nullptr;
  a.had_block = had_block;
  a.had_rscale = had_block ? 1.f / sqrtf((float)had_block) : 1.f;
  a.K = K;
  return a;
}

}  // namespace

bool e8_lut_eligible(const E8In& in) {
  if (!lut_common_eligible(in.M, in.K, E8Pol::kCols, in.had_block, in.signs, in.codes, in.x, in.x_dtype))
    return false;
  return reinterpret_cast<uintptr_t>(in.scales) % 8 == 0;
}

size_t e8_lut_partial_bytes(int M, int K) { return lut_partial_bytes(M, K, E8Pol::kCols); }

bool polar8_lut_eligible(const Polar8In& in) {
  static const int kAlloc[8] = {3, 2, 2, 2, 2, 1, 1, 1};
  for (int i = 0; i < 8; ++i)
    if (in.alloc[i] != kAlloc[i]) return false;
  return lut_common_eligible(in.M, in.K, Polar8Pol::kCols, in.had_block, in.signs, in.codes, in.x, in.x_dtype);
}

size_t polar8_lut_partial_bytes(int M, int K) { return lut_partial_bytes(M, K, Polar8Pol::kCols); }

int launch_e8_lut(const E8In* in, int count, void* workspace, cudaStream_t s, cudaError_t* err) {
  *err = cudaSuccess;
  if (count < 1 || count > kLutMaxJobs) return PF_ERR_INVALID_ARGUMENT;
  LutArgs a = lut_args(in[0].x, in[0].x_dtype, in[0].signs, in[0].had_block, in[0].K);
  const void* codes[kLutMaxJobs];
  for (int k = 0; k < count; ++k) {
    if (!e8_lut_eligible(in[k]) || in[k].x != in[0].x || in[k].K != in[0].K || in[k].had_block != in[0].had_block ||
        in[k].signs != in[0].signs || in[k].x_dtype != in[0].x_dtype)
      return PF_ERR_UNSUPPORTED;
    LutJob& jb = a.job[k];
    jb.scales = static_cast<const uint32_t*>(in[k].scales);
    jb.bias = in[k].bias;
    jb.y = in[k].y;
    jb.M = in[k].M;
    jb.out_scale = 1.f;
    codes[k] = in[k].codes;
  }
  a.n_jobs = count;
  return launch_lut<E8Pol>(a, codes, workspace, s, err);
}

int launch_polar8_lut(const Polar8In* in, int count, void* workspace, cudaStream_t s, cudaError_t* err) {
  *err = cudaSuccess;
  if (count < 1 || count > kLutMaxJobs) return PF_ERR_INVALID_ARGUMENT;
  LutArgs a = lut_args(in[0].x, in[0].x_dtype, in[0].signs, in[0].had_block, in[0].K);
  const void* codes[kLutMaxJobs];
  for (int k = 0; k < count; ++k) {
    if (!polar8_lut_eligible(in[k]) || in[k].x != in[0].x || in[k].K != in[0].K ||
        in[k].had_block != in[0].had_block || in[k].signs != in[0].signs || in[k].x_dtype != in[0].x_dtype ||
        in[k].angles != in[0].angles)
      return PF_ERR_UNSUPPORTED;
    LutJob& jb = a.job[k];
    jb.bias = in[k].bias;
    jb.y = in[k].y;
    jb.M = in[k].M;
    jb.out_scale = in[k].r_scale;
    codes[k] = in[k].codes;
  }
  a.n_jobs = count;
  a.angles = in[0].angles;
  return launch_lut<Polar8Pol>(a, codes, workspace, s, err);
}

}  // namespace pfb
