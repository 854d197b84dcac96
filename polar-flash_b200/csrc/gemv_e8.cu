// Streaming lookup-table GEMV for E8 RVQ2 weights at batch 1:
// y = x W^T with W row m, 8-vector v = s1(m, g) r[i1(m, v)] + s2(m, g) r[i2(m, v)]
// (r = the 240 E8 roots in generate_e8_roots order, g = v's 128-column group),
// and the weight's block RWHT folded into x (x' = forward RWHT of x).
//
// Because every weight vector is one of 240 roots per stage, the dot product
// of a row with x' only needs the 240 values <r_k, x'_v> per 8-vector v of x':
//   y_m = sum_g [ s1 sum_{v in g} T[v][i1] + s2 sum_{v in g} T[v][i2] ].
// A CTA builds the table T of a 256-column stage (32 vectors x 256 entries,
// fp32, 32 KB, entries 240..255 zero) in shared memory from x', then every
// weight vector costs two table reads and two adds; no weight is decoded.
//
// Work unit = (stage of 256 columns, block of 512 rows), dealt to the CTAs
// stream-K style in stage-major order, so a CTA's consecutive units share a
// stage and its table.  One 16-warp CTA per SM; every warp owns 32 rows of a
// unit and streams them through its own ring of shared-memory slots: lane 0
// issues the TMA copy of the 32 x 64-byte index tile (L2 evict-first), every
// lane copies its row's two half2 group scales with cp.async, and the copies
// arrive on the slot's mbarrier.  The first two slots are requested before
// the kernel waits for the preceding grid (weights and scales are never
// written by it); x' and the tables are built after the wait.
// Per unit a lane reads 8 vectors (16 bytes) of a row, a quarter of the row's
// 64 bytes; four lanes finish a row with two shuffles.  Each unit's row sums
// go to the workspace, and e8_combine_kernel (a programmatic dependent) adds
// a row's stage sums in stage order and writes y: deterministic.
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

constexpr int kEW = 16;                             // warps per CTA
constexpr int kET = kEW * 32;                       // threads per CTA
constexpr int kERowsW = 32;                         // rows per warp and unit
constexpr int kERows = kEW * kERowsW;               // rows per unit
constexpr int kECols = 256;                         // columns per stage
constexpr int kEVec = kECols / 8;                   // 8-vectors per stage
constexpr uint32_t kETab = kEVec * 256 * 4;         // table bytes per stage
constexpr uint32_t kECodes = kERowsW * kECols / 4;  // index bytes of a warp's tile
constexpr uint32_t kESlot = kECodes + kERowsW * 8;  // + two half2 scales per row
constexpr int kEMaxStages = 8;
constexpr int kEMaxTabs = 3;
constexpr int kESmemBudget = 220 * 1024;

struct E8Args {
  const uint32_t* scales;  // half2 [M][G] as words
  const void* x;
  const int8_t* signs;
  const float* bias;
  float* y;
  float* partials;  // [n_rb][spb][kERows] stage row sums (spb > 1)
  unsigned* status;
  float had_rscale;
  int had_block, x_dtype, M, K, G, n_rb, spb, n_units, NS, XS;
};

// x' of columns [c0, c0 + 256) into xs[0, 256): forward block RWHT of x
// (signs, Walsh-Hadamard butterflies in registers and across lanes, 1/sqrt(b))
// for rotation blocks b <= 512, or x itself when b = 0.  A warp transforms a
// chunk of 32 E columns (E = 4, 8, 16 for b <= 128, 256, 512), which holds
// whole rotation blocks.
template <int E>
__device__ __forceinline__ void xprime_chunk(const E8Args& a, int col0, int c0, float* xs, int lane) {
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
    if (col >= 0 && col < kECols) xs[col] = v[e] * a.had_rscale;
  }
}

__device__ __forceinline__ void stage_xprime(const E8Args& a, int c0, float* xs, int warp, int lane) {
  const int b = a.had_block;
  if (b == 0) {
    for (int i = threadIdx.x; i < kECols; i += kET) {
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
  if (b > 256) {
    if (warp == 0) xprime_chunk<16>(a, (c0 / 512) * 512, c0, xs, lane);
  } else if (b > 128) {
    if (warp == 0) xprime_chunk<8>(a, c0, c0, xs, lane);
  } else if (warp < 2) {
    xprime_chunk<4>(a, c0 + 128 * warp, c0, xs, lane);
  }
}

// Table entry `idx` of the table row at shared address `row` (a constant
// offset from the lane's row block, which folds into the load's immediate).
__device__ __forceinline__ float tab_read(uint32_t row, uint32_t idx) {
  float v;
  asm volatile("ld.shared.f32 %0, [%1];" : "=f"(v) : "r"(row + (idx << 2)));
  return v;
}

__global__ void __launch_bounds__(kET, 1)
    gemv_e8_lut_kernel(const __grid_constant__ CUtensorMap map, const __grid_constant__ E8Args a) {
  asm volatile("griddepcontrol.launch_dependents;");
  if (threadIdx.x == 32) asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(&map)) : "memory");

  extern __shared__ __align__(128) unsigned char smem_raw[];
  __shared__ int abort_flag;
  __shared__ __align__(16) float xs[kECols];
  unsigned char* const base = smem_raw + ((128u - (smem_u32(smem_raw) & 127u)) & 127u);
  const int NS = a.NS, XS = a.XS;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  float* const tabs = reinterpret_cast<float*>(base);
  unsigned char* const ring = base + (size_t)XS * kETab + (size_t)warp * NS * kESlot;
  const uint32_t full0 = smem_u32(base + (size_t)XS * kETab + (size_t)kEW * NS * kESlot) + warp * NS * 8;

  // root k = threadIdx.x mod 256 of the table column this thread fills (zero past 239)
  float root[8];
  {
    const int k = threadIdx.x & 255;
    if (k < 240) {
      e8_root(k, root);
    } else {
#pragma unroll
      for (int q = 0; q < 8; ++q) root[q] = 0.f;
    }
  }
  if (threadIdx.x == 0) abort_flag = 0;
  if (lane == 0) {
    for (int s = 0; s < NS; ++s) asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(full0 + 8 * s), "r"(33));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();

  const unsigned U = (unsigned)a.n_units, P = gridDim.x, cta = blockIdx.x;
  const int u0 = (int)(cta * U / P), u1 = (int)((cta + 1) * U / P);  // U * P < 2^32 (host-checked)
  const int nunits = u1 - u0;
  if (nunits <= 0) return;

  // ---- load side: this warp's next unit to request
  int fst = u0 / a.n_rb, frb = u0 - fst * a.n_rb;
  uint64_t policy;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(policy));
  const uint32_t ring_s = smem_u32(ring);
  auto request = [&](int slot) {
    const uint32_t sb = ring_s + slot * kESlot, bar = full0 + 8 * slot;
    const int row0 = frb * kERows + warp * kERowsW;
    __syncwarp();
    if (lane == 0) {
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      mbar_expect(bar, kECodes);
      tma_2d(sb, &map, fst * (kECols / 16), row0, bar, policy);
    }
    const int grow = row0 + lane;
    const bool ok = grow < a.M;
    cp_async8(sb + kECodes + lane * 8, a.scales + (ok ? (size_t)grow * a.G + 2 * fst : 0), ok ? 8u : 0u);
    cp_async_arrive(bar);
    if (++frb == a.n_rb) {
      frb = 0;
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
      stage_xprime(a, (st_first + r) * kECols, xs, warp, lane);
      __syncthreads();
      float* tab = tabs + (size_t)(r % XS) * (kEVec * 256);
      const int k = threadIdx.x & 255;
      for (int v = (threadIdx.x >> 8) * (kEVec / 2); v < ((threadIdx.x >> 8) + 1) * (kEVec / 2); ++v) {
        const float4 p0 = *reinterpret_cast<const float4*>(xs + 8 * v);
        const float4 p1 = *reinterpret_cast<const float4*>(xs + 8 * v + 4);
        float d = root[0] * p0.x;
        d = fmaf(root[1], p0.y, d);
        d = fmaf(root[2], p0.z, d);
        d = fmaf(root[3], p0.w, d);
        d = fmaf(root[4], p1.x, d);
        d = fmaf(root[5], p1.y, d);
        d = fmaf(root[6], p1.z, d);
        d = fmaf(root[7], p1.w, d);
        tab[v * 256 + k] = d;
      }
      __syncthreads();  // tables written, xs free for the next run
    }
    win_end = r1;
  };

  // x may be written by the preceding grid, and so may the workspace and y
  asm volatile("griddepcontrol.wait;" ::: "memory");
  build_window(0);
  for (; requested < NS && requested < nunits; ++requested) request(requested);

  const int r8 = lane >> 2, q = lane & 3;
  int st = st_first, rb = u0 - st_first * a.n_rb, run = 0, slot = 0;
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
      const unsigned char* tile = ring + slot * kESlot;
      // this lane's vectors 8q .. 8q + 7 of the stage: table rows 1 KB apart
      const uint32_t tab = smem_u32(tabs) + (uint32_t)(run % XS) * kETab + (uint32_t)(8 * q) * 1024u;
      float rs[4];
#pragma unroll
      for (int p = 0; p < 4; ++p) {
        const int r = 8 * p + r8;
        const uint4 cw = lds<uint4>(tile + r * 64 + q * 16);
        const uint32_t sw = lds<uint32_t>(tile + kECodes + r * 8 + (q >> 1) * 4);
        const float2 s = __half22float2(*reinterpret_cast<const __half2*>(&sw));
        const uint32_t w[4] = {cw.x, cw.y, cw.z, cw.w};
        float A1 = 0.f, A2 = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            // index bytes 2h (stage 1) and 2h + 1 (stage 2) of word j: vector 2j + h
            const uint32_t row = tab + (uint32_t)(2 * j + h) * 1024u;
            A1 += tab_read(row, __byte_perm(w[j], 0u, 0x4440u + 2 * h));
            A2 += tab_read(row, __byte_perm(w[j], 0u, 0x4441u + 2 * h));
          }
        float part = fmaf(s.x, A1, s.y * A2);
        part += __shfl_xor_sync(0xffffffffu, part, 1);
        part += __shfl_xor_sync(0xffffffffu, part, 2);
        rs[p] = part;
      }
      if (q == 0) {
#pragma unroll
        for (int p = 0; p < 4; ++p) {
          const int rl = warp * kERowsW + 8 * p + r8;
          const int row = rb * kERows + rl;
          if (a.spb == 1) {
            if (row < a.M) a.y[row] = rs[p] + (a.bias ? a.bias[row] : 0.f);
          } else {
            __stcg(a.partials + ((size_t)rb * a.spb + st) * kERows + rl, rs[p]);
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
    if (++rb == a.n_rb) {
      rb = 0;
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

// y = the sum of a row's stage sums in stage order (+ bias).
__global__ void __launch_bounds__(256) e8_combine_kernel(const __grid_constant__ E8Args a) {
  asm volatile("griddepcontrol.launch_dependents;");
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int row = blockIdx.x * 256 + threadIdx.x;
  if (row >= a.M) return;
  const int rb = row / kERows, r = row - rb * kERows;
  const float* p = a.partials + (size_t)rb * a.spb * kERows + r;
  float sum = 0.f;
  int st = 0;
  for (; st + 8 <= a.spb; st += 8) {
    float v[8];
#pragma unroll
    for (int k = 0; k < 8; ++k) v[k] = __ldcg(p + (size_t)(st + k) * kERows);
#pragma unroll
    for (int k = 0; k < 8; ++k) sum += v[k];
  }
  for (; st < a.spb; ++st) sum += __ldcg(p + (size_t)st * kERows);
  a.y[row] = sum + (a.bias ? a.bias[row] : 0.f);
}

int e8_sm_count() {
  static int n = 0;
  static std::once_flag once;
  std::call_once(once, [] {
    int dev = 0;
    cudaGetDevice(&dev);
    if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
  });
  return n;
}

PFN_cuTensorMapEncodeTiled_v12000 e8_encode_fn() {
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

}  // namespace

bool e8_lut_eligible(const E8In& in) {
  if (in.M <= 0 || in.K <= 0 || in.K % kECols) return false;
  const int b = in.had_block;
  if (b != 0) {
    if (b > 512 || (b & (b - 1)) || b < 4 || in.K % b) return false;
    if (!in.signs || reinterpret_cast<uintptr_t>(in.signs) % 4) return false;
  }
  if (reinterpret_cast<uintptr_t>(in.codes) % 16 || reinterpret_cast<uintptr_t>(in.scales) % 8) return false;
  const uintptr_t xa = in.x_dtype == PF_DTYPE_F32 ? 16 : 8;
  if (reinterpret_cast<uintptr_t>(in.x) % xa) return false;
  return e8_encode_fn() != nullptr;
}

size_t e8_lut_partial_bytes(int M, int K) {
  const size_t n_rb = (M + kERows - 1) / kERows, spb = K / kECols;
  if (spb <= 1) return 0;
  return (n_rb * spb * kERows * sizeof(float) + 255) / 256 * 256;
}

int launch_e8_lut(const E8In& in, void* workspace, cudaStream_t s, cudaError_t* err) {
  *err = cudaSuccess;
  if (!e8_lut_eligible(in)) return PF_ERR_UNSUPPORTED;
  auto fn = e8_encode_fn();
  E8Args a;
  memset(&a, 0, sizeof(a));
  a.scales = static_cast<const uint32_t*>(in.scales);
  a.x = in.x;
  a.x_dtype = in.x_dtype;
  a.signs = in.had_block ? in.signs : nullptr;
  a.had_block = in.had_block;
  a.had_rscale = in.had_block ? 1.f / sqrtf((float)in.had_block) : 1.f;
  a.bias = in.bias;
  a.y = in.y;
  a.M = in.M;
  a.K = in.K;
  a.G = in.K / 128;
  a.n_rb = (in.M + kERows - 1) / kERows;
  a.spb = in.K / kECols;
  a.n_units = a.n_rb * a.spb;
  a.status = static_cast<unsigned*>(workspace) + kWsStatusSlot;
  a.partials = reinterpret_cast<float*>(static_cast<char*>(workspace) + kWsCounterBytes);

  CUtensorMap map;
  {
    cuuint64_t dims[2] = {(cuuint64_t)(in.K / 16), (cuuint64_t)in.M};
    cuuint64_t strides[1] = {(cuuint64_t)(in.K / 4)};
    cuuint32_t box[2] = {(cuuint32_t)(kECols / 16), (cuuint32_t)kERowsW};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = fn(&map, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<void*>(in.codes), dims, strides, box, estr,
                    CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                    CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return PF_ERR_UNSUPPORTED;
  }
  int P = e8_sm_count();
  if (P > a.n_units) P = a.n_units;
  if ((unsigned long long)a.n_units * (unsigned long long)(P + 1) >= (1ull << 32)) return PF_ERR_SHAPE;
  int max_runs = 1;
  for (int cta = 0; cta < P; ++cta) {
    const int u0 = (int)((long long)cta * a.n_units / P), u1 = (int)((long long)(cta + 1) * a.n_units / P);
    if (u1 <= u0) continue;
    const int r = (u1 - 1) / a.n_rb - u0 / a.n_rb + 1;
    if (r > max_runs) max_runs = r;
  }
  const size_t per_stage = (size_t)kEW * (kESlot + 8);
  int XS = max_runs < kEMaxTabs ? max_runs : kEMaxTabs;
  while (XS > 1 && 128 + (size_t)XS * kETab + 3 * per_stage > (size_t)kESmemBudget) --XS;
  int NS = (int)(((size_t)kESmemBudget - 128 - (size_t)XS * kETab) / per_stage);
  if (NS > kEMaxStages) NS = kEMaxStages;
  if (NS < 2) return PF_ERR_UNSUPPORTED;
  a.NS = NS;
  a.XS = XS;
  const size_t smem = 128 + (size_t)XS * kETab + (size_t)NS * per_stage;
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
      e = cudaFuncSetAttribute(gemv_e8_lut_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, kESmemBudget);
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
  cfg.blockDim = dim3(kET);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, gemv_e8_lut_kernel, map, (const E8Args)a);
  if (e != cudaSuccess) {
    *err = e;
    return PF_ERR_CUDA;
  }
  note_launch();
  if (a.spb > 1) {
    cudaLaunchConfig_t cc = {};
    cc.gridDim = dim3((in.M + 255) / 256);
    cc.blockDim = dim3(256);
    cc.stream = s;
    cc.attrs = attr;
    cc.numAttrs = 1;
    e = cudaLaunchKernelEx(&cc, e8_combine_kernel, (const E8Args)a);
    if (e != cudaSuccess) {
      *err = e;
      return PF_ERR_CUDA;
    }
    note_launch();
  }
  return PF_OK;
}

}  // namespace pfb
