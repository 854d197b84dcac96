// Peer buffers for column-parallel linears whose all-gather is fused into
// the GEMV (pf_qlinear_group_gather): mapping another rank's buffer into this
// process (CUDA IPC), the wait for every rank's rows of the latest call, and
// a standalone all-gather of already computed row shards (pf_allgather_rows).
//
// Header of a peer buffer (kPeerHeader bytes): the owning rank's epoch (the
// number of gathering launches it has finished) at byte 0, then at byte
// 16 + 4 q the epoch that rank q last raised in this buffer.  A gathering
// launch's last CTA bumps the local epoch and writes it into every rank's
// flag slot with a system-scope release once all of its rows are stored.
#include <cuda.h>
#include <cudaTypedefs.h>
#include <string.h>

#include <mutex>

#include "gemv.cuh"
#include "tma.cuh"

namespace pfb {
namespace {

PFN_cuMemGetAddressRange_v3020 range_fn() {
  static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(p);
  });
  return fn;
}

// One warp: lane q < world waits until rank q's flag in this rank's buffer
// has reached this rank's epoch (bounded by kWaitNs); on expiry the status
// word records PF_ERR_TIMEOUT.
__global__ void peers_wait_kernel(const unsigned char* local, int world, unsigned* status) {
  const int q = threadIdx.x;
  if (q < world) {
    const unsigned e = *reinterpret_cast<const volatile unsigned*>(local);
    const unsigned* flag = reinterpret_cast<const unsigned*>(local + 16 + 4 * q);
    unsigned long long t0 = 0;
    for (;;) {
      unsigned f;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(f) : "l"(flag) : "memory");
      if ((int)(f - e) >= 0) break;
      const unsigned long long t = now_ns();
      if (t0 == 0) {
        t0 = t;
      } else if (t - t0 > kWaitNs) {
        atomicExch(status, (unsigned)PF_ERR_TIMEOUT);
        break;
      }
      __nanosleep(256);
    }
  }
  __syncwarp();
}

struct GatherArgs {
  unsigned char* bases[kMaxPeers];
  int world, rank;
};

// pf_allgather_rows: every block copies 16-byte words of this rank's shard
// into the same place of every rank's buffer (plain peer stores); after a
// system-scope fence per block, the last block to finish raises this rank's
// flag in every buffer to its next epoch (release) and waits, bounded, for
// every rank's flag in the local buffer (acquire).  Every rank raises its
// flag before it waits and each rank runs on its own GPU.
__global__ void __launch_bounds__(256) allgather_rows_kernel(const __grid_constant__ GatherArgs g, const uint4* src,
                                                             size_t n16, size_t dst_off, unsigned* done,
                                                             unsigned* status) {
  const size_t total = (size_t)g.world * n16;
  const size_t rank_off = dst_off + (size_t)g.rank * n16 * 16;
  for (size_t k = (size_t)blockIdx.x * blockDim.x + threadIdx.x; k < total; k += (size_t)gridDim.x * blockDim.x) {
    const int p = (int)(k / n16);
    const size_t i = k - (size_t)p * n16;
    reinterpret_cast<uint4*>(g.bases[p] + rank_off)[i] = __ldg(src + i);
  }
  __syncthreads();  // the block's peer stores come before thread 0's fence (cumulative)
  if (threadIdx.x != 0) return;
  __threadfence_system();
  if (atomicAdd(done, 1u) != gridDim.x - 1) return;
  atomicExch(done, 0u);
  __threadfence_system();
  volatile unsigned* ep = reinterpret_cast<volatile unsigned*>(g.bases[g.rank]);
  const unsigned e = *ep + 1u;
  *ep = e;
  for (int q = 0; q < g.world; ++q) {
    unsigned* flag = reinterpret_cast<unsigned*>(g.bases[q] + 16 + 4 * g.rank);
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flag), "r"(e) : "memory");
  }
  const unsigned long long t0 = now_ns();
  for (int q = 0; q < g.world; ++q) {
    const unsigned* flag = reinterpret_cast<const unsigned*>(g.bases[g.rank] + 16 + 4 * q);
    for (;;) {
      unsigned f;
      asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(f) : "l"(flag) : "memory");
      if ((int)(f - e) >= 0) break;
      if (now_ns() - t0 > kWaitNs) {
        atomicExch(status, (unsigned)PF_ERR_TIMEOUT);
        return;
      }
      __nanosleep(64);
    }
  }
}

}  // namespace
}  // namespace pfb

extern "C" {

int pf_peer_export(const void* ptr, unsigned char handle[64], size_t* offset) {
  if (!ptr || !handle || !offset) return PF_ERR_INVALID_ARGUMENT;
  auto fn = pfb::range_fn();
  if (!fn) return PF_ERR_UNSUPPORTED;
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return PF_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return pfb::report_cuda(e);
  static_assert(sizeof(h) == 64, "CUDA IPC handles are 64 bytes");
  memcpy(handle, &h, 64);
  *offset = reinterpret_cast<uintptr_t>(ptr) - (uintptr_t)base;
  return PF_OK;
}

int pf_peer_open(const unsigned char handle[64], size_t offset, void** ptr, void** mapping) {
  if (!handle || !ptr || !mapping) return PF_ERR_INVALID_ARGUMENT;
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, 64);
  void* base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return pfb::report_cuda(e);
  *mapping = base;
  *ptr = static_cast<unsigned char*>(base) + offset;
  return PF_OK;
}

int pf_peer_close(void* mapping) {
  if (!mapping) return PF_ERR_INVALID_ARGUMENT;
  const cudaError_t e = cudaIpcCloseMemHandle(mapping);
  return e == cudaSuccess ? PF_OK : pfb::report_cuda(e);
}

int pf_allgather_rows(const pf_peers* peers, const void* src, size_t bytes, size_t dst_offset, void* workspace,
                      void* stream) {
  if (!peers || !src || !workspace || peers->world < 1 || peers->world > pfb::kMaxPeers || peers->rank < 0 ||
      peers->rank >= peers->world)
    return PF_ERR_INVALID_ARGUMENT;
  for (int q = 0; q < peers->world; ++q)
    if (!peers->bases[q]) return PF_ERR_INVALID_ARGUMENT;
  if (bytes == 0 || dst_offset < pfb::kPeerHeader || dst_offset > peers->bytes ||
      (size_t)peers->world * bytes > peers->bytes - dst_offset)
    return PF_ERR_SHAPE;
  if (bytes % 16 || dst_offset % 16 || reinterpret_cast<uintptr_t>(src) % 16 ||
      reinterpret_cast<uintptr_t>(workspace) % 256)
    return PF_ERR_ALIGNMENT;
  for (int q = 0; q < peers->world; ++q)
    if (reinterpret_cast<uintptr_t>(peers->bases[q]) % 256) return PF_ERR_ALIGNMENT;
  pfb::GatherArgs g;
  memset(&g, 0, sizeof(g));
  for (int q = 0; q < peers->world; ++q) g.bases[q] = static_cast<unsigned char*>(peers->bases[q]);
  g.world = peers->world;
  g.rank = peers->rank;
  const size_t n16 = bytes / 16;
  const size_t total = (size_t)g.world * n16;
  size_t blocks = (total + 255) / 256;
  if (blocks > 148) blocks = 148;  // one pass over the words per SM at most
  unsigned* head = static_cast<unsigned*>(workspace);
  pfb::allgather_rows_kernel<<<(unsigned)blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      g, static_cast<const uint4*>(src), n16, dst_offset, head + pfb::kWsDoneSlot, head + pfb::kWsStatusSlot);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return pfb::report_cuda(e);
  pfb::note_launch();
  return PF_OK;
}

int pf_peers_wait(const pf_peers* peers, void* workspace, void* stream) {
  if (!peers || !workspace || peers->world < 1 || peers->world > pfb::kMaxPeers || peers->rank < 0 ||
      peers->rank >= peers->world || !peers->bases[peers->rank])
    return PF_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(workspace) % 256) return PF_ERR_ALIGNMENT;
  unsigned* status = static_cast<unsigned*>(workspace) + pfb::kWsStatusSlot;
  pfb::peers_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const unsigned char*>(peers->bases[peers->rank]), peers->world, status);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return pfb::report_cuda(e);
  pfb::note_launch();
  return PF_OK;
}

}  // extern "C"
