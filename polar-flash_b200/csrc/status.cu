// Device-status entry points: what a bounded device wait left in a
// workspace, and a self-test of that wait.
//
// The streaming kernels never wait without a limit: a wait that runs out
// records PF_ERR_TIMEOUT in the workspace's status word and the kernel
// finishes early, leaving its outputs incomplete.  The launch itself has
// already returned PF_OK by then, so a caller learns of it only by reading
// the status word once the stream's work is done: pf_workspace_status.
#include <string.h>

#include "gemv.cuh"
#include "tma.cuh"

namespace pfb {
namespace {

// One bounded wait on an mbarrier phase that no thread completes: the
// kernels' own wait loop (mbar_wait), given `limit_ns`, gives up and the
// block records PF_ERR_TIMEOUT, as a streaming kernel does.
__global__ void wait_selftest_kernel(unsigned* status, unsigned long long limit_ns) {
  __shared__ __align__(8) unsigned long long bar;
  __shared__ int abort_flag;
  const uint32_t b = smem_u32(&bar);
  if (threadIdx.x == 0) {
    abort_flag = 0;
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(b), "r"(1));
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  __syncthreads();
  if (threadIdx.x == 0 && !mbar_wait(b, 0, &abort_flag, limit_ns)) atomicExch(status, (unsigned)PF_ERR_TIMEOUT);
}

}  // namespace

// Reads the head of a workspace (status word and arrival counters) after the
// stream's work; see pf_workspace_status.
int read_workspace_head(void* ws, int reset, int* status, int* busy_counters, cudaStream_t s) {
  unsigned word = 0;
  cudaError_t e = cudaStreamSynchronize(s);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(&word, static_cast<unsigned*>(ws) + kWsStatusSlot, sizeof(word), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) return report_cuda(e);
  *status = word == 0u ? PF_OK : (int)word;
  if (busy_counters) {
    int busy = 0;
    unsigned chunk[1024];
    for (size_t i = 0; i < kWsStatusSlot; i += 1024) {
      const size_t n = kWsStatusSlot - i < 1024 ? kWsStatusSlot - i : 1024;
      e = cudaMemcpyAsync(chunk, static_cast<unsigned*>(ws) + i, n * sizeof(unsigned), cudaMemcpyDeviceToHost, s);
      if (e == cudaSuccess) e = cudaStreamSynchronize(s);
      if (e != cudaSuccess) return report_cuda(e);
      for (size_t k = 0; k < n; ++k) busy += chunk[k] != 0u;
    }
    *busy_counters = busy;
  }
  if (reset) {
    e = cudaMemsetAsync(ws, 0, kWsCounterBytes, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    if (e != cudaSuccess) return report_cuda(e);
  }
  return PF_OK;
}

}  // namespace pfb

extern "C" {

int pf_workspace_status(void* workspace, int reset, int* status, int* busy_counters, void* stream) {
  if (!workspace || !status) return PF_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(workspace) % 256) return PF_ERR_ALIGNMENT;
  return pfb::read_workspace_head(workspace, reset, status, busy_counters, static_cast<cudaStream_t>(stream));
}

int pf_wait_selftest(void* workspace, unsigned long long wait_ns, void* stream) {
  if (!workspace || wait_ns == 0 || wait_ns > pfb::kWaitNs) return PF_ERR_INVALID_ARGUMENT;
  if (reinterpret_cast<uintptr_t>(workspace) % 256) return PF_ERR_ALIGNMENT;
  unsigned* status = static_cast<unsigned*>(workspace) + pfb::kWsStatusSlot;
  pfb::wait_selftest_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(status, wait_ns);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return pfb::report_cuda(e);
  pfb::note_launch();
  return PF_OK;
}

}  // extern "C"
