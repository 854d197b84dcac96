// pf_qlinear_noalloc: the fused linear for callers that cannot allocate
// device memory.
//
// Some hosts of this library own every byte of device memory themselves, or
// call it from a context where allocating is not allowed: an engine plugin's
// enqueue step, a runtime with a fixed memory pool, code that must not
// trigger the CUDA caching allocator.  They cannot hand pf_qlinear a
// workspace.  This entry point uses a fixed scratch array that lives in the
// library's own device image instead: kNoAllocScratchBytes (8 MiB) per GPU,
// reserved when the library is loaded on that GPU and kept until the process
// exits.  It performs no cudaMalloc / cudaFree and calls no allocating
// library routine.
//
// Host code may not use the array's name as a device address (on the host it
// names a shadow symbol), so the first call on each device, with that device
// current, looks up the real device address with cudaGetSymbolAddress,
// zero-fills the split-K arrival counters and the status word at the start
// of the array and waits for the device to finish that fill.  That first call
// must therefore happen before any stream capture on the device.  Later
// calls reuse the cached address.
//
// A kernel whose bounded wait runs out records PF_ERR_TIMEOUT in the array's
// status word and may leave arrival counters set; the call has returned
// PF_OK by then.  pf_qlinear_noalloc_status reads that word (and counts the
// counters left set) after the stream's work and can zero them again.
//
// All calls on a device share the one array and leave their contents in it
// (the counters end every call at zero again).  Calls whose kernels overlap
// on the GPU — different streams without ordering between them — race on it:
// keep such calls ordered on one stream.
#include <mutex>

#include "gemv.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = 8u << 20;  // 8 MiB per device
constexpr size_t kNoAllocCounterBytes = pfb::kWsCounterBytes;  // split-K counters, must start at zero
constexpr int kMaxDevices = 64;

static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

std::mutex g_noalloc_mutex;
void* g_noalloc_ptr[kMaxDevices] = {nullptr};

// Device address of the scratch array on the current device (set-up on first use).
int noalloc_scratch(void** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return PF_ERR_CUDA;
  if (dev < 0 || dev >= kMaxDevices) return PF_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(g_noalloc_mutex);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return PF_ERR_CUDA;
    e = cudaMemset(p, 0, kNoAllocCounterBytes);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();  // ordered before work on any stream
    if (e != cudaSuccess) return PF_ERR_CUDA;
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return PF_OK;
}

}  // namespace

extern "C" int pf_qlinear_noalloc(const pf_qweight* w, const void* x, int x_dtype, int N, const float* bias,
                                  float* y, void* stream) {
  if (!w || N < 0) return PF_ERR_INVALID_ARGUMENT;
  size_t need = 0;
  int st = pf_qlinear_workspace_size(w, N, &need);  // also validates w
  if (st) return st;
  // the least workspace the call can run in (batches above 16 tokens then
  // take the tensor-core GEMM without stream-K partial tiles)
  need = pfb::min_workspace_bytes(w, N);
  if (need > kNoAllocScratchBytes) return PF_ERR_WORKSPACE;  // request beyond the fixed 8 MiB scratch
  void* scratch = nullptr;
  st = noalloc_scratch(&scratch);
  if (st) return st;
  return pf_qlinear(w, x, x_dtype, N, bias, y, scratch, kNoAllocScratchBytes, stream);
}

extern "C" int pf_qlinear_noalloc_status(int reset, int* status, int* busy_counters, void* stream) {
  if (!status) return PF_ERR_INVALID_ARGUMENT;
  void* scratch = nullptr;
  int st = noalloc_scratch(&scratch);
  if (st) return st;
  return pfb::read_workspace_head(scratch, reset, status, busy_counters, static_cast<cudaStream_t>(stream));
}
