// Fixed staging buffer for llvq_gemm_noalloc.
//
// The large-batch GEMM decodes weights into a bf16 staging buffer before the
// tensor-core pass.  llvq_gemm takes that buffer from a stream-ordered pool on the
// caller's stream; llvq_gemm_noalloc takes it from the array below instead,
// for callers that may not allocate device memory while they run: a serving
// engine that reserved the GPU's memory for its own pool at start-up and must
// not see a library allocate behind it, or a step that must not fail with an
// out-of-memory error halfway through.
//
// One array per device (a __device__ variable exists once in every context
// that loads this module).  Its contents need not start at zero: every byte
// the GEMM reads is written by the decode kernel of the same call.  Two calls
// that overlap on one device (different streams without ordering, or
// different host threads) share the array and race.
#include <cuda_runtime.h>

#include <cstdint>
#include <mutex>

#include "llvq_internal.h"

namespace llvq {

static __device__ __align__(256) unsigned char g_gemm_staging[kNoAllocStagingBytes];

// Address of this device's staging array (the current device at the time
// of the call).  cudaGetSymbolAddress runs on every call: once the module is
// loaded it is a host-side lookup, and a cached address could go stale if the
// caller resets the device (the module, and with it the array, is then loaded
// again, possibly elsewhere).  The first call on a device loads the module
// that holds the array -- this is when the CUDA runtime allocates its 16 MiB
// -- and sets the GEMM kernels' shared-memory limits on that device.
cudaError_t noalloc_staging(void** ptr) {
  static std::mutex mu;
  static bool configured[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  void* p = nullptr;
  e = cudaGetSymbolAddress(&p, g_gemm_staging);
  if (e != cudaSuccess) return e;
  if (!p) return cudaErrorInvalidSymbol;
  std::lock_guard<std::mutex> lock(mu);
  if (!configured[dev]) {
    e = gemm_configure_device();
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  *ptr = p;
  return cudaSuccess;
}

}  // namespace llvq
