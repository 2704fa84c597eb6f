// Seeded random Hadamard rotation along the rows of a matrix (sm_100a).
//
// For every row and every segment of `block` columns (block a power of two
// dividing the row length, up to 4096):
//   forward:  out = H (s * in) / sqrt(block)
//   inverse:  out = s * (H in) / sqrt(block)
// with H the Walsh-Hadamard matrix in natural (Sylvester) order and s the
// +-1 signs of those columns.  The rotation is orthogonal, so inverse(forward)
// is the identity up to fp32 rounding.  The reference has no rotation (it is
// listed in its README only); this is the pre-quantization step of the
// whole-model workload.
//
// One CTA per (row, segment): load to shared memory (fp16 or fp32 input),
// log2(block) butterfly stages separated by barriers, scale, store fp32.
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "llvq_internal.h"

namespace llvq {

constexpr int kHadThreads = 256;
constexpr int kMaxHadBlock = 4096;

template <bool kHalfIn>
__global__ void __launch_bounds__(kHadThreads) hadamard_kernel(const void* __restrict__ in, float* __restrict__ out,
                                                               int64_t cols, int block, int log2b,
                                                               const int8_t* __restrict__ signs, int inverse) {
  __shared__ float buf[kMaxHadBlock];
  const int64_t segs = cols / block;
  const int64_t row = blockIdx.x / segs;
  const int64_t seg = blockIdx.x % segs;
  const int64_t base = row * cols + seg * block;
  const int8_t* sg = signs + seg * block;
  for (int i = threadIdx.x; i < block; i += kHadThreads) {
    float v = kHalfIn ? __half2float(static_cast<const __half*>(in)[base + i]) : static_cast<const float*>(in)[base + i];
    if (!inverse) v = sg[i] < 0 ? -v : v;
    buf[i] = v;
  }
  __syncthreads();
  for (int st = 0; st < log2b; ++st) {
    const int h = 1 << st;
    for (int p = threadIdx.x; p < block / 2; p += kHadThreads) {
      const int i = ((p >> st) << (st + 1)) | (p & (h - 1));  // pair (i, i + h)
      const float a = buf[i], b = buf[i + h];
      buf[i] = a + b;
      buf[i + h] = a - b;
    }
    __syncthreads();
  }
  const float scale = rsqrtf((float)block);
  for (int i = threadIdx.x; i < block; i += kHadThreads) {
    float v = buf[i] * scale;
    if (inverse) v = sg[i] < 0 ? -v : v;
    out[base + i] = v;
  }
}

cudaError_t hadamard_launch(const void* in, int in_is_half, float* out, int64_t rows, int64_t cols, int block,
                            const int8_t* signs, int inverse, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  int log2b = 0;
  while ((1 << log2b) < block) ++log2b;
  const int64_t grid = rows * (cols / block);
  if (grid > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  if (in_is_half)
    hadamard_kernel<true><<<(unsigned)grid, kHadThreads, 0, stream>>>(in, out, cols, block, log2b, signs, inverse);
  else
    hadamard_kernel<false><<<(unsigned)grid, kHadThreads, 0, stream>>>(in, out, cols, block, log2b, signs, inverse);
  return cudaGetLastError();
}

}  // namespace llvq
