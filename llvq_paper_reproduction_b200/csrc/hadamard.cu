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
// One CTA per (row, segment): load to shared memory (fp32, fp16 or bf16
// input), log2(block) butterfly stages in fp32 separated by barriers, scale,
// store fp32 or bf16 (rounded once).  The bf16 form rotates a GEMM's
// activations for weights that were quantized after the same rotation:
// x W^T = (x R)(W R)^T for orthogonal R.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "llvq_internal.h"

namespace llvq {

constexpr int kHadThreads = 256;
constexpr int kMaxHadBlock = 4096;

// Element types: 0 fp32, 1 fp16, 2 bf16 (inputs); 0 fp32, 2 bf16 (outputs).
template <int kIn>
__device__ __forceinline__ float load_elem(const void* p, int64_t i) {
  if constexpr (kIn == 1) return __half2float(static_cast<const __half*>(p)[i]);
  else if constexpr (kIn == 2) return __bfloat162float(static_cast<const __nv_bfloat16*>(p)[i]);
  else return static_cast<const float*>(p)[i];
}

template <int kOut>
__device__ __forceinline__ void store_elem(void* p, int64_t i, float v) {
  if constexpr (kOut == 2) static_cast<__nv_bfloat16*>(p)[i] = __float2bfloat16_rn(v);
  else static_cast<float*>(p)[i] = v;
}

template <int kIn, int kOut>
__global__ void __launch_bounds__(kHadThreads) hadamard_kernel(const void* __restrict__ in, void* __restrict__ out,
                                                               int64_t cols, int block, int log2b,
                                                               const int8_t* __restrict__ signs, int inverse) {
  __shared__ float buf[kMaxHadBlock];
  const int64_t segs = cols / block;
  const int64_t row = blockIdx.x / segs;
  const int64_t seg = blockIdx.x % segs;
  const int64_t base = row * cols + seg * block;
  const int8_t* sg = signs + seg * block;
  for (int i = threadIdx.x; i < block; i += kHadThreads) {
    float v = load_elem<kIn>(in, base + i);
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
    store_elem<kOut>(out, base + i, v);
  }
}

cudaError_t hadamard_launch(const void* in, int in_type, void* out, int out_type, int64_t rows, int64_t cols,
                            int block, const int8_t* signs, int inverse, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  int log2b = 0;
  while ((1 << log2b) < block) ++log2b;
  const int64_t grid = rows * (cols / block);
  if (grid > 0x7FFFFFFFLL) return cudaErrorInvalidValue;
  const unsigned g = (unsigned)grid;
#define LLVQ_HAD(I, O) hadamard_kernel<I, O><<<g, kHadThreads, 0, stream>>>(in, out, cols, block, log2b, signs, inverse)
  if (out_type == 0) {
    if (in_type == 0) LLVQ_HAD(0, 0);
    else if (in_type == 1) LLVQ_HAD(1, 0);
    else LLVQ_HAD(2, 0);
  } else {
    if (in_type == 0) LLVQ_HAD(0, 2);
    else if (in_type == 1) LLVQ_HAD(1, 2);
    else LLVQ_HAD(2, 2);
  }
#undef LLVQ_HAD
  return cudaGetLastError();
}

}  // namespace llvq
