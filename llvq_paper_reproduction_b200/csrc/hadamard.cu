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

// Rotation, row scale and padding of a weight matrix for quantization, one
// CTA per row: the fp16 row with its signs into shared memory (fp32), the
// butterflies of every segment of `block` columns, 1/sqrt(block); then the
// row's RMS (a fixed-order reduction: each thread's strided partial sum, then
// a tree over the threads), rounded to fp16 (at least 1e-8 before rounding)
// as the row scale; the output row is the rotated row divided by that scale,
// zero-padded from cols to ld columns (fp32).  Replaces rotate, RMS, divide
// and pad as separate passes before the shape-gain quantizer.
constexpr int kRotThreads = 512;

__global__ void __launch_bounds__(kRotThreads) rotate_scale_kernel(const __half* __restrict__ in, int cols, int ld,
                                                                    int block, int log2b,
                                                                    const int8_t* __restrict__ signs,
                                                                    float* __restrict__ out,
                                                                    uint16_t* __restrict__ scale_out) {
  extern __shared__ float row[];
  __shared__ float red[kRotThreads / 32];
  const int64_t r = blockIdx.x;
  const __half* src = in + r * (int64_t)cols;
  for (int i = threadIdx.x; i < cols; i += kRotThreads) {
    const float v = __half2float(src[i]);
    row[i] = signs[i] < 0 ? -v : v;
  }
  __syncthreads();
  for (int st = 0; st < log2b; ++st) {
    const int h = 1 << st;
    for (int p = threadIdx.x; p < cols / 2; p += kRotThreads) {
      // pair p of the whole row: segment p / (block / 2), butterfly inside it
      const int i = ((p >> st) << (st + 1)) | (p & (h - 1));
      const float a = row[i], b = row[i + h];
      row[i] = a + b;
      row[i + h] = a - b;
    }
    __syncthreads();
  }
  const float rs = rsqrtf((float)block);
  float acc = 0.f;
  for (int i = threadIdx.x; i < cols; i += kRotThreads) {
    const float v = row[i] * rs;
    row[i] = v;
    acc = fmaf(v, v, acc);
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  float total = 0.f;
#pragma unroll
  for (int w = 0; w < kRotThreads / 32; ++w) total += red[w];
  const __half hs = __float2half_rn(fmaxf(sqrtf(total / (float)cols), 1e-8f));
  const float scale = __half2float(hs);
  if (threadIdx.x == 0) scale_out[r] = __half_as_ushort(hs);
  float* dst = out + r * (int64_t)ld;
  for (int i = threadIdx.x; i < ld; i += kRotThreads) dst[i] = i < cols ? __fdiv_rn(row[i], scale) : 0.f;
}

cudaError_t rotate_scale_launch(const void* in, int64_t rows, int64_t cols, int64_t ld, int block,
                                const int8_t* signs, float* out, uint16_t* scale_out, cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  if (block < 2 || (block & (block - 1)) || cols % block || ld < cols || rows > 0x7FFFFFFFLL)
    return cudaErrorInvalidValue;
  int log2b = 0;
  while ((1 << log2b) < block) ++log2b;
  const size_t smem = (size_t)cols * sizeof(float);
  if (smem > 200 * 1024) return cudaErrorInvalidValue;
  if (smem > 48 * 1024) {
    const cudaError_t e =
        cudaFuncSetAttribute(rotate_scale_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, 200 * 1024);
    if (e != cudaSuccess) return e;
  }
  rotate_scale_kernel<<<(unsigned)rows, kRotThreads, smem, stream>>>(static_cast<const __half*>(in), (int)cols,
                                                                      (int)ld, block, log2b, signs, out, scale_out);
  return cudaGetLastError();
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
