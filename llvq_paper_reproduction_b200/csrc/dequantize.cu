// Λ24 index -> codeword dequantizer for sm_100a.
//
// Reference: LeechLatticeVectorQuantizerGpu.dequantize / dequantize_lattice
// (impl/leech_lattice_vector_quantizer_gpu.py:267-298) and its NVRTC kernel
// (impl/llvq_cuda_dequantize.py:78-181).  One thread decodes one index in
// registers (llvq_decode.cuh) and writes it with 16-byte vector stores.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "llvq_decode.cuh"
#include "llvq_device.cuh"
#include "llvq_internal.h"

namespace llvq {

constexpr int kDeqThreads = 256;
// 5 CTAs per SM (<= 48 registers, a few bytes spilled): +6% on the Llama-3-8B
// dequant workload; the decode is issue-bound and latency-bound in turn.
constexpr int kDeqMinBlocks = 5;

template <int KIND, bool TAB>
__global__ void __launch_bounds__(kDeqThreads, kDeqMinBlocks) dequant_kernel(IndexSource index, int64_t n,
                                                              DevBook book, void* __restrict__ out,
                                                              const uint16_t* __restrict__ row_scale,
                                                              int64_t blocks_per_row, uint64_t magic_bpr,
                                                              int* error_count) {
  __shared__ DecodeShared sh;
  decode_setup(book, sh);
  __syncthreads();
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  int y[kDim];
  const bool ok = decode_any<TAB>(load_index(index, i), book, sh, y);
  if (!ok && error_count) atomicAdd(error_count, 1);
  if constexpr (KIND == 0) {
    longlong2* o = reinterpret_cast<longlong2*>(static_cast<long long*>(out) + i * kDim);
#pragma unroll
    for (int d = 0; d < kDim; d += 2) o[d / 2] = make_longlong2(y[d], y[d + 1]);
  } else if constexpr (KIND == 1 || KIND == 2) {
    float4* o = reinterpret_cast<float4*>(static_cast<float*>(out) + i * kDim);
    float f[kDim];
#pragma unroll
    for (int d = 0; d < kDim; ++d) {
      // KIND 1: fp32(1/sqrt 8) * fp32(k) rounded to fp32 (the GPU API's torch
      // multiply); KIND 2: the double product rounded to fp32 (CPU API).
      f[d] = KIND == 1 ? __fmul_rn(kLatticeScaleF, (float)y[d]) : (float)(kLatticeScaleD * (double)y[d]);
    }
#pragma unroll
    for (int d = 0; d < kDim; d += 4) o[d / 4] = make_float4(f[d], f[d + 1], f[d + 2], f[d + 3]);
  } else {
    uint64_t col;  // row = i / blocks_per_row by multiply-high with an exact correction
    const uint64_t row = div_magic((uint64_t)i, (uint64_t)blocks_per_row, magic_bpr, col);
    const float s = __half2float(__ushort_as_half(row_scale[row]));
    uint4* o = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + i * kDim);
    uint32_t w[kDim / 2];
#pragma unroll
    for (int d = 0; d < kDim; d += 2) {
      const float a = __fmul_rn(__fmul_rn(kLatticeScaleF, (float)y[d]), s);
      const float b = __fmul_rn(__fmul_rn(kLatticeScaleF, (float)y[d + 1]), s);
      const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
      w[d / 2] = *reinterpret_cast<const uint32_t*>(&h);
    }
#pragma unroll
    for (int d = 0; d < kDim / 2; d += 4) o[d / 4] = make_uint4(w[d], w[d + 1], w[d + 2], w[d + 3]);
  }
}

// Weight staging for the large-batch GEMM: indices [rows, bpr] -> bf16
// integer codewords [rows, ldw] (columns >= 24 * bpr zero), one thread per
// (row, block) plus the padding.
template <bool TAB>
__global__ void __launch_bounds__(kDeqThreads) decode_rows_bf16_kernel(IndexSource index, int rows,
                                                                       int bpr, int ldw, DevBook book,
                                                                       __nv_bfloat16* __restrict__ out, uint64_t magic_per_row) {
  __shared__ DecodeShared sh;
  decode_setup(book, sh);
  __syncthreads();
  const int per_row = ldw / kDim + 1;  // bpr blocks, then zero padding of the row tail
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= (int64_t)rows * per_row) return;
  uint64_t bq;
  const int r = (int)div_magic((uint64_t)i, (uint64_t)per_row, magic_per_row, bq), b = (int)bq;
  __nv_bfloat16* o = out + (int64_t)r * ldw;
  if (b < bpr) {
    int y[kDim];
    decode_any<TAB>(load_index(index, (int64_t)r * bpr + b), book, sh, y);
    uint4* dst = reinterpret_cast<uint4*>(o + b * kDim);
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      uint32_t pk[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const __nv_bfloat162 h = __floats2bfloat162_rn((float)y[q * 8 + 2 * e], (float)y[q * 8 + 2 * e + 1]);
        pk[e] = *reinterpret_cast<const uint32_t*>(&h);
      }
      dst[q] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
    }
  } else if (b == bpr) {
    for (int c = bpr * kDim; c < ldw; c += 8) *reinterpret_cast<uint4*>(o + c) = make_uint4(0, 0, 0, 0);
  }
}

cudaError_t decode_rows_bf16_launch(const Codebook& cb, IndexSource index, int rows, int bpr, int ldw, void* out,
                                    cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  const int64_t n = (int64_t)rows * (ldw / kDim + 1);
  const unsigned grid = (unsigned)((n + kDeqThreads - 1) / kDeqThreads);
  const uint64_t magic = ~0ull / (uint64_t)(ldw / kDim + 1);
  if (cb.dev.tab.state)
    decode_rows_bf16_kernel<true><<<grid, kDeqThreads, 0, stream>>>(index, rows, bpr, ldw, cb.dev,
                                                                     static_cast<__nv_bfloat16*>(out), magic);
  else
    decode_rows_bf16_kernel<false><<<grid, kDeqThreads, 0, stream>>>(index, rows, bpr, ldw, cb.dev,
                                                                      static_cast<__nv_bfloat16*>(out), magic);
  return cudaGetLastError();
}

cudaError_t dequantize_launch(const Codebook& cb, IndexSource index, int64_t n, void* out, int kind,
                              const uint16_t* row_scale, int64_t blocks_per_row, int* error_count,
                              cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  const unsigned blocks = (unsigned)((n + kDeqThreads - 1) / kDeqThreads);
  const uint64_t magic_bpr = ~0ull / (uint64_t)(blocks_per_row > 0 ? blocks_per_row : 1);
  const bool tab = cb.dev.tab.state != nullptr;
#define LLVQ_DEQ(K)                                                                                            \
  (tab ? dequant_kernel<K, true><<<blocks, kDeqThreads, 0, stream>>>(index, n, cb.dev, out, row_scale,          \
                                                                      blocks_per_row, magic_bpr, error_count)  \
       : dequant_kernel<K, false><<<blocks, kDeqThreads, 0, stream>>>(index, n, cb.dev, out, row_scale,         \
                                                                       blocks_per_row, magic_bpr, error_count))
  switch (kind) {
    case 0: LLVQ_DEQ(0); break;
    case 1: LLVQ_DEQ(1); break;
    case 2: LLVQ_DEQ(2); break;
    case 3: LLVQ_DEQ(3); break;
    default: return cudaErrorInvalidValue;
  }
#undef LLVQ_DEQ
  return cudaGetLastError();
}

// ------------------------------------------------------- packed indices

__global__ void pack_kernel(const int64_t* __restrict__ in, int64_t n, int bytes, uint8_t* __restrict__ out,
                            int* error_count) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint64_t ones = ~0ull >> (64 - 8 * bytes);
  const int64_t v = in[i];
  uint64_t u = (uint64_t)v;
  if (v < 0 || u >= ones) {  // -1 and anything that does not fit become all-ones
    if (v != -1 && error_count) atomicAdd(error_count, 1);
    u = ones;
  }
  uint8_t* o = out + i * bytes;
  for (int k = 0; k < bytes; ++k) o[k] = (uint8_t)(u >> (8 * k));
}

__global__ void unpack_kernel(const uint8_t* __restrict__ in, int64_t n, int bytes, int64_t* __restrict__ out) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  out[i] = load_index(IndexSource{in, bytes}, i);
}

cudaError_t pack_indices_launch(const int64_t* in, int64_t n, int bytes, uint8_t* out, int* error_count,
                                cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  pack_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(in, n, bytes, out, error_count);
  return cudaGetLastError();
}

cudaError_t unpack_indices_launch(const uint8_t* in, int64_t n, int bytes, int64_t* out, cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  unpack_kernel<<<(unsigned)((n + 255) / 256), 256, 0, stream>>>(in, n, bytes, out);
  return cudaGetLastError();
}

}  // namespace llvq
