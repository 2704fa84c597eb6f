// Dequant-GEMM for a few activation rows (m <= kGemvMaxM): the weights are
// decoded straight into registers and multiplied there, with no bf16 staging.
//
// At batch sizes this small the dequant-GEMM is bound by the decode (about
// 1.6 k instructions per 24-weight block), not by the tensor cores; the
// staged path would add a 48-byte write and read of every block and a second
// launch.  One warp computes one output row n: lane l decodes the row's
// blocks l, l + 32, ... (llvq_decode.cuh), multiplies each by the matching
// 24 activations of every batch row in fp32, and the lanes' partial sums are
// added by a fixed shuffle tree, so every output has one summation order
// (the same result on every call).  Y[m, n] = (sum_k A[m, k] * codeword[k])
// * fp32(1/sqrt 8) * row_scale[n], the epilogue of the staged path.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstdint>

#include "llvq_decode.cuh"
#include "llvq_device.cuh"
#include "llvq_internal.h"

namespace llvq {

constexpr int kGemvThreads = 256;  // 8 warps: 8 output rows per CTA

// acc += dot(8 bf16 activations, w[0..7])
__device__ __forceinline__ float dot8(uint4 v, const float* w, float acc) {
  const uint32_t u[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int e = 0; e < 4; ++e) {
    const float2 f = __bfloat1622float2(*reinterpret_cast<const __nv_bfloat162*>(&u[e]));
    acc = fmaf(f.x, w[2 * e], acc);
    acc = fmaf(f.y, w[2 * e + 1], acc);
  }
  return acc;
}

template <int MB, bool TAB>
__global__ void __launch_bounds__(kGemvThreads) gemv_decode_kernel(IndexSource index, int n_out, int bpr,
                                                                    DevBook book, const uint16_t* __restrict__ rscale,
                                                                    const __nv_bfloat16* __restrict__ a, int m, int k,
                                                                    float* __restrict__ y) {
  __shared__ DecodeShared sh;
  decode_setup(book, sh);
  __syncthreads();
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int n = blockIdx.x * (kGemvThreads / 32) + warp;
  if (n >= n_out) return;  // whole warps only, after the block's one barrier
  float acc[MB];
#pragma unroll
  for (int i = 0; i < MB; ++i) acc[i] = 0.f;
  for (int b = lane; b < bpr && 24 * b < k; b += 32) {
    int w[kDim];
    decode_any<TAB>(load_index(index, (int64_t)n * bpr + b), book, sh, w);
    float wf[kDim];
#pragma unroll
    for (int d = 0; d < kDim; ++d) wf[d] = (float)w[d];
    const int c0 = 24 * b, valid = min(kDim, k - c0);  // 8, 16 or 24: k is a multiple of 8
#pragma unroll
    for (int i = 0; i < MB; ++i) {
      if (i < m) {
        const uint4* ap = reinterpret_cast<const uint4*>(a + (int64_t)i * k + c0);  // 16-byte aligned
        float s = acc[i];
        s = dot8(__ldg(ap), wf, s);
        if (valid > 8) s = dot8(__ldg(ap + 1), wf + 8, s);
        if (valid > 16) s = dot8(__ldg(ap + 2), wf + 16, s);
        acc[i] = s;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < MB; ++i)
#pragma unroll
    for (int o = 16; o; o >>= 1) acc[i] += __shfl_xor_sync(0xffffffffu, acc[i], o);
  if (lane == 0) {
    float scale = kLatticeScaleF;
    if (rscale) scale = __fmul_rn(kLatticeScaleF, __half2float(__ushort_as_half(rscale[n])));
#pragma unroll
    for (int i = 0; i < MB; ++i)
      if (i < m) y[(int64_t)i * n_out + n] = acc[i] * scale;
  }
}

cudaError_t gemv_decode_launch(const Codebook& cb, IndexSource idx, int64_t n_out, int64_t bpr,
                               const uint16_t* rscale, const void* a, int64_t m, int64_t k, float* y,
                               cudaStream_t stream) {
  if (m <= 0 || n_out <= 0) return cudaSuccess;
  if (m > kGemvMaxM) return cudaErrorInvalidValue;
  const unsigned grid = (unsigned)((n_out + kGemvThreads / 32 - 1) / (kGemvThreads / 32));
  const auto* ab = static_cast<const __nv_bfloat16*>(a);
  const int n = (int)n_out, b = (int)bpr, mm = (int)m, kk = (int)k;
  const bool tab = cb.dev.tab.state != nullptr;
#define LLVQ_GEMV(MB)                                                                                      \
  (tab ? gemv_decode_kernel<MB, true><<<grid, kGemvThreads, 0, stream>>>(idx, n, b, cb.dev, rscale, ab, mm, \
                                                                          kk, y)                           \
       : gemv_decode_kernel<MB, false><<<grid, kGemvThreads, 0, stream>>>(idx, n, b, cb.dev, rscale, ab, mm, \
                                                                           kk, y))
  if (m == 1)
    LLVQ_GEMV(1);
  else if (m == 2)
    LLVQ_GEMV(2);
  else
    LLVQ_GEMV(4);
#undef LLVQ_GEMV
  return cudaGetLastError();
}

}  // namespace llvq
