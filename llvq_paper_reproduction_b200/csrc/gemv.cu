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

#include <algorithm>
#include <cstdint>

#include "llvq_decode.cuh"
#include "llvq_device.cuh"
#include "llvq_internal.h"

namespace llvq {

constexpr int kGemvThreads = 256;  // 8 warps: 8 output rows per CTA

constexpr int kGemvTabThreads = 512;            // persistent table-driven grid: 2 CTAs of 16 warps per SM
constexpr int kGemvTabBlocks = 2;
constexpr size_t kGemvSmemBudget = 100 * 1024;  // shared copy of the small decoder tables

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

// One output row n by one warp: lane l decodes blocks l, l + 32, ... of the
// row (decode(v, wf): the 24 integer codeword entries as fp32), multiplies
// each by the matching activations of every batch row in fp32, then a fixed
// shuffle tree adds the lanes.
template <int MB, class Decode>
__device__ __forceinline__ void gemv_row(IndexSource index, int n, int n_out, int bpr,
                                         const uint16_t* __restrict__ rscale, const __nv_bfloat16* __restrict__ a,
                                         int m, int k, float* __restrict__ y, Decode&& decode) {
  const int lane = threadIdx.x & 31;
  float acc[MB];
#pragma unroll
  for (int i = 0; i < MB; ++i) acc[i] = 0.f;
  for (int b = lane; b < bpr && 24 * b < k; b += 32) {
    float wf[kDim];
    decode(load_index(index, (int64_t)n * bpr + b), wf);
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

// Arithmetic decoder (codebooks without tables): one warp per output row.
template <int MB>
__global__ void __launch_bounds__(kGemvThreads) gemv_decode_kernel(IndexSource index, int n_out, int bpr,
                                                                    DevBook book, const uint16_t* __restrict__ rscale,
                                                                    const __nv_bfloat16* __restrict__ a, int m, int k,
                                                                    float* __restrict__ y) {
  __shared__ DecodeShared sh;
  decode_setup(book, sh);
  __syncthreads();
  const int warp = threadIdx.x >> 5;
  const int n = blockIdx.x * (kGemvThreads / 32) + warp;
  if (n >= n_out) return;  // whole warps only, after the block's one barrier
  gemv_row<MB>(index, n, n_out, bpr, rscale, a, m, k, y, [&](int64_t v, float (&wf)[kDim]) {
    int w[kDim];
    decode_index(v, book, sh, w);
#pragma unroll
    for (int d = 0; d < kDim; ++d) wf[d] = (float)w[d];
  });
}

// Table-driven decoder: a persistent grid; each CTA copies the class and
// state records to shared memory once (MODE 2) and its warps then take
// output rows in turn.
template <int MB, int MODE>
__global__ void __launch_bounds__(kGemvTabThreads, kGemvTabBlocks) gemv_tab_kernel(IndexSource index, int n_out, int bpr, DevBook book,
                                                                 TabSmem L, const uint16_t* __restrict__ rscale,
                                                                 const __nv_bfloat16* __restrict__ a, int m, int k,
                                                                 float* __restrict__ y) {
  extern __shared__ __align__(16) uint8_t dsm[];
  DecodeSharedBase& sh = *reinterpret_cast<DecodeSharedBase*>(dsm);
  decode_setup_base(book, sh);
  if constexpr (MODE == 2) tab_smem_fill(book, dsm, L);
  __syncthreads();
  const TabCtx tc = tab_ctx<MODE == 2>(book, sh, dsm, L);
  const int warp = threadIdx.x >> 5, warps = kGemvTabThreads / 32;
  for (int n = blockIdx.x * warps + warp; n < n_out; n += gridDim.x * warps)
    gemv_row<MB>(index, n, n_out, bpr, rscale, a, m, k, y, [&](int64_t v, float (&wf)[kDim]) {
      // magnitudes to fp32 (2^23 + m minus 2^23, exact), then the sign bit
      uint32_t mag[6], neg;
      tab_decode_any<MODE == 2>(tc, v, mag, neg);
#pragma unroll
      for (int p = 0; p < kDim / 2; ++p) {
        const uint32_t mw = mag[p >> 1];
        const int j = 2 * (p & 1);
        const float2 f = __fadd2_rn(make_float2(mag_float_2p23(mw, j), mag_float_2p23(mw, j + 1)),
                                    make_float2(-8388608.0f, -8388608.0f));
        wf[2 * p] = __int_as_float(__float_as_int(f.x) ^ (int)(((neg >> (2 * p)) & 1u) << 31));
        wf[2 * p + 1] = __int_as_float(__float_as_int(f.y) ^ (int)(((neg >> (2 * p + 1)) & 1u) << 31));
      }
    });
}

cudaError_t gemv_decode_launch(const Codebook& cb, IndexSource idx, int64_t n_out, int64_t bpr,
                               const uint16_t* rscale, const void* a, int64_t m, int64_t k, float* y,
                               cudaStream_t stream) {
  if (m <= 0 || n_out <= 0) return cudaSuccess;
  if (m > kGemvMaxM) return cudaErrorInvalidValue;
  const unsigned rows_grid = (unsigned)((n_out + kGemvThreads / 32 - 1) / (kGemvThreads / 32));
  const auto* ab = static_cast<const __nv_bfloat16*>(a);
  const int n = (int)n_out, b = (int)bpr, mm = (int)m, kk = (int)k;
  if (!cb.dev.tab.state) {
#define LLVQ_GEMV(MB) gemv_decode_kernel<MB><<<rows_grid, kGemvThreads, 0, stream>>>(idx, n, b, cb.dev, rscale, ab, mm, kk, y)
    if (m == 1) LLVQ_GEMV(1);
    else if (m == 2) LLVQ_GEMV(2);
    else LLVQ_GEMV(4);
#undef LLVQ_GEMV
    return cudaGetLastError();
  }
  const TabSmem L = tab_smem_layout((int)cb.cls.size(), cb.dev.tab.n_states, kGemvSmemBudget);
  const size_t smem = L.bytes ? L.bytes : sizeof(DecodeSharedBase);
  int sms = 0;
  cudaError_t e = device_sms(&sms);
  if (e != cudaSuccess) return e;
  const unsigned grid = std::min<unsigned>((unsigned)((n_out + kGemvTabThreads / 32 - 1) / (kGemvTabThreads / 32)),
                                          (unsigned)sms * kGemvTabBlocks);
#define LLVQ_GEMV(MB, MODE)                                                                              \
  do {                                                                                                   \
    if (smem > 48 * 1024 &&                                                                              \
        (e = cudaFuncSetAttribute(gemv_tab_kernel<MB, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                                  (int)kGemvSmemBudget)) != cudaSuccess)                                 \
      return e;                                                                                          \
    gemv_tab_kernel<MB, MODE><<<grid, kGemvTabThreads, smem, stream>>>(idx, n, b, cb.dev, L, rscale, ab, mm, kk, y); \
  } while (0)
  if (L.bytes) {
    if (m == 1) LLVQ_GEMV(1, 2);
    else if (m == 2) LLVQ_GEMV(2, 2);
    else LLVQ_GEMV(4, 2);
  } else {
    if (m == 1) LLVQ_GEMV(1, 1);
    else if (m == 2) LLVQ_GEMV(2, 1);
    else LLVQ_GEMV(4, 1);
  }
#undef LLVQ_GEMV
  return cudaGetLastError();
}

}  // namespace llvq
