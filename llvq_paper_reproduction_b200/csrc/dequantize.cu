// Λ24 index -> codeword dequantizer for sm_100a.
//
// Reference: LeechLatticeVectorQuantizerGpu.dequantize / dequantize_lattice
// (impl/leech_lattice_vector_quantizer_gpu.py:267-298) and its NVRTC kernel
// (impl/llvq_cuda_dequantize.py:78-181).  One thread decodes one index in
// registers -- with the table-driven decoder (llvq_tables.cuh) when the
// codebook has tables, else by arithmetic unranking (llvq_decode.cuh) -- and
// writes it with 16-byte vector stores.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "llvq_decode.cuh"
#include "llvq_device.cuh"
#include "llvq_internal.h"

namespace llvq {

constexpr int kDeqThreads = 256;
// 5 CTAs per SM (<= 48 registers, a few bytes spilled): +6% on the Llama-3-8B
// dequant workload with the arithmetic decoder; the decode is issue-bound and
// latency-bound in turn.
constexpr int kDeqMinBlocks = 5;

// Decoder modes of the kernels: the arithmetic unranking (no tables), the
// table-driven decoder reading its class and state records from global
// memory, or from a shared-memory copy (the usual case: a persistent grid
// copies them once per CTA).
enum { kModeArith = 0, kModeTabGlobal = 1, kModeTabShared = 2 };
// Persistent table-driven kernels: 2 CTAs of 512 threads per SM (64
// registers, no spills; 768-thread CTAs at 40 registers spill and ran 7%
// slower on the Llama-3-8B dequant workload).
constexpr int kTabThreads = 512;
constexpr int kTabMinBlocks = 2;
constexpr size_t kTabSmemBudget = 100 * 1024;

// Output of one decoded block in every kind (arithmetic decoder).
template <int KIND>
__device__ __forceinline__ void store_block(const int (&y)[kDim], int64_t i, void* __restrict__ out,
                                            const uint16_t* __restrict__ row_scale, int64_t blocks_per_row,
                                            uint64_t magic_bpr) {
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

template <int KIND>
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
  const bool ok = decode_index(load_index(index, i), book, sh, y);
  if (!ok && error_count) atomicAdd(error_count, 1);
  store_block<KIND>(y, i, out, row_scale, blocks_per_row, magic_bpr);
}

// ------------------------------------------------- table-driven decoder
//
// The decoded form is the 24 magnitudes by position (mag[w], byte j =
// position 4w + j) and the mask of negative coordinates; the stores build
// every output kind from it without forming the signed integers.

// Output of one decoded index in every kind (streaming stores); row is
// i / blocks_per_row (kind 3 only).  The sign is applied last (an exact
// negation of the rounded magnitude product, since round-to-nearest is
// symmetric).
template <int KIND>
__device__ __forceinline__ void store_mn(const uint32_t (&mag)[6], uint32_t neg, int64_t i, void* __restrict__ out,
                                         const uint16_t* __restrict__ row_scale, int64_t row) {
  if constexpr (KIND == 0) {
    longlong2* o = reinterpret_cast<longlong2*>(static_cast<long long*>(out) + i * kDim);
#pragma unroll
    for (int d = 0; d < kDim; d += 2) {
      const long long a = (mag[d >> 2] >> (8 * (d & 3))) & 0xFFu, b = (mag[d >> 2] >> (8 * ((d + 1) & 3))) & 0xFFu;
      __stcs(o + d / 2, make_longlong2(((neg >> d) & 1u) ? -a : a, ((neg >> (d + 1)) & 1u) ? -b : b));
    }
  } else if constexpr (KIND == 1) {
    float4* o = reinterpret_cast<float4*>(static_cast<float*>(out) + i * kDim);
#pragma unroll
    for (int d = 0; d < kDim; d += 4) {
      float f[4];
#pragma unroll
      for (int e = 0; e < 4; ++e)
        f[e] = __int_as_float(__float_as_int(mag_scaled(mag[d >> 2], e)) ^ (int)(((neg >> (d + e)) & 1u) << 31));
      __stcs(o + d / 4, make_float4(f[0], f[1], f[2], f[3]));
    }
  } else if constexpr (KIND == 2) {
    float4* o = reinterpret_cast<float4*>(static_cast<float*>(out) + i * kDim);
#pragma unroll
    for (int d = 0; d < kDim; d += 4) {
      float f[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int m = (int)((mag[d >> 2] >> (8 * e)) & 0xFFu);
        f[e] = (float)(kLatticeScaleD * (double)(((neg >> (d + e)) & 1u) ? -m : m));
      }
      __stcs(o + d / 4, make_float4(f[0], f[1], f[2], f[3]));
    }
  } else {
    const float s = __half2float(__ushort_as_half(__ldg(row_scale + row)));
    const float2 c = make_float2(kLatticeScaleF, kLatticeScaleF), d = make_float2(-8388608.0f * kLatticeScaleF,
                                                                                  -8388608.0f * kLatticeScaleF);
    const float2 s2 = make_float2(s, s);
    uint4* o = reinterpret_cast<uint4*>(static_cast<__nv_bfloat16*>(out) + i * kDim);
#pragma unroll
    for (int q = 0; q < 3; ++q) {
      uint32_t w[4];
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const int p = 4 * q + e;  // bf16 pair p: positions 2p, 2p + 1
        const uint32_t mw = mag[p >> 1];
        const int j = 2 * (p & 1);
        // fp32(fp32(1/sqrt 8) * m) * s, two lanes per instruction
        const float2 f = __fmul2_rn(__ffma2_rn(make_float2(mag_float_2p23(mw, j), mag_float_2p23(mw, j + 1)), c, d), s2);
        w[e] = bf16_pair(f.x, f.y) ^ bf16_pair_signs(neg, p);
      }
      __stcs(o + q, make_uint4(w[0], w[1], w[2], w[3]));
    }
  }
}

// Table-driven dequantizer: a persistent grid; each CTA copies the small
// tables to shared memory once (MODE kModeTabShared) and then strides over
// the indices, loading the next index before decoding the current one.
template <int KIND, int MODE>
__global__ void __launch_bounds__(kTabThreads, kTabMinBlocks) dequant_tab_kernel(
    IndexSource index, int64_t n, DevBook book, TabSmem L, void* __restrict__ out,
    const uint16_t* __restrict__ row_scale, int64_t blocks_per_row, uint64_t magic_bpr, int* error_count) {
  extern __shared__ __align__(16) uint8_t dsm[];
  DecodeSharedBase& sh = *reinterpret_cast<DecodeSharedBase*>(dsm);
  decode_setup_base(book, sh);
  if constexpr (MODE == kModeTabShared) tab_smem_fill(book, dsm, L);
  __syncthreads();
  const TabCtx tc = tab_ctx<MODE == kModeTabShared>(book, sh, dsm, L);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t v = i < n ? load_index_stream(index, i) : 0;
  // row of index i (kind 3), advanced with the stride instead of divided
  uint64_t col, dcol;
  int64_t row = 0, drow = 0;
  if constexpr (KIND == 3) {
    row = (int64_t)div_magic((uint64_t)i, (uint64_t)blocks_per_row, magic_bpr, col);
    drow = (int64_t)div_magic((uint64_t)stride, (uint64_t)blocks_per_row, magic_bpr, dcol);
  }
  int errors = 0;
  for (; i < n; i += stride) {
    const int64_t vn = i + stride < n ? load_index_stream(index, i + stride) : 0;
    uint32_t mag[6], neg;
    if (!tab_decode_any<MODE == kModeTabShared>(tc, v, mag, neg)) ++errors;
    store_mn<KIND>(mag, neg, i, out, row_scale, row);
    if constexpr (KIND == 3) {
      row += drow;
      col += dcol;
      if (col >= (uint64_t)blocks_per_row) {
        col -= (uint64_t)blocks_per_row;
        ++row;
      }
    }
    v = vn;
  }
  if (error_count) {
    const int e = __reduce_add_sync(0xFFFFFFFFu, errors);
    if ((threadIdx.x & 31) == 0 && e) atomicAdd(error_count, e);
  }
}

// Weight staging for the large-batch GEMM: indices [rows, bpr] -> bf16
// integer codewords [rows, ldw] (columns >= 24 * bpr zero), one thread per
// (row, block) plus the padding.
__device__ __forceinline__ void store_staged(const int (&y)[kDim], __nv_bfloat16* o, int b) {
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
}

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
    decode_index(load_index(index, (int64_t)r * bpr + b), book, sh, y);
    store_staged(y, o, b);
  } else if (b == bpr) {
    for (int c = bpr * kDim; c < ldw; c += 8) *reinterpret_cast<uint4*>(o + c) = make_uint4(0, 0, 0, 0);
  }
}

// Staging decode with the table-driven decoder: the indices [rows, bpr]
// decode to bf16 integer codewords at out[r * ldw + 24 b]; columns 24 bpr ..
// ldw - 1 of every row are zeroed.
template <int MODE>
__global__ void __launch_bounds__(kTabThreads, kTabMinBlocks) decode_rows_tab_kernel(
    IndexSource index, int rows, int bpr, int ldw, DevBook book, TabSmem L, __nv_bfloat16* __restrict__ out,
    uint64_t magic_bpr) {
  extern __shared__ __align__(16) uint8_t dsm[];
  DecodeSharedBase& sh = *reinterpret_cast<DecodeSharedBase*>(dsm);
  decode_setup_base(book, sh);
  if constexpr (MODE == kModeTabShared) tab_smem_fill(book, dsm, L);
  const int64_t stride = (int64_t)gridDim.x * blockDim.x;
  const int pad = (ldw - bpr * kDim) / 8;  // 16-byte groups of zero padding per row
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < (int64_t)rows * pad; i += stride) {
    const int64_t r = i / pad, c = i - r * pad;
    *reinterpret_cast<uint4*>(out + r * ldw + bpr * kDim + c * 8) = make_uint4(0, 0, 0, 0);
  }
  __syncthreads();
  const TabCtx tc = tab_ctx<MODE == kModeTabShared>(book, sh, dsm, L);
  const int64_t n = (int64_t)rows * bpr;
  int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  int64_t v = i < n ? load_index_stream(index, i) : 0;
  for (; i < n; i += stride) {
    const int64_t vn = i + stride < n ? load_index_stream(index, i + stride) : 0;
    uint32_t mag[6], neg;
    tab_decode_any<MODE == kModeTabShared>(tc, v, mag, neg);
    uint64_t b;
    const uint64_t r = div_magic((uint64_t)i, (uint64_t)bpr, magic_bpr, b);
    uint4* o = reinterpret_cast<uint4*>(out + r * ldw + b * kDim);
    uint32_t w[12];
    bf16_codeword(mag, neg, w);
#pragma unroll
    for (int q = 0; q < 3; ++q) o[q] = make_uint4(w[4 * q], w[4 * q + 1], w[4 * q + 2], w[4 * q + 3]);
    v = vn;
  }
}

// Launch shape of the table-driven kernels for a codebook: the shared copy
// when it fits, a persistent grid of at most kTabMinBlocks CTAs per SM.
struct TabLaunch {
  int mode;
  TabSmem L;
  size_t smem;
};

TabLaunch tab_launch(const Codebook& cb) {
  TabLaunch t;
  t.L = tab_smem_layout((int)cb.cls.size(), cb.dev.tab.n_states, kTabSmemBudget);
  t.mode = t.L.bytes ? kModeTabShared : kModeTabGlobal;
  t.smem = t.L.bytes ? t.L.bytes : sizeof(DecodeSharedBase);
  return t;
}

template <class K>
static cudaError_t allow_smem(K kernel, size_t bytes) {
  // above the 48 KB default: raise the kernel's limit (idempotent)
  if (bytes <= 48 * 1024) return cudaSuccess;
  return cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTabSmemBudget);
}

static unsigned tab_grid(int64_t work) {
  int sms = 0;
  if (device_sms(&sms) != cudaSuccess || sms <= 0) sms = 148;
  const int64_t blocks = (work + kTabThreads - 1) / kTabThreads;
  return (unsigned)std::max<int64_t>(1, std::min<int64_t>(blocks, (int64_t)sms * kTabMinBlocks));
}

cudaError_t decode_rows_bf16_launch(const Codebook& cb, IndexSource index, int rows, int bpr, int ldw, void* out,
                                    cudaStream_t stream) {
  if (rows <= 0) return cudaSuccess;
  auto* o = static_cast<__nv_bfloat16*>(out);
  if (cb.dev.tab.state) {
    const TabLaunch t = tab_launch(cb);
    const unsigned grid = tab_grid((int64_t)rows * bpr);
    const uint64_t magic = ~0ull / (uint64_t)bpr;
    cudaError_t e;
    if (t.mode == kModeTabShared) {
      if ((e = allow_smem(decode_rows_tab_kernel<kModeTabShared>, t.smem)) != cudaSuccess) return e;
      decode_rows_tab_kernel<kModeTabShared><<<grid, kTabThreads, t.smem, stream>>>(index, rows, bpr, ldw, cb.dev,
                                                                                  t.L, o, magic);
    } else {
      decode_rows_tab_kernel<kModeTabGlobal><<<grid, kTabThreads, t.smem, stream>>>(index, rows, bpr, ldw, cb.dev,
                                                                                  t.L, o, magic);
    }
  } else {
    const int64_t n = (int64_t)rows * (ldw / kDim + 1);
    decode_rows_bf16_kernel<<<(unsigned)((n + kDeqThreads - 1) / kDeqThreads), kDeqThreads, 0, stream>>>(
        index, rows, bpr, ldw, cb.dev, o, ~0ull / (uint64_t)(ldw / kDim + 1));
  }
  return cudaGetLastError();
}

template <int KIND>
static cudaError_t dequantize_kind(const Codebook& cb, IndexSource index, int64_t n, void* out,
                                   const uint16_t* row_scale, int64_t blocks_per_row, uint64_t magic_bpr,
                                   int* error_count, cudaStream_t stream) {
  if (cb.dev.tab.state) {
    const TabLaunch t = tab_launch(cb);
    const unsigned grid = tab_grid(n);
    if (t.mode == kModeTabShared) {
      const cudaError_t e = allow_smem(dequant_tab_kernel<KIND, kModeTabShared>, t.smem);
      if (e != cudaSuccess) return e;
      dequant_tab_kernel<KIND, kModeTabShared><<<grid, kTabThreads, t.smem, stream>>>(
          index, n, cb.dev, t.L, out, row_scale, blocks_per_row, magic_bpr, error_count);
    } else {
      dequant_tab_kernel<KIND, kModeTabGlobal><<<grid, kTabThreads, t.smem, stream>>>(
          index, n, cb.dev, t.L, out, row_scale, blocks_per_row, magic_bpr, error_count);
    }
  } else {
    const unsigned blocks = (unsigned)((n + kDeqThreads - 1) / kDeqThreads);
    dequant_kernel<KIND><<<blocks, kDeqThreads, 0, stream>>>(index, n, cb.dev, out, row_scale, blocks_per_row,
                                                             magic_bpr, error_count);
  }
  return cudaGetLastError();
}

cudaError_t dequantize_launch(const Codebook& cb, IndexSource index, int64_t n, void* out, int kind,
                              const uint16_t* row_scale, int64_t blocks_per_row, int* error_count,
                              cudaStream_t stream) {
  if (n <= 0) return cudaSuccess;
  const uint64_t magic_bpr = ~0ull / (uint64_t)(blocks_per_row > 0 ? blocks_per_row : 1);
  switch (kind) {
    case 0: return dequantize_kind<0>(cb, index, n, out, row_scale, blocks_per_row, magic_bpr, error_count, stream);
    case 1: return dequantize_kind<1>(cb, index, n, out, row_scale, blocks_per_row, magic_bpr, error_count, stream);
    case 2: return dequantize_kind<2>(cb, index, n, out, row_scale, blocks_per_row, magic_bpr, error_count, stream);
    case 3: return dequantize_kind<3>(cb, index, n, out, row_scale, blocks_per_row, magic_bpr, error_count, stream);
    default: return cudaErrorInvalidValue;
  }
}

// ------------------------------------------------------- packed indices

__global__ void pack_kernel(const int64_t* __restrict__ in, int64_t n, int bytes, uint8_t* __restrict__ out,
                            int* error_count) {
  const int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (i >= n) return;
  const uint64_t ones = ~0ull >> (64 - 8 * bytes);
  const int64_t v = in[i];
  uint64_t u = (uint64_t)v;
  // -1 and anything that does not fit become all-ones; with 8 bytes every
  // other value is an (unsigned) index
  if (bytes < 8 ? (v < 0 || u >= ones) : u == ones) {
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
