// Fused Λ24 dequant-GEMM for sm_100a (tcgen05 tensor cores, TMEM accumulators).
//
//   Y[m, n] = sum_k A[m, k] * W[n, k],   W[n, :] = row_scale[n] * fp32(1/sqrt 8) * codeword(indices[n, :])
//
// The weights are never materialised in HBM: each CTA decodes a 128-row x
// 192-column weight tile (8 indices per row) straight into shared memory in
// the 128-byte-swizzled K-major layout the tensor core reads, as bf16 copies
// of the integer codeword entries (|k| <= 22 here, exact in bf16).  The
// activation tile (bf16, up to 256 rows) is staged the same way.  One thread
// issues tcgen05.mma (M = 128 weight rows, N = activation rows, K = 16 per
// instruction, fp32 accumulation in TMEM) and commits to an mbarrier; the
// per-row scale fp32(1/sqrt 8) * row_scale[n] is applied in the epilogue, so
// the only rounding beyond fp32 accumulation is that of the bf16 activations
// themselves.  The output is written transposed from TMEM (lane = weight row,
// column = activation row), coalesced along n.
//
// Work items (weight-row tile, K split, activation pass) are spread over a
// persistent grid; with more than one K split the partial products are added
// into Y (zeroed first) with fp32 atomics.  More than 256 activation rows are
// handled in passes that decode the tile again.
//
// The reference has no GEMM (its dequantizer returns int64 codewords,
// impl/llvq_cuda_dequantize.py:78-181); the decode is the same index layout.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>

#include "llvq_decode.cuh"
#include "llvq_device.cuh"
#include "llvq_internal.h"
#include "tcgen05.cuh"

namespace llvq {

constexpr int kGemmThreads = 256;
constexpr int kTileW = 128;       // weight rows per tile (MMA M)
constexpr int kChunkBlocks = 8;   // 24-D blocks per K chunk
constexpr int kChunkK = 192;      // = 3 swizzle atoms of 64 bf16
constexpr int kAtoms = 3;
constexpr int kMaxAct = 256;      // activation rows per pass (MMA N)
constexpr uint32_t kWaitLimit = 1u << 22;

// Dynamic shared memory, 1024-byte aligned: the weight tile (3 atoms of
// 128 rows x 128 B), the activation tile (3 atoms of npad rows x 128 B, sized
// to the batch so small batches fit several CTAs per SM), the decode tables,
// the mbarrier and the TMEM address.
struct GemmLayout {
  uint32_t a_off, a_atom, dec_off, mbar_off, holder_off, bytes;
  __host__ __device__ explicit GemmLayout(int npad) {
    a_off = kAtoms * kTileW * 128;
    a_atom = (uint32_t)npad * 128;
    dec_off = a_off + kAtoms * a_atom;
    mbar_off = (dec_off + (uint32_t)sizeof(DecodeShared) + 15u) & ~15u;
    holder_off = mbar_off + 8;
    bytes = holder_off + 8 + 1024;  // + slack for aligning the base
  }
};

__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

__global__ void __launch_bounds__(kGemmThreads, 2)
    gemm_kernel(DevBook book, const int64_t* __restrict__ idx, int n_out, int bpr, const uint16_t* __restrict__ rscale,
                const __nv_bfloat16* __restrict__ A, int m_act, int k_in, float* __restrict__ Y, int splits,
                int passes, int npad, int* error_flag) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  const GemmLayout L(npad);
  uint8_t* wt = base;
  uint8_t* at = base + L.a_off;
  DecodeShared& dec = *reinterpret_cast<DecodeShared*>(base + L.dec_off);
  uint64_t* mbar_p = reinterpret_cast<uint64_t*>(base + L.mbar_off);
  uint32_t* holder = reinterpret_cast<uint32_t*>(base + L.holder_off);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;

  decode_setup(book, dec);
  if (tid == 0) {
    tc::mbar_init(tc::smem_addr(mbar_p), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  uint32_t ncols = 32;
  while ((int)ncols < npad) ncols <<= 1;
  if (warp == 0) tc::tmem_alloc(tc::smem_addr(holder), ncols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *holder;
  const uint32_t idesc = tc::idesc_bf16_f32(kTileW, npad);
  const uint32_t mbar = tc::smem_addr(mbar_p);
  const uint32_t w_base = tc::smem_addr(wt);
  const uint32_t a_base = tc::smem_addr(at);
  const float lscale = kLatticeScaleF;

  const int n_tiles = (n_out + kTileW - 1) / kTileW;
  const int chunks = (bpr + kChunkBlocks - 1) / kChunkBlocks;
  const int items = n_tiles * splits * passes;
  uint32_t phase = 0;
  bool failed = false;

  for (int item = blockIdx.x; item < items && !failed; item += gridDim.x) {
    const int pass = item % passes;
    const int split = (item / passes) % splits;
    const int tile = item / (passes * splits);
    const int n0 = tile * kTileW;
    const int c_begin = (int)((long long)chunks * split / splits);
    const int c_end = (int)((long long)chunks * (split + 1) / splits);
    const int m0 = pass * kMaxAct;
    for (int c = c_begin; c < c_end; ++c) {
      // weights: 128 rows x 8 indices, decoded into the swizzled tile
      for (int slot = tid; slot < kTileW * kChunkBlocks; slot += kGemmThreads) {
        const int r = slot >> 3, b = slot & 7;
        const int gb = c * kChunkBlocks + b;
        int y[kDim];
        if (n0 + r < n_out && gb < bpr) {
          decode_index(__ldg(idx + (int64_t)(n0 + r) * bpr + gb), book, dec, y);
        } else {
#pragma unroll
          for (int d = 0; d < kDim; ++d) y[d] = 0;
        }
#pragma unroll
        for (int q = 0; q < 3; ++q) {
          const int kk = b * kDim + q * 8;  // column inside the chunk, multiple of 8
          uint32_t pk[4];
#pragma unroll
          for (int e = 0; e < 4; ++e) {
            const __nv_bfloat162 h = __floats2bfloat162_rn((float)y[q * 8 + 2 * e], (float)y[q * 8 + 2 * e + 1]);
            pk[e] = *reinterpret_cast<const uint32_t*>(&h);
          }
          *reinterpret_cast<uint4*>(wt + (kk >> 6) * (kTileW * 128) + swz(r, (kk & 63) >> 3)) =
              make_uint4(pk[0], pk[1], pk[2], pk[3]);
        }
      }
      // activations: npad rows x 192 columns (zero outside [0, m_act) x [0, k_in))
      for (int u = tid; u < npad * (kChunkK / 8); u += kGemmThreads) {
        const int m = u / (kChunkK / 8), kc = u % (kChunkK / 8);
        const int kg = c * kChunkK + kc * 8;
        uint4 val = make_uint4(0, 0, 0, 0);
        if (m0 + m < m_act && kg < k_in)
          val = __ldg(reinterpret_cast<const uint4*>(A + (int64_t)(m0 + m) * k_in + kg));
        *reinterpret_cast<uint4*>(at + (kc >> 3) * L.a_atom + swz(m, kc & 7)) = val;
      }
      tc::fence_proxy_async();
      __syncthreads();
      if (tid == 0) {
        tc::fence_after_sync();
#pragma unroll
        for (int ks = 0; ks < kChunkK / 16; ++ks) {
          const int k = ks * 16;
          const uint32_t off = (uint32_t)((k & 63) * 2);
          const uint64_t ad = tc::desc_sw128(w_base + (uint32_t)(k >> 6) * (kTileW * 128) + off);
          const uint64_t bd = tc::desc_sw128(a_base + (uint32_t)(k >> 6) * L.a_atom + off);
          tc::mma_bf16(tmem, ad, bd, idesc, (c > c_begin || ks > 0) ? 1u : 0u);
        }
        tc::commit(mbar);
      }
      const bool done = tc::mbar_wait(mbar, phase, kWaitLimit);
      phase ^= 1;
      failed = __syncthreads_or(!done) != 0;  // block-uniform decision
      if (failed) {
        if (tid == 0 && error_flag) atomicExch(error_flag, 1);
        break;
      }
    }
    if (failed) break;
    // epilogue: TMEM lane = weight row, column = activation row
    tc::fence_after_sync();
    const int q = warp & 3, half = warp >> 2;
    const int r = q * 32 + lane, n = n0 + r;
    float scale = lscale;
    if (rscale && n < n_out) scale = __fmul_rn(lscale, __half2float(__ushort_as_half(rscale[n])));
    for (int col0 = half * 16; col0 < npad; col0 += 32) {
      float v[16];
      tc::tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)col0, v);
      if (n < n_out) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m0 + col0 + j;
          if (m < m_act && col0 + j < npad) {
            float* dst = Y + (int64_t)m * n_out + n;
            if (splits > 1) atomicAdd(dst, v[j] * scale);
            else *dst = v[j] * scale;
          }
        }
      }
    }
    tc::fence_before_sync();
    __syncthreads();
  }
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, ncols);
}

cudaError_t gemm_launch(const Codebook& cb, const int64_t* idx, int64_t n_out, int64_t bpr, const uint16_t* rscale,
                        const void* a, int64_t m, int64_t k, float* y, int* error_flag, cudaStream_t stream) {
  if (m <= 0 || n_out <= 0) return cudaSuccess;
  static bool configured = false;
  static int sms = 0;
  if (!configured) {
    int dev;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cudaError_t e = cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                         (int)GemmLayout(kMaxAct).bytes);
    if (e != cudaSuccess) return e;
    configured = true;
  }
  const int passes = (int)((m + kMaxAct - 1) / kMaxAct);
  const int rows_last = (int)std::min<int64_t>(m, kMaxAct);
  const int npad = std::max(16, (rows_last + 15) / 16 * 16);
  const int n_tiles = (int)((n_out + kTileW - 1) / kTileW);
  const int chunks = (int)((bpr + kChunkBlocks - 1) / kChunkBlocks);
  const GemmLayout L(npad);
  int per_sm = 1;
  cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, gemm_kernel, kGemmThreads, L.bytes);
  per_sm = std::max(1, per_sm);
  const int slots = sms * per_sm;
  int splits = std::max(1, std::min(chunks, (slots + n_tiles * passes - 1) / (n_tiles * passes)));
  if (splits > 1) {
    cudaError_t e = cudaMemsetAsync(y, 0, (size_t)m * (size_t)n_out * sizeof(float), stream);
    if (e != cudaSuccess) return e;
  }
  const int items = n_tiles * splits * passes;
  const int grid = std::min(items, slots);
  gemm_kernel<<<grid, kGemmThreads, L.bytes, stream>>>(cb.dev, idx, (int)n_out, (int)bpr, rscale,
                                                        static_cast<const __nv_bfloat16*>(a), (int)m, (int)k, y,
                                                        splits, passes, npad, error_flag);
  return cudaGetLastError();
}

}  // namespace llvq
