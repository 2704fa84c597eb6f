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

// ------------------------------------------------------------ large batches
//
// For batches above one pass (256 rows) the weights are first decoded once
// per row chunk into a bf16 staging buffer sized to stay in L2 (integer
// codeword entries, rows padded to a multiple of 64 columns), then a
// pipelined tcgen05 GEMM streams both operands: kStages shared-memory stages
// of 64 columns (weights 128 rows, activations 256 rows), filled with 16-byte
// cp.async copies into the 128-byte-swizzled layout (zero-filled outside the
// matrices), one thread issuing 4 MMAs (M=128, N=256, K=16) per stage and
// committing to that stage's mbarrier, which also tells the loaders when the
// stage may be overwritten.  256 TMEM columns hold the fp32 accumulators.

constexpr int kStages = 4;
constexpr int kStageW = kTileW * 128;           // 16 KB
constexpr int kStageA = kMaxAct * 128;          // 32 KB
constexpr int kStageBytes = kStageW + kStageA;  // 48 KB
constexpr size_t kStagedSmem = (size_t)kStages * kStageBytes + 64 + 1024;

__device__ __forceinline__ void cp_async16(uint32_t dst, const void* src, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(dst), "l"(src), "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() { asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory"); }

__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_staged_kernel(const __nv_bfloat16* __restrict__ Wk, int ldw, int w_rows, int n_base, int n_out,
                       const uint16_t* __restrict__ rscale, const __nv_bfloat16* __restrict__ A, int m_act, int k_in,
                       float* __restrict__ Y, int* error_flag) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* mbars = reinterpret_cast<uint64_t*>(base + kStages * kStageBytes);
  uint32_t* holder = reinterpret_cast<uint32_t*>(base + kStages * kStageBytes + 8 * kStages);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int st = 0; st < kStages; ++st) tc::mbar_init(tc::smem_addr(&mbars[st]), 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tc::tmem_alloc(tc::smem_addr(holder), kMaxAct);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *holder;
  const uint32_t idesc = tc::idesc_bf16_f32(kTileW, kMaxAct);
  const uint32_t sbase = tc::smem_addr(base);
  const int kc_total = ldw / 64;
  const int tn = (w_rows + kTileW - 1) / kTileW, tm = (m_act + kMaxAct - 1) / kMaxAct;
  uint32_t phase = 0;  // bit st = parity of stage st's next completion
  bool failed = false;


  for (int item = blockIdx.x; item < tn * tm && !failed; item += gridDim.x) {
    const int row0 = (item / tm) * kTileW, m0 = (item % tm) * kMaxAct;
    auto issue = [&](int c) {
      const int st = c % kStages;
      const uint32_t sw = sbase + st * kStageBytes, sa = sw + kStageW;
      const int kb = c * 64;
      for (int u = tid; u < kTileW * 8; u += kGemmThreads) {
        const int r = u >> 3, c8 = u & 7;
        const bool ok = row0 + r < w_rows;
        const __nv_bfloat16* src = Wk + (int64_t)(ok ? row0 + r : 0) * ldw + kb + c8 * 8;
        cp_async16(sw + swz(r, c8), src, ok);
      }
      for (int u = tid; u < kMaxAct * 8; u += kGemmThreads) {
        const int r = u >> 3, c8 = u & 7;
        const int kg = kb + c8 * 8;
        const bool ok = m0 + r < m_act && kg < k_in;
        const __nv_bfloat16* src = A + (ok ? (int64_t)(m0 + r) * k_in + kg : 0);
        cp_async16(sa + swz(r, c8), src, ok);
      }
    };
    // prologue: the first kStages-1 stages in flight
    for (int c = 0; c < kStages - 1; ++c) {
      if (c < kc_total) issue(c);
      cp_async_commit();
    }
    uint32_t pending = 0;  // stages whose MMA commit has not been waited for
    for (int c = 0; c < kc_total; ++c) {
      const int nxt = c + kStages - 1;
      if (nxt < kc_total) {
        const int st = nxt % kStages;
        if ((pending >> st) & 1u) {  // the MMA that read this stage must be done
          const bool ok = tc::mbar_wait(tc::smem_addr(&mbars[st]), (phase >> st) & 1u, kWaitLimit);
          phase ^= 1u << st;
          pending &= ~(1u << st);
          if (!ok) failed = true;
        }
        if (!failed) issue(nxt);
      }
      cp_async_commit();
      cp_async_wait<kStages - 1>();
      tc::fence_proxy_async();
      if (__syncthreads_or(failed)) {
        failed = true;
        break;
      }
      const int st = c % kStages;
      if (tid == 0) {
        tc::fence_after_sync();
        const uint32_t sw = sbase + st * kStageBytes, sa = sw + kStageW;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          tc::mma_bf16(tmem, tc::desc_sw128(sw + ks * 32), tc::desc_sw128(sa + ks * 32), idesc,
                       (c > 0 || ks > 0) ? 1u : 0u);
        }
        tc::commit(tc::smem_addr(&mbars[st]));
      }
      pending |= 1u << st;
    }
    cp_async_wait<0>();
    // drain: wait for every outstanding stage commit (the last one covers all MMAs)
    for (int st = 0; st < kStages; ++st) {
      if ((pending >> st) & 1u) {
        const bool ok = tc::mbar_wait(tc::smem_addr(&mbars[st]), (phase >> st) & 1u, kWaitLimit);
        phase ^= 1u << st;
        if (!ok) failed = true;
      }
    }
    if (__syncthreads_or(failed)) {
      failed = true;
      break;
    }
    tc::fence_after_sync();
    const int q = warp & 3, half = warp >> 2;
    const int r = q * 32 + lane, n = n_base + row0 + r;
    const bool live = row0 + r < w_rows && n < n_out;
    float scale = kLatticeScaleF;
    if (rscale && live) scale = __fmul_rn(kLatticeScaleF, __half2float(__ushort_as_half(rscale[n])));
    for (int col0 = half * 128; col0 < half * 128 + 128; col0 += 16) {
      float v[16];
      tc::tmem_ld16(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)col0, v);
      if (live) {
#pragma unroll
        for (int j = 0; j < 16; ++j) {
          const int m = m0 + col0 + j;
          if (m < m_act) Y[(int64_t)m * n_out + n] = v[j] * scale;
        }
      }
    }
    tc::fence_before_sync();
    __syncthreads();
  }
  if (failed && tid == 0 && error_flag) atomicExch(error_flag, 1);
  __syncthreads();
  if (warp == 0) tc::tmem_dealloc(tmem, kMaxAct);
}

// Sets the dynamic shared-memory limits of both GEMM kernels on the current
// device (the launchers also do this lazily on their first launch).
cudaError_t gemm_configure_device() {
  cudaError_t e = cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)GemmLayout(kMaxAct).bytes);
  if (e != cudaSuccess) return e;
  return cudaFuncSetAttribute(gemm_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kStagedSmem);
}

int64_t gemm_staging_ldw(int64_t bpr) { return (24 * bpr + 63) / 64 * 64; }

int64_t gemm_staging_bytes(int64_t n_out, int64_t bpr, int64_t budget) {
  const int64_t row_bytes = gemm_staging_ldw(bpr) * 2;
  int64_t rows = budget / row_bytes / kTileW * kTileW;
  rows = std::max<int64_t>(rows, kTileW);
  return std::min(rows, n_out) * row_bytes;
}

cudaError_t gemm_staged_launch(const Codebook& cb, const int64_t* idx, int64_t n_out, int64_t bpr,
                               const uint16_t* rscale, const void* a, int64_t m, int64_t k, float* y,
                               int* error_flag, void* staging, int64_t staging_bytes, cudaStream_t stream) {
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  static bool configured[kMaxDevices] = {};
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(gemm_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kStagedSmem);
    if (e != cudaSuccess) return e;
    configured[dev] = true;
  }
  const int ldw = (int)gemm_staging_ldw(bpr);
  int64_t chunk = std::min<int64_t>(n_out, staging_bytes / ((int64_t)ldw * 2));
  if (chunk < n_out) chunk = chunk / kTileW * kTileW;
  if (chunk <= 0) return cudaErrorInvalidValue;
  for (int64_t n0 = 0; n0 < n_out; n0 += chunk) {
    const int rows = (int)std::min<int64_t>(chunk, n_out - n0);
    e = decode_rows_bf16_launch(cb, idx + n0 * bpr, rows, (int)bpr, ldw, staging, stream);
    if (e != cudaSuccess) return e;
    const int items = ((rows + kTileW - 1) / kTileW) * (int)((m + kMaxAct - 1) / kMaxAct);
    gemm_staged_kernel<<<std::min(items, sms), kGemmThreads, kStagedSmem, stream>>>(
        static_cast<const __nv_bfloat16*>(staging), ldw, rows, (int)n0, (int)n_out, rscale,
        static_cast<const __nv_bfloat16*>(a), (int)m, (int)k, y, error_flag);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

cudaError_t gemm_launch(const Codebook& cb, const int64_t* idx, int64_t n_out, int64_t bpr, const uint16_t* rscale,
                        const void* a, int64_t m, int64_t k, float* y, int* error_flag, cudaStream_t stream) {
  if (m <= 0 || n_out <= 0) return cudaSuccess;
  int dev = 0, sms = 0;
  cudaError_t e0 = cudaGetDevice(&dev);
  if (e0 != cudaSuccess) return e0;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  static bool configured[kMaxDevices] = {};
  e0 = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e0 != cudaSuccess) return e0;
  if (!configured[dev]) {
    e0 = cudaFuncSetAttribute(gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                              (int)GemmLayout(kMaxAct).bytes);
    if (e0 != cudaSuccess) return e0;
    configured[dev] = true;
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
