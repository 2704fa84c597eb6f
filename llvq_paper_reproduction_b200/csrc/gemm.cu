// Λ24 dequant-GEMM for sm_100a (tcgen05 tensor cores, TMEM accumulators).
//
//   Y[m, n] = sum_k A[m, k] * W[n, k],   W[n, :] = row_scale[n] * fp32(1/sqrt 8) * codeword(indices[n, :])
//
// Two kernels on one stream.  The decode kernel (dequantize.cu) writes the
// weights as bf16 copies of the integer codeword entries (|k| <= 22 for the
// 48-bit codebook, exact in bf16) into a staging buffer, rows padded with
// zeros to a multiple of 64 columns, a whole matrix or a chunk of rows at a
// time.  The GEMM kernel then streams both operands through kStages shared-
// memory stages of 64 columns (weights 128 rows, activations 256 rows) in the
// 128-byte-swizzled K-major layout the tensor core reads, filled with 16-byte
// cp.async copies (zero outside the matrices).  One thread issues 4 MMAs
// (M = 128 weight rows, N = 256 activation rows, K = 16 each, fp32 in TMEM)
// per stage and commits them to that stage's mbarrier; the MMAs of chunk c
// are queued behind those of chunk c - 1 before the stage chunk c - 1 used is
// refilled, so the tensor pipe does not drain between chunks.  The epilogue
// applies fp32(1/sqrt 8) * row_scale[n], so the only rounding beyond fp32
// accumulation is that of the bf16 activations; it writes Y transposed from
// TMEM (lane = weight row, column = activation row), coalesced along n.
// When the matrix has fewer output tiles than SMs the K range is split in two
// and the halves are added into Y (zeroed first) with fp32 atomics.
//
// The reference has no GEMM (its dequantizer returns int64 codewords,
// impl/llvq_cuda_dequantize.py:78-181); the decode is the same index layout.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <cstdint>
#include <mutex>

#include "llvq_device.cuh"
#include "llvq_internal.h"
#include "tcgen05.cuh"

namespace llvq {

constexpr int kGemmThreads = 256;
constexpr int kTileW = 128;   // weight rows per tile (MMA M)
constexpr int kMaxAct = 256;  // activation rows per tile (MMA N)
constexpr uint32_t kWaitLimit = 1u << 22;

// Byte offset of 16-byte column chunk `chunk` of row `row` in a 128-byte-
// swizzled K-major tile (the SWIZZLE_128B layout the MMA descriptors name).
__device__ __forceinline__ uint32_t swz(int row, int chunk) {
  return (uint32_t)(row * 128 + ((chunk ^ (row & 7)) << 4));
}

// ------------------------------------------------------------ the GEMM

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
                       float* __restrict__ Y, int splits, int* error_flag) {
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


  // work unit = (weight tile, activation tile, K split), splits fastest so
  // the units of one weight tile run side by side and share it in L2
  for (int item = blockIdx.x; item < tn * tm * splits && !failed; item += gridDim.x) {
    const int split = item % splits, tile = item / splits;
    const int row0 = (tile / tm) * kTileW, m0 = (tile % tm) * kMaxAct;
    const int c_begin = kc_total * split / splits, c_end = kc_total * (split + 1) / splits;
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
    for (int c = c_begin; c < c_begin + kStages - 1; ++c) {
      if (c < c_end) issue(c);
      cp_async_commit();
    }
    uint32_t pending = 0;  // stages whose MMA commit has not been waited for
    for (int c = c_begin; c < c_end; ++c) {
      // chunk c has landed (groups committed so far: c - c_begin + kStages - 1)
      cp_async_wait<kStages - 2>();
      tc::fence_proxy_async();
      if (__syncthreads_or(failed)) {
        failed = true;
        break;
      }
      const int st = c % kStages;
      if (tid == 0) {  // queued behind MMA(c - 1): the tensor pipe does not drain between chunks
        tc::fence_after_sync();
        const uint32_t sw = sbase + st * kStageBytes, sa = sw + kStageW;
#pragma unroll
        for (int ks = 0; ks < 4; ++ks) {
          tc::mma_bf16(tmem, tc::desc_sw128(sw + ks * 32), tc::desc_sw128(sa + ks * 32), idesc,
                       (c > c_begin || ks > 0) ? 1u : 0u);
        }
        tc::commit(tc::smem_addr(&mbars[st]));
      }
      pending |= 1u << st;
      // refill the stage MMA(c - 1) read with chunk c + kStages - 1
      const int nxt = c + kStages - 1;
      if (nxt < c_end) {
        const int sn = nxt % kStages;
        if ((pending >> sn) & 1u) {
          const bool ok = tc::mbar_wait(tc::smem_addr(&mbars[sn]), (phase >> sn) & 1u, kWaitLimit);
          phase ^= 1u << sn;
          pending &= ~(1u << sn);
          if (!ok) failed = true;
        }
        if (!failed) issue(nxt);
      }
      cp_async_commit();
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
          if (m < m_act) {
            float* dst = Y + (int64_t)m * n_out + n;
            if (splits > 1) atomicAdd(dst, v[j] * scale);  // two halves into zero: order-free
            else *dst = v[j] * scale;
          }
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

// Sets the GEMM kernel's dynamic shared-memory limit on the current device
// (the launcher also does this lazily on its first launch).
cudaError_t gemm_configure_device() {
  return cudaFuncSetAttribute(gemm_staged_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kStagedSmem);
}

// The library's staging pool on the current device: stream-ordered like the
// default pool, but it keeps what it has reserved (release threshold = max),
// so a GEMM after a synchronize does not map the staging memory again.  It
// holds at most one staging buffer per concurrent call (256 MiB each).
cudaError_t gemm_staging_pool(cudaMemPool_t* pool) {
  static std::mutex mu;
  static cudaMemPool_t pools[kMaxDevices] = {};
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  std::lock_guard<std::mutex> lock(mu);
  if (!pools[dev]) {
    cudaMemPoolProps props = {};
    props.allocType = cudaMemAllocationTypePinned;
    props.location.type = cudaMemLocationTypeDevice;
    props.location.id = dev;
    cudaMemPool_t p = nullptr;
    e = cudaMemPoolCreate(&p, &props);
    if (e != cudaSuccess) return e;
    uint64_t keep = UINT64_MAX;
    e = cudaMemPoolSetAttribute(p, cudaMemPoolAttrReleaseThreshold, &keep);
    if (e != cudaSuccess) {
      cudaMemPoolDestroy(p);
      return e;
    }
    pools[dev] = p;
  }
  *pool = pools[dev];
  return cudaSuccess;
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
  if (m <= 0 || n_out <= 0) return cudaSuccess;
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
  // Split K in two when the whole matrix has fewer tiles than SMs.  Decided
  // from the whole matrix, not the chunk, so every staging size gives each
  // output the same sums; two partial sums added into zero commute exactly.
  const int64_t tiles = ((n_out + kTileW - 1) / kTileW) * ((m + kMaxAct - 1) / kMaxAct);
  const int splits = (tiles < sms && ldw / 64 >= 2) ? 2 : 1;
  if (splits > 1) {
    e = cudaMemsetAsync(y, 0, (size_t)m * (size_t)n_out * sizeof(float), stream);
    if (e != cudaSuccess) return e;
  }
  for (int64_t n0 = 0; n0 < n_out; n0 += chunk) {
    const int rows = (int)std::min<int64_t>(chunk, n_out - n0);
    e = decode_rows_bf16_launch(cb, idx + n0 * bpr, rows, (int)bpr, ldw, staging, stream);
    if (e != cudaSuccess) return e;
    const int items = ((rows + kTileW - 1) / kTileW) * (int)((m + kMaxAct - 1) / kMaxAct) * splits;
    gemm_staged_kernel<<<std::min(items, sms), kGemmThreads, kStagedSmem, stream>>>(
        static_cast<const __nv_bfloat16*>(staging), ldw, rows, (int)n0, (int)n_out, rscale,
        static_cast<const __nv_bfloat16*>(a), (int)m, (int)k, y, splits, error_flag);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace llvq
