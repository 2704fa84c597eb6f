// Λ24 dequant-GEMM for sm_100a (TMA, tcgen05 tensor cores, TMEM accumulators).
//
//   Y[m, n] = sum_k A[m, k] * W[n, k],   W[n, :] = row_scale[n] * fp32(1/sqrt 8) * codeword(indices[n, :])
//
// Two kernels on one stream.  The decode kernel (dequantize.cu) writes the
// weights as bf16 copies of the integer codeword entries (|k| <= 22 for the
// 48-bit codebook, exact in bf16) into a staging buffer, rows padded with
// zeros to a multiple of 64 columns, a whole matrix or a chunk of rows at a
// time.  The GEMM kernel is persistent (one 192-thread CTA per SM) and warp-
// specialised: one thread loads each 64-column stage of both operands
// (weights 128 rows, activations 256 rows) with 2-D TMA tile loads in the
// 128-byte-swizzled K-major layout the tensor core reads (zero fill outside
// the matrices, no multicast); one thread issues 4 tcgen05 MMAs per stage
// (M = 128 weight rows, N = 256 activation rows, K = 16 each, fp32 in TMEM);
// four warps read finished accumulators from TMEM, apply
// fp32(1/sqrt 8) * row_scale[n] and store Y transposed (lane = weight row,
// column = activation row), coalesced along n.  Stages and the two TMEM
// accumulators are handed over with mbarriers (TMA transaction counts,
// tcgen05.commit arrivals, epilogue arrivals); every wait is bounded and sets
// the caller's error flag when it gives up.  The only rounding beyond fp32
// accumulation is that of the bf16 activations.  When the matrix has fewer
// output tiles than SMs the K range is split in two and the halves are added
// into Y (zeroed first) with fp32 atomics.
//
// The reference has no GEMM (its dequantizer returns int64 codewords,
// impl/llvq_cuda_dequantize.py:78-181); the decode is the same index layout.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <mutex>

#include "llvq_device.cuh"
#include "llvq_internal.h"
#include "tcgen05.cuh"

namespace llvq {

constexpr int kTileW = 128;   // weight rows per tile (MMA M)
constexpr int kMaxAct = 256;  // activation rows per tile (MMA N)
constexpr uint32_t kWaitLimit = 1u << 22;

// Shared memory: kStages stages of [weights 128 rows | activations 256 rows]
// x 64 bf16 columns in the 128-byte swizzle (each stage 1024-byte aligned),
// then the mbarriers: full[kStages], empty[kStages], accumulator full[2] and
// empty[2], drain; then the TMEM address.
//
// Roles: warp 0 (one thread) loads both operand tiles of a stage with TMA
// (the box bytes complete the stage's "full" mbarrier); warp 1 (one thread)
// waits for a full stage, issues the 4 MMAs and commits them to the stage's
// "empty" mbarrier (and, after the last chunk of a tile, to the
// accumulator's "full" mbarrier); warps 2-5 read the finished accumulator
// from TMEM, scale and store it, then release it.  Two 256-column
// accumulators let the epilogue of one tile overlap the MMAs of the next.
constexpr int kStages = 4;
constexpr int kStageW = kTileW * 128;           // 16 KB
constexpr int kStageA = kMaxAct * 128;          // 32 KB
constexpr int kStageBytes = kStageW + kStageA;  // 48 KB
constexpr int kTmaThreads = 192;
constexpr int kAccCols = kMaxAct;  // fp32 columns per accumulator
constexpr size_t kTmaBarOff = (size_t)kStages * kStageBytes;
constexpr size_t kTmaSmem = kTmaBarOff + 8 * (2 * kStages + 5) + 16 + 1024;

// Units are (weight tile, activation tile of kMaxAct rows, K split).  When
// the units do not fill the last wave of CTAs, the units of that wave may be
// split into two units of kMaxAct / 2 activation rows each (items from
// full_units on: the activation map `ta_half`, MMA N = 128), so the last wave
// takes half as long; a unit's outputs keep their K order.
__global__ void __launch_bounds__(kTmaThreads, 1)
    gemm_tma_kernel(const __grid_constant__ CUtensorMap tw, const __grid_constant__ CUtensorMap ta,
                    const __grid_constant__ CUtensorMap ta_half, int kc_total, int w_rows, int n_base, int n_out,
                    const uint16_t* __restrict__ rscale, int m_act, float* __restrict__ Y, int splits,
                    int full_units, int* error_flag) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + kTmaBarOff);
  uint32_t* holder = reinterpret_cast<uint32_t*>(bars + 2 * kStages + 5);
  const uint32_t sbase = tc::smem_addr(base);
  auto full = [&](int st) { return tc::smem_addr(&bars[st]); };
  auto empty = [&](int st) { return tc::smem_addr(&bars[kStages + st]); };
  auto acc_full = [&](int a) { return tc::smem_addr(&bars[2 * kStages + a]); };
  auto acc_empty = [&](int a) { return tc::smem_addr(&bars[2 * kStages + 2 + a]); };
  const uint32_t drain = tc::smem_addr(&bars[2 * kStages + 4]);  // the MMA issuer's last commit
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  if (tid == 0) {
    for (int st = 0; st < kStages; ++st) {
      tc::mbar_init(full(st), 1);
      tc::mbar_init(empty(st), 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(acc_full(a), 1);
      tc::mbar_init(acc_empty(a), 4);  // one arrival per epilogue warp
    }
    tc::mbar_init(drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == 0) tc::tmem_alloc(tc::smem_addr(holder), 2 * kAccCols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *holder;
  const int tn = (w_rows + kTileW - 1) / kTileW, tm = (m_act + kMaxAct - 1) / kMaxAct;
  const int units = full_units + 2 * (tn * tm * splits - full_units);
  bool failed = false;
  // item -> (weight tile, activation rows m0 .. m0 + width, K split), splits fastest
  auto unit_of = [&](int item, int& row0, int& m0, int& c_begin, int& c_end, int& width) {
    int half = 0;
    width = kMaxAct;
    if (item >= full_units) {
      half = (item - full_units) & 1;
      item = full_units + ((item - full_units) >> 1);
      width = kMaxAct / 2;
    }
    const int split = item % splits, tile = item / splits;
    row0 = (tile / tm) * kTileW;
    m0 = (tile % tm) * kMaxAct + half * (kMaxAct / 2);
    c_begin = kc_total * split / splits;
    c_end = kc_total * (split + 1) / splits;
  };

  if (warp == 0) {
    if (lane == 0) {  // TMA producer
      uint32_t g = 0;
      for (int item = blockIdx.x; item < units && !failed; item += gridDim.x) {
        int row0, m0, c_begin, c_end, width;
        unit_of(item, row0, m0, c_begin, c_end, width);
        const bool half = width < kMaxAct;
        for (int c = c_begin; c < c_end; ++c, ++g) {
          const int st = (int)(g % kStages);
          const uint32_t use = g / kStages;
          if (use > 0 && !tc::mbar_wait(empty(st), (use - 1) & 1u, kWaitLimit)) {
            failed = true;
            break;
          }
          const uint32_t sw = sbase + st * kStageBytes;
          tc::mbar_arrive_expect_tx(full(st), half ? kStageW + kStageA / 2 : kStageBytes);
          tc::tma_load_2d(sw, &tw, c * 64, row0, full(st));
          tc::tma_load_2d(sw + kStageW, half ? &ta_half : &ta, c * 64, m0, full(st));
        }
      }
      // no copy may still be in flight when the block exits (after a timeout
      // elsewhere): wait for the last use of every stage
      for (uint32_t u = g > (uint32_t)kStages ? g - kStages : 0u; u < g; ++u)
        tc::mbar_wait(full((int)(u % kStages)), (u / kStages) & 1u, kWaitLimit);
    }
  } else if (warp == 1) {
    if (lane == 0) {  // MMA issuer
      const uint32_t idesc_full = tc::idesc_bf16_f32(kTileW, kMaxAct);
      const uint32_t idesc_half = tc::idesc_bf16_f32(kTileW, kMaxAct / 2);
      uint32_t g = 0;
      int it = 0;
      for (int item = blockIdx.x; item < units && !failed; item += gridDim.x, ++it) {
        int row0, m0, c_begin, c_end, width;
        unit_of(item, row0, m0, c_begin, c_end, width);
        const uint32_t idesc = width < kMaxAct ? idesc_half : idesc_full;
        const int a = it & 1;
        const uint32_t use_acc = (uint32_t)it >> 1;
        if (use_acc > 0 && !tc::mbar_wait(acc_empty(a), (use_acc - 1) & 1u, kWaitLimit)) {
          failed = true;
          break;
        }
        tc::fence_after_sync();
        const uint32_t d = tmem + (uint32_t)(a * kAccCols);
        for (int c = c_begin; c < c_end; ++c, ++g) {
          const int st = (int)(g % kStages);
          if (!tc::mbar_wait(full(st), (g / kStages) & 1u, kWaitLimit)) {
            failed = true;
            break;
          }
          tc::fence_after_sync();
          const uint32_t sw = sbase + st * kStageBytes, sa = sw + kStageW;
#pragma unroll
          for (int ks = 0; ks < 4; ++ks)
            tc::mma_bf16(d, tc::desc_sw128(sw + ks * 32), tc::desc_sw128(sa + ks * 32), idesc,
                         (c > c_begin || ks > 0) ? 1u : 0u);
          tc::commit(empty(st));
        }
        if (failed) break;
        tc::commit(acc_full(a));
      }
      // every MMA issued has finished before TMEM is freed
      tc::commit(drain);
      tc::mbar_wait(drain, 0, kWaitLimit);
    }
  } else {  // epilogue: warps 2..5 read TMEM lane quarters 2, 3, 0, 1
    const int q = warp & 3;
    int it = 0;
    for (int item = blockIdx.x; item < units && !failed; item += gridDim.x, ++it) {
      int row0, m0, c_begin, c_end, width;
      unit_of(item, row0, m0, c_begin, c_end, width);
      const int a = it & 1;
      if (!tc::mbar_wait(acc_full(a), ((uint32_t)it >> 1) & 1u, kWaitLimit)) {
        failed = true;
        break;
      }
      tc::fence_after_sync();
      const int r = q * 32 + lane, n = n_base + row0 + r;
      const bool live = row0 + r < w_rows && n < n_out;
      float scale = kLatticeScaleF;
      if (rscale && live) scale = __fmul_rn(kLatticeScaleF, __half2float(__ushort_as_half(rscale[n])));
      const uint32_t t0 = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(a * kAccCols);
      for (int col0 = 0; col0 < width; col0 += 16) {
        float v[16];
        tc::tmem_ld16(t0 + (uint32_t)col0, v);
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
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(acc_empty(a));
    }
  }
  // every role has left its loop (each wait is bounded); reconverge, then free TMEM
  __syncwarp();
  if (failed && error_flag) atomicExch(error_flag, 1);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == 0) tc::tmem_dealloc(tmem, 2 * kAccCols);
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link
// against the driver library).
PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// bf16 row-major [rows, cols] (row stride `stride` elements), box 64 columns
// x box_rows rows, 128-byte swizzle, zero fill outside the matrix.
cudaError_t encode_bf16_map(CUtensorMap* map, const void* ptr, uint64_t cols, uint64_t rows, uint64_t stride,
                            uint32_t box_rows) {
  PFN_cuTensorMapEncodeTiled_v12000 enc = tensor_map_encoder();
  if (!enc) return cudaErrorNotSupported;
  const cuuint64_t dims[2] = {cols, rows};
  const cuuint64_t strides[1] = {stride * 2};
  const cuuint32_t box[2] = {64, box_rows};
  const cuuint32_t elem[2] = {1, 1};
  const CUresult r = enc(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(ptr), dims, strides, box, elem,
                         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? cudaSuccess : cudaErrorInvalidValue;
}

// Sets the GEMM kernel's dynamic shared-memory limit on the current device
// (the launcher also does this lazily on its first launch).
cudaError_t gemm_configure_device() {
  return cudaFuncSetAttribute(gemm_tma_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kTmaSmem);
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

// SM count of the current device, looked up once per device.
cudaError_t device_sms(int* sms) {
  static std::atomic<int> cache[kMaxDevices];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  int v = cache[dev].load(std::memory_order_relaxed);
  if (v <= 0) {
    e = cudaDeviceGetAttribute(&v, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    cache[dev].store(v, std::memory_order_relaxed);
  }
  *sms = v;
  return cudaSuccess;
}

int64_t gemm_staging_ldw(int64_t bpr) { return (24 * bpr + 63) / 64 * 64; }

int64_t gemm_staging_bytes(int64_t n_out, int64_t bpr, int64_t budget) {
  const int64_t row_bytes = gemm_staging_ldw(bpr) * 2;
  int64_t rows = budget / row_bytes / kTileW * kTileW;
  rows = std::max<int64_t>(rows, kTileW);
  return std::min(rows, n_out) * row_bytes;
}

cudaError_t gemm_staged_launch(const Codebook& cb, IndexSource idx, int64_t n_out, int64_t bpr,
                               const uint16_t* rscale, const void* a, int64_t m, int64_t k, float* y,
                               int* error_flag, void* staging, int64_t staging_bytes, cudaStream_t stream) {
  if (m <= 0 || n_out <= 0) return cudaSuccess;
  if (m <= kGemvMaxM) return gemv_decode_launch(cb, idx, n_out, bpr, rscale, a, m, k, y, stream);
  int dev = 0, sms = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  static std::atomic<bool> configured[kMaxDevices];  // kernel attributes set (idempotent if raced)
  e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  if (e != cudaSuccess) return e;
  if (!configured[dev].load(std::memory_order_acquire)) {
    e = gemm_configure_device();
    if (e != cudaSuccess) return e;
    configured[dev].store(true, std::memory_order_release);
  }
  const int ldw = (int)gemm_staging_ldw(bpr);
  CUtensorMap ta, ta_half;
  e = encode_bf16_map(&ta, a, (uint64_t)k, (uint64_t)m, (uint64_t)k, kMaxAct);
  if (e != cudaSuccess) return e;
  e = encode_bf16_map(&ta_half, a, (uint64_t)k, (uint64_t)m, (uint64_t)k, kMaxAct / 2);
  if (e != cudaSuccess) return e;
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
    const IndexSource part{static_cast<const uint8_t*>(idx.ptr) + n0 * bpr * idx.bytes, idx.bytes};
    e = decode_rows_bf16_launch(cb, part, rows, (int)bpr, ldw, staging, stream);
    if (e != cudaSuccess) return e;
    const int items = ((rows + kTileW - 1) / kTileW) * (int)((m + kMaxAct - 1) / kMaxAct) * splits;
    // halve the units of a partial last wave when the halves fit in one wave
    int full_units = items;
    if (splits == 1 && items > sms) {
      const int tail = items % sms;
      if (tail > 0 && 2 * tail <= sms) full_units = items - tail;
    }
    const int launch_items = full_units + 2 * (items - full_units);
    CUtensorMap tw;
    e = encode_bf16_map(&tw, staging, (uint64_t)ldw, (uint64_t)rows, (uint64_t)ldw, kTileW);
    if (e != cudaSuccess) return e;
    gemm_tma_kernel<<<std::min(launch_items, sms), kTmaThreads, kTmaSmem, stream>>>(
        tw, ta, ta_half, ldw / 64, rows, (int)n0, (int)n_out, rscale, (int)m, y, splits, full_units, error_flag);
    e = cudaGetLastError();
    if (e != cudaSuccess) return e;
  }
  return cudaSuccess;
}

}  // namespace llvq
