// Fused Λ24 dequant-GEMM for sm_100a: weights decoded straight into the
// tensor cores' shared-memory operand, no bf16 staging in HBM.
//
//   Y[m, n] = sum_k A[m, k] * W[n, k],   W[n, :] = row_scale[n] * fp32(1/sqrt 8) * codeword(indices[n, :])
//
// For 5 <= m <= 256 (one activation tile) and a codebook with decoder tables.
// Work is the flattened list of (weight tile of 128 rows, group of 8 index
// blocks = 192 columns); each persistent CTA takes one contiguous range of it
// (stream-K: every CTA gets the same number of groups, a tile can be shared by
// consecutive CTAs).  Per CTA (one per SM, 30 warps):
//   warps 0-23  decode the group's 128 x 8 blocks (one or two per thread)
//               with the table-driven decoder (its small tables copied to
//               shared memory) and store them as bf16 into one of two
//               group slots: three 64-column K-major sub-tiles in the 128-byte
//               swizzle the MMA descriptors read; then fence the writes to the
//               async proxy and arrive on the slot's "full" barrier;
//   warp 24     (one thread) loads the activation columns of each 64-column
//               chunk with 2-D TMA (no multicast; rows >= m and columns >= k
//               read as zero) into a ring of chunk slots;
//   warp 25     (one thread) issues 4 tcgen05 MMAs per chunk (M = 128 weight
//               rows, N = m rounded up to 16, K = 16) into one of two TMEM
//               accumulators and commits them to the chunk's and the group's
//               "empty" barriers, and to the accumulator's "full" barrier at
//               the end of a tile segment;
//   warps 26-29 read a finished accumulator (one TMEM lane quarter each) and
//               write Y, scaled by fp32(1/sqrt 8) * row_scale (a whole tile),
//               or the unscaled partial sums into the CTA's workspace slot (a
//               tile shared with a neighbouring CTA).
// A fixup kernel then adds each shared tile's partial sums in CTA order and
// scales them, so every output has one summation order (the same bits on
// every call, whatever the number of SMs).  Every barrier wait is bounded and
// sets the caller's error flag when it gives up.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda.h>
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cstdint>

#include "llvq_decode.cuh"
#include "llvq_device.cuh"
#include "llvq_internal.h"
#include "tcgen05.cuh"

namespace llvq {

cudaError_t encode_bf16_map(CUtensorMap* map, const void* ptr, uint64_t cols, uint64_t rows, uint64_t stride,
                            uint32_t box_rows);

namespace {

constexpr int kFRows = 128;                  // weight rows per tile (MMA M)
constexpr int kFGroupBlocks = 8;             // index blocks per group: 192 columns = 3 chunks of 64
constexpr int kFChunks = 3;
constexpr int kFSubTile = kFRows * 128;      // one 64-column chunk of the weight tile: 16 KB
constexpr int kFGroupBytes = kFChunks * kFSubTile;
constexpr int kFDecodeWarps = 24;
constexpr int kFDecodeThreads = kFDecodeWarps * 32;
constexpr int kFWarps = kFDecodeWarps + 6;
constexpr int kFThreads = kFWarps * 32;      // 960: at most 64 registers
constexpr int kFTmaWarp = kFDecodeWarps, kFMmaWarp = kFDecodeWarps + 1, kFEpiWarp0 = kFDecodeWarps + 2;
constexpr uint32_t kFWaitLimit = 1u << 22;
constexpr size_t kFSmemBudget = 227 * 1024;

struct FusedLayout {
  int n_mma;        // MMA N: m rounded up to 16 (<= 256)
  int a_bytes;      // one activation chunk: n_mma rows x 128 B
  int a_slots;      // activation chunk ring
  TabSmem T;        // the decoder's shared tables, at off_tab (DecodeSharedBase first)
  size_t off_a, off_tab, off_bar, smem;
};

// Weight slots, then the activation ring, the decoder's tables (with the
// Golay word lists when three activation slots still fit, else without:
// those are read through the cache) and the barriers.
FusedLayout fused_layout(const Codebook& cb, int m) {
  FusedLayout L{};
  L.n_mma = (m + 15) / 16 * 16;
  L.a_bytes = L.n_mma * 128;
  const int ncls = (int)cb.cls.size(), nst = cb.dev.tab.n_states;
  for (int with_words = 1; with_words >= 0; --with_words) {
    const TabSmem T = tab_smem_layout(ncls, nst, ~size_t(0) >> 1, 0, with_words != 0);
    const size_t fixed = 2 * (size_t)kFGroupBytes + (T.bytes + 15) / 16 * 16 + 1024 + 256;
    const int slots = fixed >= kFSmemBudget ? 0 : (int)std::min<size_t>(6, (kFSmemBudget - fixed) / (size_t)L.a_bytes);
    if (slots >= (with_words ? 3 : 2)) {
      L.a_slots = slots;
      L.T = T;
      break;
    }
  }
  L.off_a = 2 * (size_t)kFGroupBytes;
  L.off_tab = L.off_a + (size_t)L.a_slots * L.a_bytes;
  L.off_bar = (L.off_tab + L.T.bytes + 15) / 16 * 16;
  L.smem = L.off_bar + 8 * (size_t)(4 + 2 * L.a_slots + 5) + 16 + 1024;  // + alignment slack
  return L;
}

__host__ __device__ __forceinline__ int64_t range_begin(int64_t L, int C, int c) { return L * c / C; }
__host__ __device__ __forceinline__ int cta_of(int64_t L, int C, int64_t g) {
  return (int)(((g + 1) * C + L - 1) / L) - 1;
}

}  // namespace

__global__ void __launch_bounds__(kFThreads, 1)
    gemm_fused_kernel(const __grid_constant__ CUtensorMap ta, IndexSource index, int n_out, int bpr,
                      DevBook book, TabSmem T, const uint16_t* __restrict__ rscale, int m_act, int n_mma, int a_bytes,
                      int a_slots, uint32_t off_a, uint32_t off_sh, uint32_t off_bar, int64_t total_groups,
                      int groups_per_tile, float* __restrict__ Y, float* __restrict__ ws, int* error_flag) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* base = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                             ~static_cast<uintptr_t>(1023));
  DecodeSharedBase& sh = *reinterpret_cast<DecodeSharedBase*>(base + off_sh);
  uint64_t* bars = reinterpret_cast<uint64_t*>(base + off_bar);
  uint32_t* holder = reinterpret_cast<uint32_t*>(bars + 4 + 2 * a_slots + 5);
  const uint32_t sbase = tc::smem_addr(base);
  auto wfull = [&](int s) { return tc::smem_addr(&bars[s]); };
  auto wempty = [&](int s) { return tc::smem_addr(&bars[2 + s]); };
  auto afull = [&](int s) { return tc::smem_addr(&bars[4 + s]); };
  auto aempty = [&](int s) { return tc::smem_addr(&bars[4 + a_slots + s]); };
  auto accfull = [&](int a) { return tc::smem_addr(&bars[4 + 2 * a_slots + a]); };
  auto accempty = [&](int a) { return tc::smem_addr(&bars[4 + 2 * a_slots + 2 + a]); };
  const uint32_t drain = tc::smem_addr(&bars[4 + 2 * a_slots + 4]);
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const int C = gridDim.x, cta = blockIdx.x;
  const int64_t gb = range_begin(total_groups, C, cta), ge = range_begin(total_groups, C, cta + 1);
  const int G = groups_per_tile;
  const int first_tile = (int)(gb / G);
  uint32_t tmem_cols = 32;
  while (tmem_cols < (uint32_t)(2 * n_mma)) tmem_cols <<= 1;

  decode_setup_base(book, sh);
  tab_smem_fill(book, base + off_sh, T);
  if (tid == 0) {
    for (int s = 0; s < 2; ++s) {
      tc::mbar_init(wfull(s), kFDecodeWarps);
      tc::mbar_init(wempty(s), 1);
    }
    for (int s = 0; s < a_slots; ++s) {
      tc::mbar_init(afull(s), 1);
      tc::mbar_init(aempty(s), 1);
    }
    for (int a = 0; a < 2; ++a) {
      tc::mbar_init(accfull(a), 1);
      tc::mbar_init(accempty(a), 4);
    }
    tc::mbar_init(drain, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (warp == kFTmaWarp) tc::tmem_alloc(tc::smem_addr(holder), tmem_cols);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  const uint32_t tmem = *holder;
  bool failed = false;

  if (warp < kFDecodeWarps) {
    // ---- decoders: the CTA's blocks in one sequence (1024 per group), thread
    // t taking t, t + 768, ...: every warp meets every group at least once
    // (its blocks are 768 apart) and arrives on a group's barrier when it
    // moves past it, so the decode work is spread evenly over the warps
    const TabCtx tcx = tab_ctx<true>(book, sh, base + off_sh, T);
    constexpr int kItems = kFRows * kFGroupBlocks;
    const int64_t nitems = (ge - gb) * kItems;
    int64_t cur_g = -1;
    uint8_t* wslot = base;
    auto finish_group = [&](int64_t g) {
      tc::fence_proxy_async();  // the MMA reads these bytes through the async proxy
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(wfull((int)((g - gb) & 1)));
    };
#pragma unroll 1
    for (int64_t it = tid; it < nitems; it += kFDecodeThreads) {
      const int64_t g = gb + it / kItems;
      if (g != cur_g) {
        if (cur_g >= 0) finish_group(cur_g);
        cur_g = g;
        const int i = (int)(g - gb);
        const uint32_t use = (uint32_t)i >> 1;
        if (use > 0 && !tc::mbar_wait(wempty(i & 1), (use - 1) & 1u, kFWaitLimit)) {
          failed = true;
          break;
        }
        wslot = base + (i & 1) * kFGroupBytes;
      }
      const int tile = (int)(g / G), gl = (int)(g % G);
      const int blk = (int)(it % kItems);
      const int r = blk >> 3, j = blk & 7;
      const int n = tile * kFRows + r, b = gl * kFGroupBlocks + j;
      uint32_t mag[6], neg;
      tab_decode_any<true>(tcx, n < n_out && b < bpr ? load_index(index, (int64_t)n * bpr + b) : -1, mag, neg);
      uint32_t w[12];
      bf16_codeword(mag, neg, w);
#pragma unroll
      for (int e = 0; e < 3; ++e) {
        const int c8 = 3 * j + e, st = c8 >> 3, q = c8 & 7;
        *reinterpret_cast<uint4*>(wslot + st * kFSubTile + r * 128 + ((q ^ (r & 7)) << 4)) =
            make_uint4(w[4 * e], w[4 * e + 1], w[4 * e + 2], w[4 * e + 3]);
      }
    }
    if (cur_g >= 0 && !failed) finish_group(cur_g);
  } else if (warp == kFTmaWarp) {
    if (lane == 0) {  // ---- activation chunks
      uint32_t q = 0;
      for (int64_t g = gb; g < ge && !failed; ++g) {
        const int gl = (int)(g % G);
        for (int j = 0; j < kFChunks; ++j, ++q) {
          const int s = (int)(q % (uint32_t)a_slots);
          const uint32_t use = q / (uint32_t)a_slots;
          if (use > 0 && !tc::mbar_wait(aempty(s), (use - 1) & 1u, kFWaitLimit)) {
            failed = true;
            break;
          }
          tc::mbar_arrive_expect_tx(afull(s), (uint32_t)a_bytes);
          tc::tma_load_2d(sbase + off_a + (uint32_t)s * a_bytes, &ta, gl * (kFGroupBlocks * kDim) + j * 64, 0,
                          afull(s));
        }
      }
      // no copy may still be in flight when the block exits
      for (uint32_t u = q > (uint32_t)a_slots ? q - a_slots : 0u; u < q; ++u)
        tc::mbar_wait(afull((int)(u % (uint32_t)a_slots)), (u / (uint32_t)a_slots) & 1u, kFWaitLimit);
    }
  } else if (warp == kFMmaWarp) {
    if (lane == 0) {  // ---- tensor-core issue
      const uint32_t idesc = tc::idesc_bf16_f32(kFRows, n_mma);
      uint32_t q = 0;
      int seg = 0;
      for (int64_t g = gb; g < ge && !failed;) {
        const int tile = (int)(g / G);
        const int64_t seg_end = std::min<int64_t>(ge, (int64_t)(tile + 1) * G);
        const int a = seg & 1;
        const uint32_t use_acc = (uint32_t)seg >> 1;
        if (use_acc > 0 && !tc::mbar_wait(accempty(a), (use_acc - 1) & 1u, kFWaitLimit)) {
          failed = true;
          break;
        }
        tc::fence_after_sync();
        const uint32_t d = tmem + (uint32_t)(a * n_mma);
        bool first = true;
        for (; g < seg_end && !failed; ++g) {
          const int i = (int)(g - gb), slot = i & 1;
          if (!tc::mbar_wait(wfull(slot), ((uint32_t)i >> 1) & 1u, kFWaitLimit)) {
            failed = true;
            break;
          }
          for (int j = 0; j < kFChunks; ++j, ++q) {
            const int s = (int)(q % (uint32_t)a_slots);
            if (!tc::mbar_wait(afull(s), (q / (uint32_t)a_slots) & 1u, kFWaitLimit)) {
              failed = true;
              break;
            }
            tc::fence_after_sync();
            const uint32_t sw = sbase + slot * kFGroupBytes + j * kFSubTile;
            const uint32_t sa = sbase + off_a + (uint32_t)s * a_bytes;
#pragma unroll
            for (int ks = 0; ks < 4; ++ks) {
              tc::mma_bf16(d, tc::desc_sw128(sw + ks * 32), tc::desc_sw128(sa + ks * 32), idesc, first ? 0u : 1u);
              first = false;
            }
            tc::commit(aempty(s));
          }
          if (failed) break;
          tc::commit(wempty(slot));
        }
        if (failed) break;
        tc::commit(accfull(a));
        ++seg;
      }
      tc::commit(drain);  // every MMA issued has finished before TMEM is freed
      tc::mbar_wait(drain, 0, kFWaitLimit);
    }
  } else if (warp >= kFEpiWarp0) {
    // ---- epilogue: warps 18..21 read TMEM lane quarters 2, 3, 0, 1
    const int qtr = warp & 3;
    int seg = 0;
    for (int64_t g = gb; g < ge && !failed; ++seg) {
      const int tile = (int)(g / G);
      const int64_t seg_begin = g, seg_end = std::min<int64_t>(ge, (int64_t)(tile + 1) * G);
      g = seg_end;
      const bool whole = seg_begin == (int64_t)tile * G && seg_end == (int64_t)(tile + 1) * G;
      const int slot = tile == first_tile ? 0 : 1;
      const int a = seg & 1;
      if (!tc::mbar_wait(accfull(a), ((uint32_t)seg >> 1) & 1u, kFWaitLimit)) {
        failed = true;
        break;
      }
      tc::fence_after_sync();
      const int r = qtr * 32 + lane, n = tile * kFRows + r;
      const bool live = n < n_out;
      float scale = kLatticeScaleF;
      if (rscale && live) scale = __fmul_rn(kLatticeScaleF, __half2float(__ushort_as_half(rscale[n])));
      float* wsp = ws + ((size_t)(2 * cta + slot) * n_mma) * kFRows + r;
      const uint32_t t0 = tmem + ((uint32_t)(qtr * 32) << 16) + (uint32_t)(a * n_mma);
      for (int col0 = 0; col0 < n_mma; col0 += 16) {
        float v[16];
        tc::tmem_ld16(t0 + (uint32_t)col0, v);
#pragma unroll
        for (int jj = 0; jj < 16; ++jj) {
          const int m = col0 + jj;
          if (m < m_act) {
            if (whole) {
              if (live) Y[(int64_t)m * n_out + n] = v[jj] * scale;
            } else {
              wsp[(size_t)m * kFRows] = v[jj];
            }
          }
        }
      }
      tc::fence_before_sync();
      __syncwarp();
      if (lane == 0) tc::mbar_arrive(accempty(a));
    }
  }
  __syncwarp();
  if (failed && error_flag) atomicExch(error_flag, 1);
  tc::fence_before_sync();
  __syncthreads();
  tc::fence_after_sync();
  if (warp == kFTmaWarp) tc::tmem_dealloc(tmem, tmem_cols);
}

// Shared tiles: the partial sums of the CTAs that covered the tile, added in
// CTA order, then scaled.  One CTA per tile; tiles a single CTA finished were
// written by the GEMM kernel.
__global__ void __launch_bounds__(256) gemm_fused_fixup(int n_out, const uint16_t* __restrict__ rscale, int m_act,
                                                        int n_mma, int64_t total_groups, int groups_per_tile,
                                                        int ctas, const float* __restrict__ ws,
                                                        float* __restrict__ Y) {
  const int tile = blockIdx.x, G = groups_per_tile;
  const int c0 = cta_of(total_groups, ctas, (int64_t)tile * G);
  const int c1 = cta_of(total_groups, ctas, (int64_t)(tile + 1) * G - 1);
  if (c0 == c1) return;
  const int slot0 = range_begin(total_groups, ctas, c0) < (int64_t)tile * G ? 1 : 0;
  for (int e = threadIdx.x; e < m_act * kFRows; e += blockDim.x) {
    const int m = e / kFRows, r = e % kFRows, n = tile * kFRows + r;
    if (n >= n_out) continue;
    float s = 0.f;
    for (int c = c0; c <= c1; ++c) {
      const int slot = c == c0 ? slot0 : 0;
      s += ws[((size_t)(2 * c + slot) * n_mma + m) * kFRows + r];
    }
    float scale = kLatticeScaleF;
    if (rscale) scale = __fmul_rn(kLatticeScaleF, __half2float(__ushort_as_half(rscale[n])));
    Y[(int64_t)m * n_out + n] = s * scale;
  }
}

bool gemm_fused_ok(const Codebook& cb, int64_t m) {
  return cb.dev.tab.state && m > kGemvMaxM && m <= 256 && fused_layout(cb, (int)m).a_slots >= 2;
}

int64_t gemm_fused_workspace_bytes(int64_t n_out, int64_t bpr, int64_t m, int sms) {
  const int64_t total = ((n_out + kFRows - 1) / kFRows) * ((bpr + kFGroupBlocks - 1) / kFGroupBlocks);
  const int64_t ctas = std::min<int64_t>(sms, total);
  return ctas * 2 * ((m + 15) / 16 * 16) * kFRows * (int64_t)sizeof(float);
}

cudaError_t gemm_fused_launch(const Codebook& cb, IndexSource idx, int64_t n_out, int64_t bpr, const uint16_t* rscale,
                              const void* a, int64_t m, int64_t k, float* y, int* error_flag, void* workspace,
                              int64_t workspace_bytes, int sms, cudaStream_t stream) {
  if (m <= 0 || n_out <= 0) return cudaSuccess;
  if (!gemm_fused_ok(cb, m)) return cudaErrorInvalidValue;
  const FusedLayout L = fused_layout(cb, (int)m);
  if (L.a_slots < 2) return cudaErrorInvalidValue;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  static std::atomic<bool> configured[kMaxDevices];
  if (!configured[dev].load(std::memory_order_acquire)) {
    e = cudaFuncSetAttribute(gemm_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)kFSmemBudget);
    if (e != cudaSuccess) return e;
    configured[dev].store(true, std::memory_order_release);
  }
  const int64_t tiles = (n_out + kFRows - 1) / kFRows, G = (bpr + kFGroupBlocks - 1) / kFGroupBlocks;
  const int64_t total = tiles * G;
  const int ctas = (int)std::min<int64_t>(sms, total);
  if (gemm_fused_workspace_bytes(n_out, bpr, m, sms) > workspace_bytes) return cudaErrorInvalidValue;
  CUtensorMap ta;
  e = encode_bf16_map(&ta, a, (uint64_t)k, (uint64_t)m, (uint64_t)k, (uint32_t)L.n_mma);
  if (e != cudaSuccess) return e;
  gemm_fused_kernel<<<ctas, kFThreads, L.smem, stream>>>(
      ta, idx, (int)n_out, (int)bpr, cb.dev, L.T, rscale, (int)m, L.n_mma, L.a_bytes, L.a_slots, (uint32_t)L.off_a,
      (uint32_t)L.off_tab, (uint32_t)L.off_bar, total, (int)G, y, static_cast<float*>(workspace), error_flag);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;
  gemm_fused_fixup<<<(unsigned)tiles, 256, 0, stream>>>((int)n_out, rscale, (int)m, L.n_mma, total, (int)G, ctas,
                                                        static_cast<const float*>(workspace), y);
  return cudaGetLastError();
}

}  // namespace llvq
