// Internal (C++) interfaces between the codebook builder, the kernels and the
// C-ABI layer.  Not part of the public header.
#pragma once

#include <cuda_runtime.h>

#include <cstdint>
#include <string>
#include <vector>

#include "llvq_device.cuh"

namespace llvq {

// Optional gain code written by the quantizer's finalize step (shape-gain
// quantization): thresholds (ascending fp64, nthr of them, 2^bits - 1 for a
// bits-bit code), optional per-row divisor sigma (one per bpr blocks), the
// gain code per block into gain_out (may be null) and, with pack, the index
// replaced by index << bits | gain.  thr == null: no gain code.
struct GainCode {
  const double* thr = nullptr;
  int nthr = 0;
  int bits = 0;
  const float* sigma = nullptr;
  int64_t bpr = 1;
  int* gain_out = nullptr;
  int pack = 0;
};

using SearchLauncher = cudaError_t (*)(const float*, int64_t, const DevBook&, long long*, long long*, float*,
                                       const GainCode&, cudaStream_t);

// A generated search specialisation: its class signature, launcher and the
// window constants of its FFMA chains.
struct SpecEntry {
  const int* sig;
  SearchLauncher launch;
  const char* name;
  float l1max, win_mg, win_am;
  bool angular;  // scores proj / |y| (multi-shell shape of shape-gain) instead of the reference score
};

// Host copy of the table-driven decoder's tables (llvq_tables.cuh; built by
// decode_tables.cu).  ok is false when the codebook's parts are too large to
// tabulate; the kernels then unrank arithmetically (llvq_decode.cuh).
struct TabHost {
  bool ok = false;
  std::vector<uint4> state;            // 2 per state
  std::vector<uint4> crec;             // kTabClassRecords per class
  std::vector<uint4> entry;
  std::vector<uint4> slot;
  std::vector<unsigned long long> tail;  // nibble-string tails
  std::vector<uint32_t> tail2;           // bit-plane tails (parts of two-part classes)
  std::vector<uint32_t> expand2;         // kTabExpand2Words per word in weight order
  std::vector<uint16_t> bucket;        // index bucket -> class (host copy for the host decoder)
  int max_searches = 0;
};

struct Codebook {
  int device = -1;
  int min_shell = 0, max_shell = 0;
  int64_t total = 0;
  std::vector<DevClass> cls;           // host copy, global class order
  std::vector<int64_t> class_start;
  std::vector<uint32_t> golay;         // lexicographic order
  std::vector<uint16_t> golay_wrank;
  std::vector<uint32_t> wlist_word;
  std::vector<uint16_t> wlist_lex;
  std::vector<uint16_t> by_weight;
  std::vector<uint32_t> plist_word;    // one word of each complementary pair (the lighter; bit 0 clear at weight 12)
  std::vector<uint16_t> plist_lex;
  int32_t weight_start[25] = {};
  DevBook dev{};                       // device pointers (valid when device >= 0)
  void* dev_alloc = nullptr;
  size_t dev_bytes = 0;
  const SpecEntry* spec = nullptr;     // generated search code for this class list, or null
  const SpecEntry* spec_ang = nullptr; // generated angular (shape) search code for it, or null
  float rt_l1max = 0, rt_mg = 0, rt_am = 0;  // window constants of the table-driven chains
  TabHost tab;                         // table-driven decoder (host copy)
  std::string tab_why;                 // why the tables are off, when they are
};

// Build the table-driven decoder's tables of a codebook (false: not
// tabulable, with the reason); decode one index on the host with them.
bool build_decode_tables(const Codebook& cb, TabHost& t, std::string* why);
bool decode_index_tables_host(const Codebook& cb, int64_t v, int32_t* out);

const SpecEntry* spec_table(int* count);

cudaError_t quantize_launch(const Codebook& cb, const float* x, int64_t n, long long* index, long long* pair,
                            float* score, cudaStream_t stream, bool force_runtime, const GainCode& gc = GainCode{},
                            bool angular = false);

// Where a kernel reads its indices: int64 (bytes = 8) or packed little-endian
// unsigned integers of 1..7 bytes, the all-ones value standing for an
// invalid index (-1).
struct IndexSource {
  const void* ptr;
  int bytes;
};

// kind: 0 int64 codewords, 1 fp32 (fp32(1/sqrt 8) * k, torch semantics),
// 2 fp32 (fp32 of the double product), 3 bf16 with per-row fp16 scale.
cudaError_t dequantize_launch(const Codebook& cb, IndexSource index, int64_t n, void* out, int kind,
                              const uint16_t* row_scale, int64_t blocks_per_row, int* error_count,
                              cudaStream_t stream);

// int64 <-> packed indices; pack counts (and writes all-ones for) entries
// that are negative or do not fit.
cudaError_t pack_indices_launch(const int64_t* in, int64_t n, int bytes, uint8_t* out, int* error_count,
                                cudaStream_t stream);
cudaError_t unpack_indices_launch(const uint8_t* in, int64_t n, int bytes, int64_t* out, cudaStream_t stream);

// Dequant-GEMM: weights decoded (a chunk of rows at a time) into a bf16
// staging buffer of staging_bytes (rows padded to gemm_staging_ldw(bpr)
// columns), then a pipelined tcgen05 GEMM over it.  gemm_staging_bytes gives
// the buffer size for a byte budget (at least one 128-row tile, at most the
// whole matrix).
constexpr int kMaxDevices = 64;
int64_t gemm_staging_ldw(int64_t bpr);
cudaError_t gemm_staging_pool(cudaMemPool_t* pool);
int64_t gemm_staging_bytes(int64_t n_out, int64_t bpr, int64_t budget);
cudaError_t decode_rows_bf16_launch(const Codebook& cb, IndexSource index, int rows, int bpr, int ldw, void* out,
                                    cudaStream_t stream);
cudaError_t gemm_staged_launch(const Codebook& cb, IndexSource idx, int64_t n_out, int64_t bpr,
                               const uint16_t* rscale, const void* a, int64_t m, int64_t k, float* y,
                               int* error_flag, void* staging, int64_t staging_bytes, cudaStream_t stream);

// Dequant-GEMM for m <= kGemvMaxM activation rows: decode in registers, no
// staging (gemv.cu); gemm_staged_launch takes this path by itself.  On the
// Llama-3 MLP shapes it beats the staged path up to m = 4 (m = 1: 0.36 vs
// 0.47 ms; m = 4: 0.42 vs 0.44; m = 8: 0.51 vs 0.44).
constexpr int kGemvMaxM = 4;
cudaError_t gemv_decode_launch(const Codebook& cb, IndexSource idx, int64_t n_out, int64_t bpr,
                               const uint16_t* rscale, const void* a, int64_t m, int64_t k, float* y,
                               cudaStream_t stream);

// Fused dequant-GEMM (gemm_fused.cu) for 5 <= m <= 256 on codebooks with
// decoder tables: weights decoded into shared memory, stream-K over (tile,
// group) with a per-CTA partial-sum workspace of gemm_fused_workspace_bytes
// and a fixup kernel (no device allocation inside).
bool gemm_fused_ok(const Codebook& cb, int64_t m);
int64_t gemm_fused_workspace_bytes(int64_t n_out, int64_t bpr, int64_t m, int sms);
cudaError_t gemm_fused_launch(const Codebook& cb, IndexSource idx, int64_t n_out, int64_t bpr, const uint16_t* rscale,
                              const void* a, int64_t m, int64_t k, float* y, int* error_flag, void* workspace,
                              int64_t workspace_bytes, int sms, cudaStream_t stream);
cudaError_t device_sms(int* sms);

// Static staging for the no-allocation GEMM entry point: 16 MiB per device,
// enough for one 128-row tile of rows up to 65536 columns.
constexpr int64_t kNoAllocStagingBytes = 16ll << 20;
cudaError_t noalloc_staging(void** ptr);
cudaError_t gemm_configure_device();

// Rotation (fp16 in), fp16 RMS row scale and zero padding to ld columns in
// one pass (hadamard.cu).
cudaError_t rotate_scale_launch(const void* in, int64_t rows, int64_t cols, int64_t ld, int block,
                                const int8_t* signs, float* out, uint16_t* scale_out, cudaStream_t stream);

// Element types 0 fp32, 1 fp16, 2 bf16 (out: 0 or 2).
cudaError_t hadamard_launch(const void* in, int in_type, void* out, int out_type, int64_t rows, int64_t cols,
                            int block, const int8_t* signs, int inverse, cudaStream_t stream);

}  // namespace llvq
