/*
 * llvq_b200.h -- C ABI of the B200 (sm_100a) Leech-lattice (Λ24) quantizer.
 *
 * Plain pointers and sizes only.  Device pointers must be on the codebook's
 * device; `stream` is a cudaStream_t (NULL = legacy default stream).  Every
 * GPU entry point is asynchronous on `stream`, never synchronises, and returns
 * a status code (llvq_status); llvq_last_error() gives the message of the last
 * failure on the calling thread.
 *
 * The drop-in boundary replaces the reference's two NVRTC launchers of
 * dmnunez1993/llvq-paper-reproduction:
 *   impl/llvq_cuda_quantize.py:544-602    quantize_lattice_cuda
 *   impl/llvq_cuda_dequantize.py:221-261  dequantize_lattice_cuda
 * and the device tables its caller builds
 *   impl/leech_lattice_vector_quantizer_gpu.py:345-411  _quantize_cuda_metadata
 *   impl/leech_lattice_vector_quantizer_gpu.py:424-518  _codeword_cuda_metadata
 */
#ifndef LLVQ_B200_H
#define LLVQ_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef struct llvq_codebook llvq_codebook;

typedef enum {
  LLVQ_OK = 0,
  LLVQ_ERR_INVALID_ARGUMENT = 1, /* the reference raises ValueError (bad device, dtype, shape) */
  LLVQ_ERR_CUDA = 2,             /* the reference raises RuntimeError(str(CUresult)) */
  LLVQ_ERR_UNSUPPORTED = 3,      /* codebook the library cannot index in 64 bits */
  LLVQ_ERR_OUT_OF_MEMORY = 4,
  LLVQ_ERR_INDEX_RANGE = 5,      /* the reference raises IndexError */
  LLVQ_ERR_NOT_A_CODEWORD = 6    /* the reference's encode_codeword raises ValueError */
} llvq_status;

/* Output kinds of the dequantizer. */
enum {
  LLVQ_OUT_INT64 = 0,          /* integer codeword (dequantize_lattice) */
  LLVQ_OUT_F32 = 1,            /* fp32(1/sqrt 8) * k in fp32: the GPU API's dequantize (_gpu.py:298) */
  LLVQ_OUT_F32_DOUBLE = 2,     /* the CPU API's double 1/sqrt(8) * k, rounded to fp32 (CPU module :243-245) */
  LLVQ_OUT_BF16_ROWSCALE = 3   /* bf16(fp32 value * fp16 per-row scale) */
};

/* Quantizer option flags. */
enum { LLVQ_FLAG_TABLE_DRIVEN = 1 /* score with the table-driven chains even if generated code exists */ };

/* Codebook from a class list in index order (shell ascending, then the
 * reference's class order): per class its shell, parity (0 even, 1 odd) and
 * the 24 absolute values of its leader in descending order.  Builds the Golay
 * tables, offsets and counts on the host and uploads them to `device`
 * (device < 0: host-only codebook, usable by the *_host functions).
 * Replaces the table construction of LeechLatticeVectorQuantizerGpu.__init__
 * and its two *_cuda_metadata caches (_gpu.py:154-212, :345-518).
 * Indices are unsigned 64-bit: a codebook may hold up to 2^64 - 2 codewords
 * (shells 2..32 hold 1.09e19, past the reference's int64 torch.long), and
 * every int64 index argument or output carries the two's-complement image of
 * its unsigned value (negative from 2^63 on); -1 (all ones) is never a
 * codeword and stays the invalid index. */
int llvq_codebook_create(int32_t n_classes, const int32_t* shell, const int32_t* parity, const int32_t* leader,
                         int device, llvq_codebook** out);
void llvq_codebook_destroy(llvq_codebook* cb);
/* total_count (= reference total_count, as the int64 image of an unsigned
 * value), class count, shell range, and whether
 * generated scoring code matches this class list (1) or the table-driven path runs (0). */
int llvq_codebook_info(const llvq_codebook* cb, int64_t* total_count, int32_t* n_classes, int32_t* min_shell,
                       int32_t* max_shell, int32_t* specialized);

/* Nearest codeword of each 24-D fp32 row: indices[i] is the reference index
 * (bit-exact with LeechLatticeVectorQuantizer.quantize, ties in its loop
 * order), best_pair[i] = class_id * 4096 + golay_index and best_score[i] the
 * fp32 rounding of the reference's fp64 score.  Rows with NaN/Inf get index,
 * pair -1 and score NaN.  Two kernel launches (search, then finalize);
 * best_pair / best_score carry the hand-over between them.  Replaces
 * quantize_lattice_cuda (impl/llvq_cuda_quantize.py:544-602). */
int llvq_quantize(const llvq_codebook* cb, const float* x, int64_t n, int64_t* indices, int64_t* best_pair,
                  float* best_score, void* stream);
int llvq_quantize_ex(const llvq_codebook* cb, const float* x, int64_t n, int64_t* indices, int64_t* best_pair,
                     float* best_score, uint32_t flags, void* stream);

/* Shape-gain quantization in one pass (no reference counterpart: the
 * reference lists shape-gain in its README only).  The shape is llvq_quantize's
 * codeword (for a single-shell codebook: the shell point of largest
 * correlation with x); the gain g = <x, y> / |y| (the same compensated fp64
 * projection as the score, |y| = sqrt(16 shell)), divided by row_sigma[i /
 * blocks_per_row] when row_sigma (fp32, device) is not NULL, is coded as the
 * number of the 2^gain_bits - 1 ascending fp64 gain_thresholds (device) below
 * it.  gain_index[i] (int32, may be NULL) receives the code; with
 * LLVQ_GAIN_PACK in flags, indices[i] = shape << gain_bits | code (shape bits
 * + gain_bits <= 63), else the shape index.  With LLVQ_GAIN_ANGULAR the shape
 * is the multi-shell one: the codeword of largest <x, y> / |y| over all the
 * codebook's shells (fp64, ties in the reference's loop order), which needs
 * generated angular search code for the class list (else
 * LLVQ_ERR_UNSUPPORTED); without it, the reference's nearest codeword.  Rows
 * with NaN/Inf: index -1, code -1.  Same launches, scratch and stream rules as
 * llvq_quantize. */
enum { LLVQ_GAIN_PACK = 1, LLVQ_GAIN_ANGULAR = 2 };
int llvq_quantize_gain(const llvq_codebook* cb, const float* x, int64_t n, int64_t* indices, int64_t* best_pair,
                       float* best_score, const double* gain_thresholds, int32_t gain_bits, const float* row_sigma,
                       int64_t blocks_per_row, int32_t* gain_index, uint32_t flags, void* stream);

/* Integer codewords [n,24] of indices [n].  Out-of-range indices give zero
 * rows and are counted into *error_count (device int, may be NULL).
 * Replaces dequantize_lattice_cuda (impl/llvq_cuda_dequantize.py:221-261). */
int llvq_dequantize_lattice(const llvq_codebook* cb, const int64_t* indices, int64_t n, int64_t* out,
                            int32_t* error_count, void* stream);
/* Scaled fp32 vectors [n,24] (kind LLVQ_OUT_F32 or LLVQ_OUT_F32_DOUBLE).
 * Replaces LeechLatticeVectorQuantizerGpu.dequantize on tensors (_gpu.py:290-298). */
int llvq_dequantize(const llvq_codebook* cb, const int64_t* indices, int64_t n, float* out, int32_t kind,
                    int32_t* error_count, void* stream);
/* bf16 weights [n,24] = bf16(dequantize * row_scale[i / blocks_per_row]),
 * row_scale fp16 bit patterns.  No reference counterpart (the reference has
 * neither bf16 output nor per-row scales). */
int llvq_dequantize_bf16(const llvq_codebook* cb, const int64_t* indices, int64_t n, const uint16_t* row_scale_f16,
                         int64_t blocks_per_row, uint16_t* out_bf16, int32_t* error_count, void* stream);

/* Dequant-GEMM: y[m, n] = sum_k a[m, k] * W[n, k], where row n of W is the
 * dequantized indices[n * blocks_per_row + b] (b = 0 .. blocks_per_row-1,
 * 24 columns each) times row_scale[n] (fp16 bits; NULL means 1).  a: bf16
 * [m, k] row-major, 16-byte aligned, k % 8 == 0, k <= 24 * blocks_per_row
 * (W columns at k and beyond meet zeros); y: fp32 [m, n_out].  For m <= 4
 * one kernel decodes each weight block in registers and multiplies it there
 * (a warp per output row, a fixed summation order; nothing is allocated).
 * For 5 <= m <= 256 on a codebook with decoder tables (llvq_codebook_tables)
 * one fused kernel decodes the weights straight into the shared-memory
 * operand of tcgen05 MMAs (stream-K over tiles and K groups; the partial sums
 * of tiles shared by two SMs go to a workspace of at most 39 MB from the
 * library's pool and a second kernel adds them in a fixed order).
 * Otherwise the weights
 * are decoded into a bf16 staging buffer (at most 256 MiB, chunk by chunk
 * beyond that; stream-ordered on `stream` from a library-owned memory pool
 * that keeps its reservation between calls) that a pipelined
 * tcgen05 GEMM reads, accumulating in fp32; when the matrix has fewer
 * 128 x 256 output tiles than SMs the K range is split in two and y is
 * zeroed first (cudaMemsetAsync).  Every path gives each output one
 * summation order (the same bits on every call).  *error_flag (device int,
 * may be NULL) is set to 1 if a tensor-core wait timed out.  No reference
 * counterpart (the reference has no GEMM). */
int llvq_gemm(const llvq_codebook* cb, const int64_t* indices, int64_t n_out, int64_t blocks_per_row,
              const uint16_t* row_scale_f16, const uint16_t* a_bf16, int64_t m, int64_t k, float* y,
              int32_t* error_flag, void* stream);

/* llvq_gemm without device allocation.  No counterpart in the reference.
 * For callers that may not allocate device memory while they run (a serving
 * engine that reserved the GPU's memory for its own pool, a step that must not
 * fail on out-of-memory halfway): a fixed LLVQ_GEMM_NOALLOC_STAGING_BYTES
 * (16 MiB) array compiled into the library, one per device, replaces the
 * stream-ordered pool buffer: as the fused kernel's partial-sum workspace
 * when that fits it, else as the bf16 staging, a chunk of rows at a time
 * (batches of m <= 4 are decoded in registers, as in llvq_gemm, and do
 * not use the array).  Same arguments, results and error flag as llvq_gemm, plus,
 * for m > 4, the limit blocks_per_row <= LLVQ_GEMM_NOALLOC_MAX_BLOCKS_PER_ROW
 * (2730: one 128-row tile of rows up to 65536 columns fits the array); wider
 * rows return LLVQ_ERR_INVALID_ARGUMENT.  The array needs no initial contents.
 * The array is device memory that the CUDA runtime allocates when it loads
 * the library module holding it, which (with lazy module loading, the CUDA 12
 * default) is the first call of this function on each device.  So make one
 * call per device -- an empty one (m = 0 or n_out = 0) is enough -- before
 * reserving the GPU's memory and before any stream capture; that call also
 * sets the kernels' shared-memory limits.  Calls that overlap on one device
 * (unordered streams, concurrent host threads) share the array and race:
 * order them. */
#define LLVQ_GEMM_NOALLOC_STAGING_BYTES (16 << 20)
#define LLVQ_GEMM_NOALLOC_MAX_BLOCKS_PER_ROW 2730
int llvq_gemm_noalloc(const llvq_codebook* cb, const int64_t* indices, int64_t n_out, int64_t blocks_per_row,
                      const uint16_t* row_scale_f16, const uint16_t* a_bf16, int64_t m, int64_t k, float* y,
                      int32_t* error_flag, void* stream);

/* Packed index storage (no reference counterpart: the reference keeps int64
 * indices, _gpu.py:333).  An index takes index_bytes little-endian bytes
 * (6 for the 48-bit codebook of shells 2..13 instead of 8); the all-ones
 * value stands for the invalid index -1.
 * llvq_pack_indices: int64 [n] -> packed [n * index_bytes]; entries that are
 *   negative (other than -1) or do not fit below all-ones are counted into
 *   *error_count (device int, may be NULL) and stored as all-ones.
 * llvq_unpack_indices: packed -> int64 (all-ones -> -1).
 * llvq_dequantize_packed: any LLVQ_OUT_* kind from packed indices (row_scale
 *   and blocks_per_row for LLVQ_OUT_BF16_ROWSCALE only).
 * llvq_gemm_packed: llvq_gemm reading packed indices.
 * The codebook-bound calls need index_bytes with total_count <= all-ones. */
int llvq_pack_indices(const int64_t* indices, int64_t n, int32_t index_bytes, uint8_t* packed, int32_t* error_count,
                      void* stream);
int llvq_unpack_indices(const uint8_t* packed, int64_t n, int32_t index_bytes, int64_t* indices, void* stream);
int llvq_dequantize_packed(const llvq_codebook* cb, const uint8_t* packed, int32_t index_bytes, int64_t n, void* out,
                           int32_t kind, const uint16_t* row_scale_f16, int64_t blocks_per_row,
                           int32_t* error_count, void* stream);
int llvq_gemm_packed(const llvq_codebook* cb, const uint8_t* packed, int32_t index_bytes, int64_t n_out,
                     int64_t blocks_per_row, const uint16_t* row_scale_f16, const uint16_t* a_bf16, int64_t m,
                     int64_t k, float* y, int32_t* error_flag, void* stream);

/* Seeded random Hadamard rotation of each row of a [rows, cols] matrix, in
 * segments of `block` columns (a power of two, <= 4096, dividing cols):
 * forward out = H (signs * in) / sqrt(block), inverse out = signs * (H in) /
 * sqrt(block); signs: int8 +-1 per column (device).  in: fp16 (in_is_half)
 * or fp32; out: fp32 (may alias an fp32 input).  Device: the current one.
 * No reference counterpart (the reference README lists the rotation only). */
int llvq_hadamard(const void* in, int32_t in_is_half, float* out, int64_t rows, int64_t cols, int32_t block,
                  const int8_t* signs, int32_t inverse, void* stream);
/* The same rotation with element types LLVQ_DT_F32 / LLVQ_DT_F16 /
 * LLVQ_DT_BF16 in and LLVQ_DT_F32 / LLVQ_DT_BF16 out (butterflies in fp32,
 * one rounding at the store; out must not alias in for bf16).  The bf16 ->
 * bf16 form rotates a GEMM's activations for weights quantized after the
 * same rotation: x W^T = (x R)(W R)^T.  No reference counterpart. */
enum { LLVQ_DT_F32 = 0, LLVQ_DT_F16 = 1, LLVQ_DT_BF16 = 2 };
int llvq_hadamard_ex(const void* in, int32_t in_type, void* out, int32_t out_type, int64_t rows, int64_t cols,
                     int32_t block, const int8_t* signs, int32_t inverse, void* stream);

/* Weight preparation for quantization in one pass: each fp16 row of a
 * [rows, cols] matrix is rotated forward as llvq_hadamard does (signs,
 * segments of `block` columns), its RMS over the cols entries (a fixed-order
 * fp32 reduction) is rounded to fp16 (at least 1e-8) into row_scale_out[row],
 * and out[row] (fp32, ld >= cols columns) receives the rotated row divided by
 * that scale, zero from column cols on.  cols * 4 bytes must fit 200 KiB of
 * shared memory.  No reference counterpart. */
int llvq_rotate_scale(const uint16_t* in_f16, int64_t rows, int64_t cols, int64_t ld, int32_t block,
                      const int8_t* signs, float* out, uint16_t* row_scale_out, void* stream);

/* Host-side scalar paths (no GPU needed).
 * llvq_codeword_host:  LeechLatticeVectorQuantizerGpu.codeword (_gpu.py:262-265)
 * llvq_encode_host:    LeechLatticeVectorQuantizer.encode_codeword (CPU module :247-280) */
int llvq_codeword_host(const llvq_codebook* cb, int64_t index, int32_t* out24);
int llvq_encode_host(const llvq_codebook* cb, const int32_t* codeword24, int64_t* index);

/* Integer codewords [n,24] of indices [n] on the host, decoded with the same
 * tables and code as the GPU kernels' table-driven decoder (the entry point
 * its CPU tests use).  Needs a codebook with tables (llvq_codebook_tables);
 * out-of-range indices give zero rows and are counted in *bad (may be NULL).
 * Host counterpart of dequantize_lattice_cuda (impl/llvq_cuda_dequantize.py:
 * 221-261); the reference's CPU codeword() is impl/leech_lattice_vector_quantizer.py:235-245. */
int llvq_codeword_batch_host(const llvq_codebook* cb, const int64_t* indices, int64_t n, int32_t* out, int64_t* bad);
/* Whether the codebook's decoder is table-driven (1) or unranks arithmetically
 * (0: parts too large to tabulate), the tables' size in bytes and the most
 * table lookups one index takes.  No reference counterpart. */
int llvq_codebook_tables(const llvq_codebook* cb, int32_t* tabulated, int64_t* table_bytes, int32_t* max_lookups);

const char* llvq_status_string(int status);
const char* llvq_last_error(void);
int llvq_version(void);

#ifdef __cplusplus
}
#endif

#endif /* LLVQ_B200_H */
