// Per-index Λ24 decoder shared by the dequantizer and the dequant-GEMM's
// weight staging.
//
// Index layout and unranking as in the reference's codeword() path
// (impl/leech_lattice_vector_quantizer.py:196-245, :774-867): class by binary
// search over the class starts, a 96-byte decode record (six 16-byte loads),
// the per-class splits by multiply-high with an exact correction,
// then one 24-step lexicographic unranking loop shared by both parities (an
// even class unranks its |v| = 2 mod 4 part on the word's positions, then its
// |v| = 0 mod 4 part on the others), so warps holding both parities do not
// diverge there.  Lexicographic unranking picks, at each step, the value
// whose branch [N*C_{j-1}/rem, N*C_j/rem) holds the rank (C = cumulative
// counts, N the multinomial of what remains, rem the positions left).
// For parts of at most four distinct values (fast_step) the three boundaries
// are computed exactly -- a product, a shift by the power of two in rem and a
// multiply by the inverse of its odd part -- and compared with the rank; the
// magnitude goes straight to its position in a per-thread shared-memory row.
// The last eight steps, which always end a part, are one lookup in a table of
// all eight-step sequences over four values (DevBook::tail_seq).
// Parts of up to eight values, or whose N stays at or above 2^32 past their
// first step, use the same step with seven boundaries (wide_step, 64-bit while
// N >= 2^32), taken by a whole warp at once.
// Other classes use a general step (fp32 estimate of rank*rem/N, byte-wise
// compare of the packed cumulative counts, exact verification; a 64-bit scan
// while N >= 2^32) and a nibble sequence scattered afterwards.  Even-class
// signs use the closed form of rank_even_signs (llvq_device.cuh).
#pragma once

#include <cuda_bf16.h>

#include <cstdint>

#include "llvq_device.cuh"
#include "llvq_internal.h"
#include "llvq_tables.cuh"

namespace llvq {

// Index i of a source: one 8-byte load, or the packed bytes (6-byte indices,
// the 48-bit codebook's, as three 2-byte loads); all-ones packed -> -1.
__device__ __forceinline__ int64_t load_index(IndexSource src, int64_t i) {
  if (src.bytes == 8) return __ldg(static_cast<const int64_t*>(src.ptr) + i);
  uint64_t v = 0;
  if (src.bytes == 6) {
    const uint16_t* h = static_cast<const uint16_t*>(src.ptr) + i * 3;
    v = (uint64_t)__ldg(h) | ((uint64_t)__ldg(h + 1) << 16) | ((uint64_t)__ldg(h + 2) << 32);
  } else {
    const uint8_t* b = static_cast<const uint8_t*>(src.ptr) + i * src.bytes;
    for (int k = 0; k < src.bytes; ++k) v |= (uint64_t)__ldg(b + k) << (8 * k);
  }
  return v == (~0ull >> (64 - 8 * src.bytes)) ? -1 : (int64_t)v;
}

constexpr int kMaxSmemClasses = 1024;
constexpr int kDecodeThreads = 256;  // blocks up to this size get per-thread rows
constexpr int kRowWords = 7;         // 24 magnitude bytes per thread; a 28-byte stride reads without bank conflicts

// What both decoders keep in shared memory: the class starts (binary
// search) and the sign-deposit table.
struct DecodeSharedBase {
  int64_t starts[kMaxSmemClasses];
  uint8_t deposit4[256];  // [m * 16 + s]: the low popc(m) bits of s placed on the set bits of m, in order
};

// The arithmetic decoder's shared memory: the base plus division constants
// and per-thread magnitude rows.
struct DecodeShared : DecodeSharedBase {
  uint64_t inv[kDim + 1];   // inverse of the odd part of d modulo 2^64
  uint32_t shift[kDim + 1]; // trailing zeros of d
  uint2 div32[kDim + 1];    // {inverse of the odd part of d modulo 2^32, trailing zeros of d}
  uint32_t rows[kDecodeThreads * kRowWords];  // each thread's codeword magnitudes, by position
};

// Fill the base tables (call with the whole block, then __syncthreads()).
__device__ __forceinline__ void decode_setup_base(const DevBook& book, DecodeSharedBase& sh) {
  if (book.n_classes <= kMaxSmemClasses)
    for (int k = threadIdx.x; k < book.n_classes; k += blockDim.x) sh.starts[k] = book.class_start[k];
  for (int i = threadIdx.x; i < 256; i += blockDim.x) {
    const uint32_t m = i >> 4;
    uint32_t src = i & 15, dep = 0;
    for (int b = 0; b < 4; ++b)
      if ((m >> b) & 1u) {
        dep |= (src & 1u) << b;
        src >>= 1;
      }
    sh.deposit4[i] = (uint8_t)dep;
  }
}

// Fill the shared tables (call with the whole block, then __syncthreads()).
__device__ __forceinline__ void decode_setup(const DevBook& book, DecodeShared& sh) {
  decode_setup_base(book, sh);
  if (threadIdx.x <= kDim && threadIdx.x > 0) {
    const uint32_t d = threadIdx.x, s = __ffs(d) - 1;
    sh.shift[d] = s;
    sh.inv[d] = inv_odd64(d >> s);
    sh.div32[d] = make_uint2((uint32_t)sh.inv[d], s);
  }
}

__device__ __forceinline__ uint32_t byte_at(uint64_t packed, int j) { return (uint32_t)(packed >> (8 * j)) & 0xFFu; }

// a / b for any a and b >= 1, given magic = floor((2^64 - 1) / b): the high
// half of a * magic is floor(a / b) or one less (division by an invariant
// integer by multiplication, Granlund and Montgomery 1994), fixed up by one
// comparison of the remainder.  Integer pipes only.
__device__ __forceinline__ uint64_t div_magic(uint64_t a, uint64_t b, uint64_t magic, uint64_t& rem) {
  uint64_t q = __umul64hi(a, magic);
  uint64_t r = a - q * b;
  if (r >= b) {
    ++q;
    r -= b;
  }
  rem = r;
  return q;
}

// One unranking step: the value index whose branch holds `rank`; updates
// rank, N (multinomial of what remains) and the packed counts.
__device__ __forceinline__ uint32_t unrank_step(uint64_t& rank, uint64_t& N, uint64_t& cnt, int rem,
                                                const DecodeShared& sh) {
  const uint32_t s = sh.shift[rem];
  uint32_t j = 0;
  if (N >> 32) {  // 64-bit branch-by-branch scan (first steps of the largest classes only)
    const uint64_t inv = sh.inv[rem];
    for (; j < kMaxVals; ++j) {
      const uint64_t c = byte_at(cnt, j);
      if (!c) continue;
      const uint64_t br = ((N * c) >> s) * inv;
      if (rank < br) { N = br; break; }
      rank -= br;
    }
    cnt -= 1ull << (8 * j);
    return j;
  }
  const uint32_t inv = (uint32_t)sh.inv[rem];
  const uint32_t r = (uint32_t)rank, n32 = (uint32_t)N;
  const uint64_t cum = cnt * 0x0101010101010101ull;  // byte i = c_0 + ... + c_i (sums <= 24)
  const float q = __fmul_rn(__uint2float_rn(r), __fmul_rn((float)rem, __frcp_rn(__uint2float_rn(n32))));
  uint32_t t = min((uint32_t)q, (uint32_t)rem - 1u);
  const uint32_t tb = t * 0x01010101u;
  j = (__popc(__vcmpleu4((uint32_t)cum, tb)) + __popc(__vcmpleu4((uint32_t)(cum >> 32), tb))) >> 3;
  const uint64_t x = (uint64_t)r * (uint32_t)rem;
  uint64_t lo = (uint64_t)n32 * ((uint32_t)((cum << 8) >> (8 * j)) & 0xFFu);
  uint32_t c = byte_at(cnt, j);
  uint64_t hi = lo + (uint64_t)n32 * c;
  // fp32 estimate landed in a neighbouring bucket: step to it (at most 8
  // buckets exist; j stays in [0, 7])
  for (int guard = 0; (x < lo || x >= hi) && guard < 2 * kMaxVals; ++guard) {
    if (x < lo) {
      if (j == 0) break;
      --j;
    } else {
      if (j == kMaxVals - 1) break;
      ++j;
    }
    c = byte_at(cnt, j);
    lo = (uint64_t)n32 * ((uint32_t)((cum << 8) >> (8 * j)) & 0xFFu);
    hi = lo + (uint64_t)n32 * c;
  }
  rank = (uint32_t)((x - lo) >> s) * inv;
  N = (uint32_t)(((uint64_t)n32 * c) >> s) * inv;
  cnt -= 1ull << (8 * j);
  return j;
}

// One unranking step for a part of at most four distinct values: the
// branch boundaries B_i = N * C_i / rem (C_i = c_0 + ... + c_i, exact
// integers because N * c_j / rem is the multinomial of what remains after
// value j) are computed exactly, the value taken is the number of boundaries
// at or below `rank`, and the new rank and N are rank - B_{j-1} and
// B_j - B_{j-1}.  C_i of absent values equals rem, so their boundary is N
// and is never taken.  32-bit arithmetic once N < 2^32 (every step but the
// first few of the largest classes).
struct FastPart {
  uint32_t rank, N;         // N < 2^32 after the first step of a part
  uint32_t c0, c1, c2;      // cumulative counts of the first 1, 2, 3 values
  uint32_t v0, v1, v2, v3;  // the values, descending
};

// Exact N * c / d for d = rem, given d's {odd-part inverse mod 2^32, shift},
// when the quotient is an integer below 2^32.
__device__ __forceinline__ uint32_t exact_div32(uint32_t n, uint32_t c, uint2 d) {
  const uint64_t q = (uint64_t)n * c;
  return __funnelshift_r((uint32_t)q, (uint32_t)(q >> 32), d.y) * d.x;
}

__device__ __forceinline__ uint32_t fast_step(FastPart& p, uint2 d) {
  const uint32_t b0 = exact_div32(p.N, p.c0, d), b1 = exact_div32(p.N, p.c1, d), b2 = exact_div32(p.N, p.c2, d);
  const bool p0 = b0 <= p.rank, p1 = b1 <= p.rank, p2 = b2 <= p.rank;
  const uint32_t lo = p2 ? b2 : p1 ? b1 : p0 ? b0 : 0u;
  const uint32_t hi = !p0 ? b0 : !p1 ? b1 : !p2 ? b2 : p.N;
  p.rank -= lo;
  p.N = hi - lo;
  // the value taken loses one count: every cumulative count from it on
  p.c0 -= !p0;
  p.c1 -= !p1;
  p.c2 -= !p2;
  return p2 ? p.v3 : p1 ? p.v2 : p0 ? p.v1 : p.v0;
}

// The first step of a part whose N may reach 2^32 (64-bit boundaries, the
// 64-bit inverse of rem's odd part); leaves N below 2^32.
__device__ __forceinline__ uint32_t fast_first_step(FastPart& p, uint64_t rank, uint64_t N, int rem,
                                                    const DecodeShared& sh) {
  if (!(N >> 32)) {
    p.rank = (uint32_t)rank;
    p.N = (uint32_t)N;
    return fast_step(p, sh.div32[rem]);
  }
  const uint32_t s = sh.shift[rem];
  const uint64_t inv = sh.inv[rem];
  const uint64_t b0 = ((N * p.c0) >> s) * inv, b1 = ((N * p.c1) >> s) * inv, b2 = ((N * p.c2) >> s) * inv;
  const bool p0 = b0 <= rank, p1 = b1 <= rank, p2 = b2 <= rank;
  const uint64_t lo = p2 ? b2 : p1 ? b1 : p0 ? b0 : 0ull;
  const uint64_t hi = !p0 ? b0 : !p1 ? b1 : !p2 ? b2 : N;
  p.rank = (uint32_t)(rank - lo);
  p.N = (uint32_t)(hi - lo);
  p.c0 -= !p0;
  p.c1 -= !p1;
  p.c2 -= !p2;
  return p2 ? p.v3 : p1 ? p.v2 : p0 ? p.v1 : p.v0;
}

__device__ __forceinline__ void fast_part_load(FastPart& p, uint64_t pv, uint64_t pm) {
  p.v0 = byte_at(pv, 0);
  p.v1 = byte_at(pv, 1);
  p.v2 = byte_at(pv, 2);
  p.v3 = byte_at(pv, 3);
  p.c0 = byte_at(pm, 0);
  p.c1 = p.c0 + byte_at(pm, 1);
  p.c2 = p.c1 + byte_at(pm, 2);
}

// The fast step for parts of up to eight values (kMaxVals) and any N below
// 2^59: the value taken is the number of the seven boundaries B_i = N * C_i /
// rem at or below `rank` (they do not decrease; C_i of absent values equals
// rem, so their boundary is N and is never at or below it), then rank and N
// become rank - B_{j-1} and B_j - B_{j-1}, recomputed from the packed
// cumulative counts.  Exact divisions as in fast_step: in 32 bits once N <
// 2^32, before that with the 64-bit inverse of rem's odd part (N * C < 2^64).
struct WidePart {
  uint64_t rank, N;
  uint64_t cum;  // byte i = C_i = c_0 + ... + c_i (byte 7: all that remain)
  uint64_t pv;   // byte j = value j, descending
};

__device__ __forceinline__ void wide_part_load(WidePart& p, uint64_t pv, uint64_t pm, uint64_t rank, uint64_t N) {
  p.pv = pv;
  p.rank = rank;
  p.N = N;
  p.cum = pm * 0x0101010101010101ull;  // prefix sums of the count bytes (at most 24: no carries)
}

// The value index taken; rank, N and the counts updated.  WIDE: N may be at
// or above 2^32 (64-bit boundaries).  nb: boundaries to test, at least the
// part's distinct values - 1 (the boundaries past it are N).
template <bool WIDE>
__device__ __forceinline__ uint32_t wide_step(WidePart& p, int rem, int nb, const DecodeShared& sh) {
  uint32_t j = 0;
  uint64_t lo, hi;
  if constexpr (WIDE) {
    const uint32_t s = sh.shift[rem];
    const uint64_t inv = sh.inv[rem];
#pragma unroll
    for (int i = 0; i < kMaxVals - 1; ++i)
      if (i < nb) j += ((p.N * byte_at(p.cum, i)) >> s) * inv <= p.rank;
    lo = ((p.N * byte_at(p.cum << 8, j)) >> s) * inv;
    hi = ((p.N * byte_at(p.cum, j)) >> s) * inv;
  } else {
    const uint2 d = sh.div32[rem];
    const uint32_t n = (uint32_t)p.N, r = (uint32_t)p.rank;
#pragma unroll
    for (int i = 0; i < kMaxVals - 1; ++i)
      if (i < nb) j += exact_div32(n, byte_at(p.cum, i), d) <= r;
    lo = exact_div32(n, byte_at(p.cum << 8, j), d);
    hi = exact_div32(n, byte_at(p.cum, j), d);
  }
  p.rank -= lo;
  p.N = hi - lo;
  p.cum -= 0x0101010101010101ull << (8 * j);  // the value taken loses one count
  return j;
}

// Magnitudes by position with wide_step, into the thread's shared-memory row.
// Out of line: a warp runs it only when one of its indices needs it.  Each
// step takes the 64-bit form while any index of the warp has N >= 2^32, and
// tests as many boundaries as the warp's largest part needs (nvals: this
// index's largest count of distinct values in a part).
static __device__ __noinline__ void decode_wide(uint32_t word, bool odd, int nfirst, uint64_t rank, uint64_t N, uint64_t cnt,
                                         uint64_t rank2, uint64_t N2, uint64_t cnt2, uint64_t pv0, uint64_t pv1,
                                         int nvals, const DecodeShared& sh, uint8_t* row) {
  const unsigned lanes = __activemask();  // every lane here runs the 24 steps
  const int nb = (int)__reduce_max_sync(lanes, (unsigned)nvals) - 1;
  WidePart p;
  wide_part_load(p, odd ? pv0 : pv1, cnt, rank, N);
  uint32_t mask = odd ? kFull24 : word;  // positions still to fill, lowest first
#pragma unroll 1
  for (int t = 0; t < kDim; ++t) {
    if (t == nfirst) {  // even: the word's positions are done, the f0 part fills the rest
      wide_part_load(p, pv0, cnt2, rank2, N2);
      mask = ~word & kFull24;
    }
    const int rem = t < nfirst ? nfirst - t : kDim - t;
    const uint32_t j =
        __any_sync(lanes, (p.N >> 32) != 0) ? wide_step<true>(p, rem, nb, sh) : wide_step<false>(p, rem, nb, sh);
    row[__ffs(mask) - 1] = (uint8_t)byte_at(p.pv, (int)j);
    mask &= mask - 1u;
  }
}

// Magnitudes by position for the classes the fast path does not take (a part
// with more than four values, or N >= 2^32 after a part's first step): the
// general step, a nibble sequence of value indices, then the scatter.  Kept
// out of line: rarely run, and the decoder's hot code must stay small.
static __device__ __noinline__ void decode_general(uint32_t word, bool odd, int nfirst, uint64_t rank, uint64_t N, uint64_t cnt,
                                            uint64_t rank2, uint64_t N2, uint64_t cnt2, uint64_t pv0, uint64_t pv1,
                                            const DecodeShared& sh, uint32_t* mag) {
  uint64_t seq_lo = 0, seq_hi = 0;  // 4-bit value indices, step order
#pragma unroll 4
  for (int t = 0; t < kDim; ++t) {
    if (t == nfirst) {
      rank = rank2;
      N = N2;
      cnt = cnt2;
    }
    const int rem = t < nfirst ? nfirst - t : kDim - t;
    const uint32_t j = unrank_step(rank, N, cnt, rem, sh);
    if (t < 16) seq_lo |= (uint64_t)j << (4 * t);
    else seq_hi |= (uint64_t)j << (4 * (t - 16));
  }
  // scatter: odd -> step d at position d; even -> the word's positions take
  // the first (f1) part in order, the others the second (f0) part
  uint32_t m[6] = {0, 0, 0, 0, 0, 0};
#pragma unroll
  for (int d = 0; d < kDim; ++d) {
    const bool bit = (word >> d) & 1u;
    const bool part1 = !odd && bit;
    const int below1 = __popc(word & ((1u << d) - 1u));
    const int t = odd ? d : (bit ? below1 : nfirst + d - below1);
    const uint32_t nib = (uint32_t)((t < 16 ? seq_lo >> (4 * t) : seq_hi >> (4 * (t - 16))) & 15u);
    m[d >> 2] |= byte_at(part1 ? pv1 : pv0, (int)nib) << (8 * (d & 3));
  }
#pragma unroll
  for (int w = 0; w < 6; ++w) mag[w] = m[w];
}

// Class of a valid index: the bucket table narrows the search to the classes
// between the owners of the bucket's lowest index and of the next bucket's
// (1.5 to 2.3 binary-search steps on average at shells 2..13 instead of 9).
__device__ __forceinline__ int find_class_bucketed(const DevBook& book, const int64_t* starts, int64_t v) {
  const uint64_t u = (uint64_t)v;
  int key = 0;
  if (u) {
    const int e = 63 - __clzll((long long)u);
    key = 1 + e * 16 + (int)((e >= 4 ? u >> (e - 4) : u << (4 - e)) & 15u);
  }
  int lo = __ldg(book.bucket + key), hi = __ldg(book.bucket + key + 1) + 1;
  while (lo + 1 < hi) {
    const int mid = (lo + hi) >> 1;
    if ((uint64_t)starts[mid] <= (uint64_t)v) lo = mid; else hi = mid;
  }
  return lo;
}

// Integer codeword of index v (before the 1/sqrt(8) scale); false and zeros
// when v is outside the codebook.  Classes whose parts have at most four
// distinct values (all but a few classes) unrank with fast_step, the others
// with a part multinomial below 2^59 with wide_step; both write each magnitude
// to its position in the thread's shared-memory row.  The rest (none up to
// shell 32) use the general step and a nibble sequence.
__device__ __forceinline__ bool decode_index(int64_t v, const DevBook& book, DecodeShared& sh, int (&y)[kDim]) {
  bool ok = (uint64_t)v < (uint64_t)book.total;  // indices are unsigned (codebooks past 2^63)
  if (ok) {
    const int k = find_class_bucketed(book, book.n_classes <= kMaxSmemClasses ? sh.starts : book.class_start, v);
    const uint4* rp = reinterpret_cast<const uint4*>(book.dcls + k);
    const uint4 w0 = __ldg(rp), w1 = __ldg(rp + 1), w2 = __ldg(rp + 2), w3 = __ldg(rp + 3), w4 = __ldg(rp + 4),
                w5 = __ldg(rp + 5);
    auto u64 = [](uint32_t lo, uint32_t hi) { return ((uint64_t)hi << 32) | lo; };
    const uint64_t start = u64(w0.x, w0.y), perm = u64(w0.z, w0.w);
    const uint64_t magic_perm = u64(w1.x, w1.y);
    const uint64_t f0p = u64(w1.z, w1.w);
    const uint32_t f1p = w2.x, meta = w2.y, gbase = w2.z;
    const uint64_t magic_f1 = u64(w3.x, w3.y);
    const uint64_t pv0 = u64(w3.z, w3.w), pm0 = u64(w4.x, w4.y), pv1 = u64(w4.z, w4.w), pm1 = u64(w5.x, w5.y);
    const bool odd = meta & 1;
    const int weight = (meta >> 1) & 31, sshift = (meta >> 6) & 31;
    uint64_t prank;
    const uint64_t cur = div_magic((uint64_t)v - start, perm, magic_perm, prank);
    uint32_t word;
    uint64_t sign = 0;
    // first part: odd -> all 24 coordinates; even -> the word's f1 part, then f0
    uint64_t rank, N, cnt, rank2 = 0, N2 = 1, cnt2 = 0;
    int nfirst;
    if (odd) {
      word = __ldg(book.golay + (int)cur);
      rank = prank;
      N = perm;
      cnt = pm0;
      nfirst = kDim;
    } else {
      sign = cur & ((1ull << sshift) - 1);
      const uint64_t g = cur >> sshift;
      word = __ldg(book.golay + __ldg(book.by_weight + gbase + (int)g));
      uint64_t r1;
      const uint64_t r0 = div_magic(prank, f1p, magic_f1, r1);
      rank = r1;
      N = f1p;
      cnt = pm1;
      rank2 = r0;
      N2 = f0p;
      cnt2 = pm0;
      nfirst = weight;
    }
    uint32_t mag[6];  // magnitudes by position, 4 per word
    if ((meta & kMetaWide) && threadIdx.x < kDecodeThreads) {
      uint8_t* row = reinterpret_cast<uint8_t*>(sh.rows + threadIdx.x * kRowWords);
      // The whole warp takes the eight-value variant when one of its indices
      // needs it (any index may: it decodes every fast class), so a warp runs
      // one of the two step loops, never both.
      if (__any_sync(__activemask(), !(meta & kMetaFast))) {
        decode_wide(word, odd, nfirst, rank, N, cnt, rank2, N2, cnt2, pv0, pv1,
                    (int)max((meta >> 11) & 15u, (meta >> 15) & 15u), sh, row);
      } else {
        // A part can only start at step 0 or at a word weight (8, 12, 16), and
        // N can only reach 2^32 at step 0.
        FastPart part;
        uint32_t mask, val;  // mask: positions still to fill, lowest first
        int base;            // rem = base - t
        uint32_t pvals = (uint32_t)(nfirst == 0 || odd ? pv0 : pv1);  // the part's values, bytes 0..3
        if (nfirst == 0) {  // weight 0: only the f0 part
          fast_part_load(part, pv0, cnt2);
          mask = kFull24;
          base = kDim;
          val = fast_first_step(part, rank2, N2, kDim, sh);
        } else {
          fast_part_load(part, odd ? pv0 : pv1, cnt);
          mask = odd ? kFull24 : word;
          base = nfirst;
          val = fast_first_step(part, rank, N, nfirst, sh);
        }
        row[__ffs(mask) - 1] = (uint8_t)val;
        mask &= mask - 1u;
        const uint2* div = sh.div32 + base;  // div[-t] = rem's constants at step t
#pragma unroll
        for (int t = 1; t < 4; ++t) {
          val = fast_step(part, div[-t]);
          row[__ffs(mask) - 1] = (uint8_t)val;
          mask &= mask - 1u;
        }
        // steps 4..15 in blocks of four, not unrolled (a part can only switch
        // at a block start: 8, 12 or 16), so the code stays small enough for
        // the instruction cache
#pragma unroll 1
        for (int tb = 4; tb < kDim - kTailLen; tb += 4) {
          if (tb == nfirst) {  // even: the word's positions are done, the f0 part fills the rest
            fast_part_load(part, pv0, cnt2);
            part.rank = (uint32_t)rank2;
            part.N = (uint32_t)N2;
            mask = ~word & kFull24;
            div = sh.div32 + kDim;
            pvals = (uint32_t)pv0;
          }
          const uint2* d = div - tb;
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            val = fast_step(part, d[-i]);
            row[__ffs(mask) - 1] = (uint8_t)val;
            mask &= mask - 1u;
          }
        }
        if (nfirst == kDim - kTailLen) {  // weight 16: the f0 part is exactly the last eight steps
          fast_part_load(part, pv0, cnt2);
          part.rank = (uint32_t)rank2;
          mask = ~word & kFull24;
          pvals = (uint32_t)pv0;
        }
        // Steps 16..23 end the last part of every class (odd, weight 0 or 24:
        // the only part; weight 8, 12 or 16: the f0 part): one lookup in the
        // tail table by the remaining counts and rank (bounded by the table
        // sizes, which valid counts and ranks never reach).
        const uint32_t key = min(part.c0 * 81u + part.c1 * 9u + part.c2, (uint32_t)kTailKeys - 1u);
        const uint32_t seq = __ldg(book.tail_seq + min(__ldg(book.tail_off + key) + part.rank, (uint32_t)kTailSeqs - 1u));
#pragma unroll
        for (int i = 0; i < kTailLen; ++i) {
          row[__ffs(mask) - 1] = (uint8_t)__byte_perm(pvals, 0u, (seq >> (2 * i)) & 3u);
          mask &= mask - 1u;
        }
      }
      const uint32_t* rw = sh.rows + threadIdx.x * kRowWords;
#pragma unroll
      for (int w = 0; w < 6; ++w) mag[w] = rw[w];
    } else {
      decode_general(word, odd, nfirst, rank, N, cnt, rank2, N2, cnt2, pv0, pv1, sh, mag);
    }
    // Per-position bits of the magnitudes, four bytes at a time (every
    // magnitude is below 128, so byte + 0x7F carries into bit 7 exactly when
    // it is nonzero; a multiply by 0x01020408 gathers bit 0 of the four bytes
    // into the top nibble).
    uint32_t nzmask = 0, b1mask = 0;
#pragma unroll
    for (int w = 0; w < 6; ++w) {
      const uint32_t t = mag[w];
      nzmask |= (((((t + 0x7F7F7F7Fu) >> 7) & 0x01010101u) * 0x01020408u) >> 24) << (4 * w);
      b1mask |= ((((t >> 1) & 0x01010101u) * 0x01020408u) >> 24) << (4 * w);
    }
    uint32_t neg;  // coordinates to negate
    if (odd) {
      // y = m where m = 1 mod 4 off the word or m = 3 mod 4 on it, else -m
      neg = b1mask ^ word;
    } else {
      // signs: insert, at the first word coordinate, the bit that gives the
      // class's parity of negative word coordinates (weight 0: rank = mask),
      // then deposit the bits on the nonzero coordinates in position order
      const int nz = __popc(nzmask);
      uint32_t cmask;
      if (word) {
        const int p = __popc(nzmask & ((word & (0u - word)) - 1u));
        const uint32_t rr = (uint32_t)sign;
        ok = (sign >> (nz - 1)) == 0;
        cmask = ((rr >> p) << (p + 1)) | (rr & ((1u << p) - 1u));
      } else {
        ok = nz >= 32 || (sign >> nz) == 0;
        cmask = (uint32_t)sign;
      }
      neg = 0;
#pragma unroll
      for (int k = 0; k < kDim / 4; ++k) {  // four positions at a time
        const uint32_t m = (nzmask >> (4 * k)) & 15u;
        neg |= (uint32_t)sh.deposit4[m * 16 + (cmask & 15u)] << (4 * k);
        cmask >>= __popc(m);
      }
      if (word && (__popc(neg & word) & 1) != (int)((meta >> 19) & 1)) neg ^= word & (0u - word);
    }
#pragma unroll
    for (int d = 0; d < kDim; ++d) {
      const int m = (int)((mag[d >> 2] >> (8 * (d & 3))) & 0xFFu);
      y[d] = ((neg >> d) & 1u) ? -m : m;
    }
  }
  if (!ok) {
#pragma unroll
    for (int d = 0; d < kDim; ++d) y[d] = 0;
  }
  return ok;
}

// Shared-memory copy of a codebook's small table-driven decoder tables
// (after the DecodeSharedBase block of class starts and deposit table): the
// index bucket table, the Golay words in weight and in lexicographic order,
// the class records (64 B each) and the state records (32 B each).  Offsets
// in bytes from the start of dynamic shared memory; bytes == 0 when the copy
// would not fit (the decoder then reads them from global memory).
struct TabSmem {
  uint32_t bucket, words, golay, crec, srec, extra, bytes;
};

// `extra` bytes (16-byte aligned) after the tables for the kernel's own use.
// Without `with_words` the two Golay word lists stay in global memory
// (words == golay == 0).
inline TabSmem tab_smem_layout(int n_classes, int n_states, size_t budget, size_t extra = 0,
                               bool with_words = true) {
  TabSmem L{};
  size_t off = (sizeof(DecodeSharedBase) + 15) / 16 * 16;
  const size_t bucket = off; off += ((size_t)kBuckets * 4 + 15) / 16 * 16;
  const size_t words = with_words ? off : 0; off += with_words ? (size_t)kNumGolay * 4 : 0;
  const size_t golay = with_words ? off : 0; off += with_words ? (size_t)kNumGolay * 4 : 0;
  const size_t crec = off; off += (size_t)n_classes * 16 * kTabClassRecords;
  const size_t srec = off; off += (size_t)n_states * 32;
  const size_t ext = off; off += (extra + 15) / 16 * 16;
  if (n_classes > kMaxSmemClasses || off > budget) return L;
  L.bucket = (uint32_t)bucket;
  L.words = (uint32_t)words;
  L.golay = (uint32_t)golay;
  L.crec = (uint32_t)crec;
  L.srec = (uint32_t)srec;
  L.extra = (uint32_t)ext;
  L.bytes = (uint32_t)off;
  return L;
}

// Fill the shared copy (whole block; call __syncthreads() afterwards).
__device__ __forceinline__ void tab_smem_fill(const DevBook& book, uint8_t* smem, const TabSmem& L) {
  uint32_t* bucket = reinterpret_cast<uint32_t*>(smem + L.bucket);
  uint32_t* words = reinterpret_cast<uint32_t*>(smem + L.words);
  uint32_t* golay = reinterpret_cast<uint32_t*>(smem + L.golay);
  uint4* crec = reinterpret_cast<uint4*>(smem + L.crec);
  uint4* srec = reinterpret_cast<uint4*>(smem + L.srec);
  for (int i = threadIdx.x; i < kBuckets; i += blockDim.x)
    bucket[i] = (uint32_t)__ldg(book.bucket + i) | ((uint32_t)__ldg(book.bucket + i + 1) << 16);
  if (L.words)
    for (int i = threadIdx.x; i < kNumGolay; i += blockDim.x) {
      words[i] = __ldg(book.wlist_word + i);
      golay[i] = __ldg(book.golay + i);
    }
  // field-major: record j of class k at j * n_classes + k (spreads a warp's random records over the banks)
  for (int i = threadIdx.x; i < kTabClassRecords * book.n_classes; i += blockDim.x)
    crec[(i % kTabClassRecords) * book.n_classes + i / kTabClassRecords] = __ldg(book.tab.crec + i);
  for (int i = threadIdx.x; i < 2 * book.tab.n_states; i += blockDim.x)
    srec[(i & 1) * book.tab.n_states + (i >> 1)] = __ldg(book.tab.state + i);
}

// The decoder's view of the tables: the small ones from the shared copy
// (SMEM) or from global memory; class starts and the deposit table from
// DecodeSharedBase.
template <bool SMEM>
__device__ __forceinline__ TabCtx tab_ctx(const DevBook& book, const DecodeSharedBase& sh, const uint8_t* smem,
                                          const TabSmem& L) {
  TabCtx tc;
  tc.srec = SMEM ? reinterpret_cast<const uint4*>(smem + L.srec) : book.tab.state;
  tc.crec = SMEM ? reinterpret_cast<const uint4*>(smem + L.crec) : book.tab.crec;
  tc.bucket = book.bucket;
  tc.bucket2 = SMEM ? reinterpret_cast<const uint32_t*>(smem + L.bucket) : nullptr;
  tc.words = SMEM && L.words ? reinterpret_cast<const uint32_t*>(smem + L.words) : book.wlist_word;
  tc.golay = SMEM && L.words ? reinterpret_cast<const uint32_t*>(smem + L.golay) : book.golay;
  tc.starts = book.n_classes <= kMaxSmemClasses ? sh.starts : book.class_start;
  tc.deposit4 = sh.deposit4;
  tc.entry = book.tab.entry;
  tc.slot = book.tab.slot;
  tc.tail = book.tab.tail;
  tc.tail2 = book.tab.tail2;
  tc.expand2 = book.tab.expand2;
  tc.n_classes = book.n_classes;
  tc.n_states = book.tab.n_states;
  tc.max_searches = book.tab.max_searches;
  tc.total = book.total;
  return tc;
}

// ------------------------------------------------ decoded-form helpers
//
// The table-driven decoder's output is the 24 magnitudes by position
// (mag[w], byte j = position 4w + j) and the mask of negative coordinates.

// 2^23 + m as fp32 bits for the magnitude in byte j of w (m < 256).
__device__ __forceinline__ float mag_float_2p23(uint32_t w, int j) {
  return __int_as_float((int)__byte_perm(w, 0x4B000000u, 0x7540u | (uint32_t)j));
}
// fp32(fp32(1/sqrt 8) * m) in one rounding: (2^23 + m) * c - 2^23 * c.
__device__ __forceinline__ float mag_scaled(uint32_t w, int j) {
  return fmaf(mag_float_2p23(w, j), kLatticeScaleF, -8388608.0f * kLatticeScaleF);
}
// Sign bits of positions 2p and 2p + 1 of neg, as the sign bits of a bf16 pair.
__device__ __forceinline__ uint32_t bf16_pair_signs(uint32_t neg, int p) {
  return (((neg >> (2 * p)) & 3u) * 0x40008000u) & 0x80008000u;
}
__device__ __forceinline__ uint32_t bf16_pair(float lo, float hi) {
  const __nv_bfloat162 h = __floats2bfloat162_rn(lo, hi);
  return *reinterpret_cast<const uint32_t*>(&h);
}

// The integer codeword as 12 bf16 pairs (exact: |k| <= 22), positions 2p
// and 2p + 1 in w[p].
__device__ __forceinline__ void bf16_codeword(const uint32_t (&mag)[6], uint32_t neg, uint32_t (&w)[12]) {
#pragma unroll
  for (int p = 0; p < 12; ++p) {
    const uint32_t mw = mag[p >> 1];
    const int j = 2 * (p & 1);
    const float2 f = __fadd2_rn(make_float2(mag_float_2p23(mw, j), mag_float_2p23(mw, j + 1)),
                                make_float2(-8388608.0f, -8388608.0f));
    w[p] = bf16_pair(f.x, f.y) ^ bf16_pair_signs(neg, p);
  }
}

__device__ __forceinline__ int64_t load_index_stream(IndexSource src, int64_t i) {
  if (src.bytes == 8) return __ldcs(static_cast<const long long*>(src.ptr) + i);
  return load_index(src, i);
}

// Decode of a valid or invalid index into (mag, neg); false (and zeros)
// outside the codebook.
template <bool SMEM>
__device__ __forceinline__ bool tab_decode_any(const TabCtx& tc, int64_t v, uint32_t (&mag)[6], uint32_t& neg) {
  bool ok = (uint64_t)v < (uint64_t)tc.total;
  neg = 0;
  if (ok) ok = tab_decode_mn<SMEM>(tc, v, tab_find_class<SMEM>(tc, v), mag, neg);
  if (!ok) {
#pragma unroll
    for (int w = 0; w < 6; ++w) mag[w] = 0;
    neg = 0;
  }
  return ok;
}

}  // namespace llvq
