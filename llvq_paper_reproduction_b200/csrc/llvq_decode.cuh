// Per-index Λ24 decoder shared by the dequantizer and the fused dequant-GEMM.
//
// Index layout and unranking as in the reference's codeword() path
// (impl/leech_lattice_vector_quantizer.py:196-245, :774-867): class by binary
// search over the class starts, a 96-byte decode record (six 16-byte loads),
// the per-class splits by reciprocal multiplication with an exact correction,
// then one 24-step lexicographic unranking loop shared by both parities (an
// even class unranks its |v| = 2 mod 4 part, then its |v| = 0 mod 4 part), so
// warps holding both parities do not diverge there.  Each step finds the value
// whose branch holds the rank, with branch = N * count / remaining computed
// exactly: a shift by the power of two of `remaining` and a multiply by the
// inverse of its odd part (modulo 2^32 once the multinomial N fits 32 bits,
// modulo 2^64 before).  Then the signs.
#pragma once

#include <cstdint>

#include "llvq_device.cuh"

namespace llvq {

constexpr int kMaxSmemClasses = 1024;

struct DecodeShared {
  int64_t starts[kMaxSmemClasses];
  uint64_t inv[kDim + 1];   // inverse of the odd part of d modulo 2^64
  uint32_t shift[kDim + 1]; // trailing zeros of d
};

// Fill the shared tables (call with the whole block, then __syncthreads()).
__device__ __forceinline__ void decode_setup(const DevBook& book, DecodeShared& sh) {
  if (book.n_classes <= kMaxSmemClasses)
    for (int k = threadIdx.x; k < book.n_classes; k += blockDim.x) sh.starts[k] = book.class_start[k];
  if (threadIdx.x <= kDim && threadIdx.x > 0) {
    const uint32_t d = threadIdx.x, s = __ffs(d) - 1;
    sh.shift[d] = s;
    sh.inv[d] = inv_odd64(d >> s);
  }
}

__device__ __forceinline__ uint32_t byte_at(uint64_t packed, int j) { return (uint32_t)(packed >> (8 * j)) & 0xFFu; }

// a / b for a < 2^63, b >= 1, with inv_b ~ 1/b: a reciprocal estimate fixed
// up by one exact step; hardware division for a >= 2^52 (huge codebooks only).
__device__ __forceinline__ uint64_t div_recip(uint64_t a, uint64_t b, double inv_b, uint64_t& rem) {
  uint64_t q;
  if (a >> 52) {
    q = a / b;
  } else {
    q = (uint64_t)__dmul_rz((double)a, inv_b);
    int64_t r = (int64_t)(a - q * b);
    if (r < 0) { --q; r += (int64_t)b; }
    else if ((uint64_t)r >= b) { ++q; r -= (int64_t)b; }
  }
  rem = a - q * b;
  return q;
}

// One unranking step: the value index whose branch holds `rank`; updates
// rank, N (multinomial of what remains) and the packed counts.
__device__ __forceinline__ uint32_t unrank_step(uint64_t& rank, uint64_t& N, uint64_t& cnt, int rem,
                                                const DecodeShared& sh) {
  const uint32_t s = sh.shift[rem];
  uint32_t j = 0;
  if (N >> 32) {
    const uint64_t inv = sh.inv[rem];
    for (; j < kMaxVals; ++j) {
      const uint64_t c = byte_at(cnt, j);
      if (!c) continue;
      const uint64_t br = ((N * c) >> s) * inv;
      if (rank < br) { N = br; break; }
      rank -= br;
    }
  } else {
    const uint32_t inv = (uint32_t)sh.inv[rem];
    uint32_t r = (uint32_t)rank, n32 = (uint32_t)N;
    // The smallest remaining value (tried last) is usually the most frequent
    // one: test its branch, the top of the rank range, first.
    const uint32_t last = (uint32_t)(63 - __clzll((long long)cnt)) >> 3;
    const uint32_t blast = (uint32_t)(((uint64_t)n32 * byte_at(cnt, last)) >> s) * inv;
    if (r >= n32 - blast) {
      rank = r - (n32 - blast);
      N = blast;
      cnt -= 1ull << (8 * last);
      return last;
    }
    for (; j < kMaxVals; ++j) {
      const uint32_t c = byte_at(cnt, j);
      if (!c) continue;
      const uint32_t br = (uint32_t)(((uint64_t)n32 * c) >> s) * inv;
      if (r < br) { n32 = br; break; }
      r -= br;
    }
    rank = r;
    N = n32;
  }
  cnt -= 1ull << (8 * j);
  return j;
}

// Integer codeword of index v (before the 1/sqrt(8) scale); false and zeros
// when v is outside the codebook.
__device__ __forceinline__ bool decode_index(int64_t v, const DevBook& book, const DecodeShared& sh, int (&y)[kDim]) {
  bool ok = v >= 0 && v < book.total;
  if (ok) {
    const int k = find_class(book.n_classes <= kMaxSmemClasses ? sh.starts : book.class_start, book.n_classes, v);
    const uint4* rp = reinterpret_cast<const uint4*>(book.dcls + k);
    const uint4 w0 = __ldg(rp), w1 = __ldg(rp + 1), w2 = __ldg(rp + 2), w3 = __ldg(rp + 3), w4 = __ldg(rp + 4),
                w5 = __ldg(rp + 5);
    auto u64 = [](uint32_t lo, uint32_t hi) { return ((uint64_t)hi << 32) | lo; };
    const uint64_t start = u64(w0.x, w0.y), perm = u64(w0.z, w0.w);
    const double inv_perm = __longlong_as_double((long long)u64(w1.x, w1.y));
    const uint64_t f0p = u64(w1.z, w1.w);
    const uint32_t f1p = w2.x, meta = w2.y, gbase = w2.z;
    const double inv_f1 = __longlong_as_double((long long)u64(w3.x, w3.y));
    const uint64_t pv0 = u64(w3.z, w3.w), pm0 = u64(w4.x, w4.y), pv1 = u64(w4.z, w4.w), pm1 = u64(w5.x, w5.y);
    const bool odd = meta & 1;
    const int weight = (meta >> 1) & 31, sshift = (meta >> 6) & 31;
    uint64_t prank;
    const uint64_t cur = div_recip((uint64_t)v - start, perm, inv_perm, prank);
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
      const uint64_t r0 = div_recip(prank, f1p, inv_f1, r1);
      rank = r1;
      N = f1p;
      cnt = pm1;
      rank2 = r0;
      N2 = f0p;
      cnt2 = pm0;
      nfirst = weight;
    }
    uint64_t seq_lo = 0, seq_hi = 0;  // 4-bit value indices, step order
#pragma unroll
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
    int i0 = 0, i1 = 0;
#pragma unroll
    for (int d = 0; d < kDim; ++d) {
      const bool bit = (word >> d) & 1u;
      const bool part1 = !odd && bit;
      const int t = odd ? d : (bit ? i1 : nfirst + i0);
      const uint32_t nib = (uint32_t)((t < 16 ? seq_lo >> (4 * t) : seq_hi >> (4 * (t - 16))) & 15u);
      const int m = (int)byte_at(part1 ? pv1 : pv0, (int)nib);
      i1 += part1;
      i0 += !odd && !bit;
      y[d] = odd ? (((m & 3) == (bit ? 3 : 1)) ? m : -m) : m;
    }
    if (!odd) ok = unrank_even_signs(y, sign, (meta >> 19) & 1);
  }
  if (!ok) {
#pragma unroll
    for (int d = 0; d < kDim; ++d) y[d] = 0;
  }
  return ok;
}

}  // namespace llvq
