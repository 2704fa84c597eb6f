// Per-index Λ24 decoder shared by the dequantizer and the fused dequant-GEMM.
//
// Index layout and unranking as in the reference's codeword() path
// (impl/leech_lattice_vector_quantizer.py:196-245, :774-867): class by binary
// search over the class starts, a 96-byte decode record (six 16-byte loads),
// the per-class splits by reciprocal multiplication with an exact correction,
// then one 24-step lexicographic unranking loop shared by both parities (an
// even class unranks its |v| = 2 mod 4 part, then its |v| = 0 mod 4 part), so
// warps holding both parities do not diverge there.  Lexicographic
// unranking picks, at each step, the value whose branch [N*C_{j-1}/rem,
// N*C_j/rem) holds the rank (C = cumulative counts, N the multinomial of
// what remains, rem the positions left), i.e. the bucket of
// t = floor(rank * rem / N) among the cumulative counts.  Once N fits 32
// bits, t is estimated in fp32, the bucket found with a byte-wise compare of
// the packed cumulative counts, and the choice verified exactly with two
// 32x32->64 products (a miss, at an fp32 rounding boundary, is stepped to
// the neighbouring bucket).  The new rank and N are exact divisions by rem:
// a shift by its power of two and a multiply by the inverse of its odd part
// (mod 2^32).  Larger N (the first steps of the largest classes) use the
// 64-bit branch-by-branch scan.  Even-class signs use the closed form of
// rank_even_signs (llvq_device.cuh) inside the scatter loop.
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
    // scatter: odd -> step d at position d; even -> the word's positions take
    // the first (f1) part in order, the others the second (f0) part
    uint32_t nzmask = 0;
#pragma unroll
    for (int d = 0; d < kDim; ++d) {
      const bool bit = (word >> d) & 1u;
      const bool part1 = !odd && bit;
      const int below1 = __popc(word & ((1u << d) - 1u));
      const int t = odd ? d : (bit ? below1 : nfirst + d - below1);
      const uint32_t nib = (uint32_t)((t < 16 ? seq_lo >> (4 * t) : seq_hi >> (4 * (t - 16))) & 15u);
      const int m = (int)byte_at(part1 ? pv1 : pv0, (int)nib);
      nzmask |= (uint32_t)(m != 0) << d;
      y[d] = odd ? (((m & 3) == (bit ? 3 : 1)) ? m : -m) : m;
    }
    if (!odd) {
      // signs: insert, at the first word coordinate, the bit that gives the
      // class's parity of negative word coordinates (weight 0: rank = mask)
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
      uint32_t neg = 0;
      int ci = 0;
#pragma unroll
      for (int d = 0; d < kDim; ++d) {
        const bool nzd = (nzmask >> d) & 1u;
        neg |= (nzd ? (cmask >> ci) & 1u : 0u) << d;
        ci += nzd;
      }
      if (word && (__popc(neg & word) & 1) != (int)((meta >> 19) & 1)) neg ^= word & (0u - word);
#pragma unroll
      for (int d = 0; d < kDim; ++d) y[d] = ((neg >> d) & 1u) ? -y[d] : y[d];
    }
  }
  if (!ok) {
#pragma unroll
    for (int d = 0; d < kDim; ++d) y[d] = 0;
  }
  return ok;
}

}  // namespace llvq
