// Shared host/device definitions for the Λ24 (Leech lattice) codebook:
// table layout in device memory and the exact integer rank/unrank maths that
// turn a codeword into its hierarchical index and back.
//
// Index layout (reference impl/leech_lattice_vector_quantizer.py):
//   global = class_start + local                         (rank_class, :187-194; offsets :336-353)
//   local  = (golay_choice * sign_count + sign_choice) * perm_count + perm
//                                                        (rank_class_codeword, :692-708)
//   even perm = f0_rank * f1_perm + f1_rank              (rank_even_codeword, :711-737)
// Multiset ranks are lexicographic with values tried in descending order
// (rank_multiset_sequence :870-889); the even sign rank orders the valid
// negative-masks (signed sum = 0 mod 8) by their value as integers, bit i =
// i-th nonzero coordinate (rank_even_signs :819-841).
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define LLVQ_HD __host__ __device__ __forceinline__
#else
#define LLVQ_HD inline
#endif

namespace llvq {

constexpr int kDim = 24;
constexpr int kNumGolay = 4096;
constexpr int kMaxVals = 8;           // distinct magnitudes per class part
constexpr uint32_t kFull24 = 0xFFFFFFu;
// 1.0 / sqrt(8.0) rounded to double exactly as CPython evaluates it.
constexpr double kLatticeScaleD = 0.35355339059327373;
// The same constant rounded to fp32 (what torch multiplies by in fp32).
constexpr float kLatticeScaleF = 0.35355339059327373f;
constexpr float kSqrt8F = 2.8284270763397216796875f;  // fp32(sqrt(8))
constexpr int kQBits = 19;            // |q| <= 2^19 keeps every suffix sum exact in fp32

// Per-class tables (global order: shell ascending, reference class order inside a shell).
struct DevClass {
  int64_t start;        // global index of the first codeword of the class
  uint64_t perm_count;  // f0_perm * f1_perm (even) or multinomial (odd)
  uint64_t sign_count;  // power of two (even) or 1 (odd)
  uint64_t f1_perm;     // multinomial of the |v| = 2 mod 4 part (even), 1 (odd)
  int32_t shell;
  int32_t parity;       // 0 even, 1 odd
  int32_t even_weight;  // #coords with |v| = 2 mod 4 (even)
  int32_t required;     // (sum(leader) % 8) / 4 (even)
  int32_t golay_count;
  int32_t sign_shift;   // log2(sign_count)
  int32_t nv0, nv1;     // distinct values: even f0 / f1 part, odd: all magnitudes in nv0
  int32_t v0[kMaxVals], m0[kMaxVals];  // descending values and multiplicities
  int32_t v1[kMaxVals], m1[kMaxVals];
  int8_t asc0[kDim];    // even: f0 magnitudes ascending; odd: signed values ascending
  int8_t asc1[kDim];    // even: f1 magnitudes ascending
  int32_t l1;           // sum of the leader
  int32_t nterms;       // FFMA chain used by the table-driven search
  float term_coef[16];
  int8_t term_kind[16]; // 0 = R, 1 = R0, 2 = R1, 3 = P0, 4 = P1
  int8_t term_idx[16];
};

// Compact per-class record for the decoders: 96 bytes, read with six 16-byte
// loads and kept in registers (values and multiplicities packed as bytes,
// reciprocals for the two per-class divisions).
struct alignas(16) DecodeClass {
  int64_t start;
  uint64_t perm_count;
  uint64_t magic_perm;  // floor((2^64 - 1) / perm_count), for div_magic
  uint64_t f0_perm;     // perm_count / f1_perm
  uint32_t f1_perm;     // 1 for odd classes
  uint32_t meta;        // parity | even_weight << 1 | sign_shift << 6 | nv0 << 11 | nv1 << 15 | required << 19
                        // | kMetaFast (the decoder's four-value fast path applies)
                        // | kMetaWide (its eight-value, 64-bit variant applies)
  uint32_t golay_base;  // even: start of its weight group in by_weight
  uint32_t pad;
  uint64_t magic_f1;    // floor((2^64 - 1) / f1_perm)
  uint64_t v0, m0, v1, m1;  // byte j = j-th value / multiplicity (descending values)
};
static_assert(sizeof(DecodeClass) == 96, "decode record is six 16-byte loads");
constexpr uint32_t kMetaFast = 1u << 20;
constexpr uint32_t kMetaWide = 1u << 21;

// Tail table of the decoder: the last kTailLen steps of a part of at most
// four values are one lookup.  Block of the count vector (n0..n3), n0 + ... +
// n3 = 8, at tail_off[c0 * 81 + c1 * 9 + c2] (cumulative c0 = n0, c1 = n0 +
// n1, c2 = n0 + n1 + n2); inside it, the multinomial(n) sequences in
// lexicographic order (value 0 first), value index of step i in bits 2i..2i+1.
constexpr int kTailLen = 8;
constexpr int kTailKeys = 9 * 9 * 9;
constexpr int kTailSeqs = 1 << (2 * kTailLen);

// Tables of the table-driven decoder in global memory (layout in
// llvq_tables.cuh); state == nullptr when the codebook is not tabulated.
struct TabView {
  const uint4* state;      // 2 per state
  const uint4* crec;       // 3 per class
  const uint4* entry;
  const uint4* slot;
  const unsigned long long* tail;
  const uint32_t* tail2;   // bit-plane tails
  const uint4* expand2;    // bit-plane deposit masks per Golay word in weight order
  int n_states;
  int max_searches;        // searches of the longest class (both parts)
};

// Everything a kernel needs about one codebook (plain pointers, passed by value).
struct DevBook {
  const DevClass* cls;
  const DecodeClass* dcls;        // [n_classes] compact decode records
  const uint16_t* bucket;         // [kBuckets + 1] class holding the lowest index of each bucket
  const int64_t* class_start;     // [n_classes] (binary search)
  const uint32_t* golay;          // [4096] lexicographic order, bit d = coordinate d
  const uint16_t* golay_wrank;    // [4096] position among the words of equal weight
  const uint32_t* wlist_word;     // [4096] words sorted by (weight, lex)
  const uint16_t* wlist_lex;      // [4096] their lexicographic indices
  const uint16_t* by_weight;      // [4096] lex indices grouped by weight (lex order inside)
  const uint32_t* plist_word;     // [2048] the lighter word of each complementary pair, weights 0, 8, 12 in order
  const uint16_t* plist_lex;      // [2048] its lexicographic index (the complement's is 4095 minus it)
  const uint32_t* tail_off;       // [kTailKeys] start of each count vector's block in tail_seq
  const uint16_t* tail_seq;       // [kTailSeqs] every 8-step sequence over 4 values, by count vector then rank
  int32_t weight_start[25];       // start of each weight group in by_weight
  int32_t n_classes;
  int32_t min_shell, max_shell;
  int64_t total;
  // window constants of the active scoring code (see quantize.cu)
  float l1max, win_mg, win_am;
  // table-driven decoder (llvq_tables.cuh); state == nullptr when the
  // codebook is not tabulated
  TabView tab;
};

// ---------------------------------------------------------------- integers

// Exact v / d for 1 <= d <= 24 when d divides v: shift out the power of two,
// multiply by the inverse of the odd part modulo 2^64.
LLVQ_HD uint64_t inv_odd64(uint64_t o) {
  uint64_t x = o;  // Newton iteration x <- x(2 - o x) doubles the correct low bits
  for (int i = 0; i < 5; ++i) x *= 2 - o * x;
  return x;
}

LLVQ_HD uint64_t exact_div_small(uint64_t v, uint32_t d) {
#if defined(__CUDA_ARCH__)
  const int s = __ffs(d) - 1;
#else
  const int s = __builtin_ctz(d);
#endif
  return (v >> s) * inv_odd64(d >> s);
}

// Lexicographic rank of `seq` (length n) among the orderings of the multiset
// (vals descending, mult), trying values in descending order.  `total` is the
// multinomial of the full multiset.  Returns UINT64_MAX if seq is not an
// ordering of the multiset.
LLVQ_HD uint64_t rank_multiset(const int* seq, int n, const int32_t* vals, const int32_t* mult, int nv,
                               uint64_t total) {
  int cnt[kMaxVals];
  for (int j = 0; j < kMaxVals; ++j) cnt[j] = j < nv ? mult[j] : 0;
  uint64_t N = total, rank = 0;
  int rem = n;
  for (int i = 0; i < n; ++i) {
    const int a = seq[i];
    int ja = -1;
    for (int j = 0; j < nv; ++j) {
      if (vals[j] == a) { ja = j; break; }
      if (cnt[j]) rank += exact_div_small(N * (uint64_t)cnt[j], (uint32_t)rem);
    }
    if (ja < 0 || cnt[ja] == 0) return UINT64_MAX;
    N = exact_div_small(N * (uint64_t)cnt[ja], (uint32_t)rem);
    cnt[ja]--;
    rem--;
  }
  return rank;
}

// Inverse of rank_multiset.  Returns false if rank >= total.
LLVQ_HD bool unrank_multiset(uint64_t rank, const int32_t* vals, const int32_t* mult, int nv, int n, uint64_t total,
                             int* out) {
  if (rank >= total) return false;
  int cnt[kMaxVals];
  for (int j = 0; j < kMaxVals; ++j) cnt[j] = j < nv ? mult[j] : 0;
  uint64_t N = total;
  int rem = n;
  for (int i = 0; i < n; ++i) {
    int pick = -1;
    for (int j = 0; j < nv; ++j) {
      if (!cnt[j]) continue;
      const uint64_t br = exact_div_small(N * (uint64_t)cnt[j], (uint32_t)rem);
      if (rank < br) { pick = j; N = br; break; }
      rank -= br;
    }
    if (pick < 0) return false;
    out[i] = vals[pick];
    cnt[pick]--;
    rem--;
  }
  return true;
}

// Number of sign patterns of the nonzero coordinates below the current one
// (f0n with |v| = 0 mod 4, f1n with |v| = 2 mod 4, all-positive sum = fixed
// mod 8) whose signed sum is `need` mod 8.  Flipping a |v| = 0 mod 4 value
// moves the sum by 0 mod 8, a |v| = 2 mod 4 value by 4 mod 8.
LLVQ_HD uint64_t lower_sign_count(int f0n, int f1n, int fixed, int need) {
  const int delta = (need - fixed) & 7;
  if (delta != 0 && delta != 4) return 0;
  if (f1n == 0) return delta == 0 ? (1ull << f0n) : 0ull;
  return 1ull << (f0n + f1n - 1);
}

// Even sign patterns (rank_even_signs / apply_even_signs of the reference,
// impl/leech_lattice_vector_quantizer.py:804-841): masks over the nonzero
// coordinates (bit i = i-th nonzero coordinate negative) whose signed sum is
// 0 mod 8, counted in increasing mask order.  Only coordinates with
// |v| = 2 (mod 4) -- the Golay word's positions -- move the sum mod 8 (by 4),
// so a mask is valid iff its count of negative word coordinates has the
// class's parity.  With p the bit of the first word coordinate, deleting bit
// p maps the valid masks onto all masks of the remaining bits and preserves
// their order (masks that agree above p and differ below it agree at p,
// because no word coordinate lies below p).  So the rank is the mask with bit
// p deleted, and unranking inserts the bit that fixes the parity.  Without
// word coordinates (weight-0 classes) every mask is valid and rank = mask.

// Rank of the sign pattern of even codeword y; UINT64_MAX if its signed sum
// is not 0 mod 8.
LLVQ_HD uint64_t rank_even_signs(const int* y) {
  int sum = 0, nz = 0, p = -1;
  uint32_t mask = 0;
  for (int d = 0; d < kDim; ++d) {
    sum += y[d];
    const int a = y[d] < 0 ? -y[d] : y[d];
    if (!a) continue;
    if (p < 0 && (a & 3) == 2) p = nz;
    if (y[d] < 0) mask |= 1u << nz;
    nz++;
  }
  if (sum & 7) return UINT64_MAX;
  if (p < 0) return mask;
  return ((uint64_t)(mask >> (p + 1)) << p) | (mask & ((1u << p) - 1u));
}

// Apply the sign pattern of rank `rank` to the nonnegative magnitudes v of an
// even class whose signed sum must have negative-word-coordinate parity
// `required`.
LLVQ_HD bool unrank_even_signs(int* v, uint64_t rank, int required) {
  int nz = 0, p = -1;
  for (int d = 0; d < kDim; ++d) {
    if (!v[d]) continue;
    if (p < 0 && (v[d] & 3) == 2) p = nz;
    nz++;
  }
  uint32_t mask;
  if (p < 0) {
    if (nz < 32 && (rank >> nz)) return false;
    mask = (uint32_t)rank;
  } else {
    if (rank >> (nz - 1)) return false;
    const uint32_t r = (uint32_t)rank;
    mask = ((r >> p) << (p + 1)) | (r & ((1u << p) - 1u));
    int negw = 0, i = 0;
    for (int d = 0; d < kDim; ++d) {
      if (!v[d]) continue;
      if ((v[d] & 3) == 2 && ((mask >> i) & 1u)) negw++;
      i++;
    }
    if ((negw & 1) != required) mask |= 1u << p;
  }
  int i = 0;
  for (int d = 0; d < kDim; ++d) {
    if (!v[d]) continue;
    if ((mask >> i) & 1u) v[d] = -v[d];
    i++;
  }
  return true;
}

// codeword (integer coordinates, before the 1/sqrt(8) scale) -> global index
// within the given class and Golay word; returns -1 if y is not in the class.
LLVQ_HD int64_t rank_codeword(const DevClass& c, const int* y, uint32_t word, int golay_choice) {
  uint64_t local;
  if (c.parity == 0) {
    int s0[kDim], s1[kDim], n0 = 0, n1 = 0;
    for (int d = 0; d < kDim; ++d) {
      const int a = y[d] < 0 ? -y[d] : y[d];
      if ((word >> d) & 1u) s1[n1++] = a; else s0[n0++] = a;
    }
    const uint64_t f0_perm = c.perm_count / c.f1_perm;
    const uint64_t r0 = rank_multiset(s0, n0, c.v0, c.m0, c.nv0, f0_perm);
    const uint64_t r1 = rank_multiset(s1, n1, c.v1, c.m1, c.nv1, c.f1_perm);
    const uint64_t sr = rank_even_signs(y);
    if (r0 == UINT64_MAX || r1 == UINT64_MAX || sr == UINT64_MAX || sr >= c.sign_count) return -1;
    const uint64_t perm = r0 * c.f1_perm + r1;
    local = (((uint64_t)golay_choice << c.sign_shift) + sr) * c.perm_count + perm;
  } else {
    int mags[kDim];
    for (int d = 0; d < kDim; ++d) mags[d] = y[d] < 0 ? -y[d] : y[d];
    const uint64_t r = rank_multiset(mags, kDim, c.v0, c.m0, c.nv0, c.perm_count);
    if (r == UINT64_MAX) return -1;
    local = (uint64_t)golay_choice * c.perm_count + r;
  }
  return (int64_t)((uint64_t)c.start + local);
}

// Decompose a class-local index and build the integer codeword.
// `word_of_choice` maps a Golay choice to the Golay word bits.
template <class WordOf>
LLVQ_HD bool unrank_codeword(const DevClass& c, uint64_t local, WordOf word_of_choice, int* out) {
  const uint64_t cur = local / c.perm_count;
  const uint64_t perm = local - cur * c.perm_count;
  if (c.parity == 0) {
    const uint64_t sign = cur & (c.sign_count - 1);
    const uint64_t g = cur >> c.sign_shift;
    if (g >= (uint64_t)c.golay_count) return false;
    const uint32_t word = word_of_choice((int)g);
    const uint64_t f0_perm = c.perm_count / c.f1_perm;
    const uint64_t r0 = perm / c.f1_perm, r1 = perm - r0 * c.f1_perm;
    int s0[kDim], s1[kDim];
    const int n1 = c.even_weight, n0 = kDim - n1;
    if (!unrank_multiset(r0, c.v0, c.m0, c.nv0, n0, f0_perm, s0)) return false;
    if (!unrank_multiset(r1, c.v1, c.m1, c.nv1, n1, c.f1_perm, s1)) return false;
    int i0 = 0, i1 = 0;
    for (int d = 0; d < kDim; ++d) out[d] = ((word >> d) & 1u) ? s1[i1++] : s0[i0++];
    return unrank_even_signs(out, sign, c.required);
  }
  if (cur >= (uint64_t)kNumGolay) return false;
  const uint32_t word = word_of_choice((int)cur);
  int mags[kDim];
  if (!unrank_multiset(perm, c.v0, c.m0, c.nv0, kDim, c.perm_count, mags)) return false;
  for (int d = 0; d < kDim; ++d) {
    const int target = ((word >> d) & 1u) ? 3 : 1;
    out[d] = ((mags[d] & 3) == target) ? mags[d] : -mags[d];
  }
  return true;
}

// Class containing a global index: last class whose start is <= index.
// Index buckets for the class search: a bucket is an index's leading bit
// and the four bits after it (relative width 1/16, like a float with a 4-bit
// mantissa), so the exponentially growing shells and classes spread over a
// few buckets each.  Bucket 0 holds index 0; bucket 1 + 16 e + j the indices
// with leading bit e and next four bits j.  bucket_low(b) is the smallest
// index of bucket b (all-ones past the last bucket).
constexpr int kBuckets = 1 + 64 * 16;

LLVQ_HD uint64_t bucket_low(int b) {
  if (b <= 0) return 0;
  const int e = (b - 1) / 16;
  const uint64_t j = (uint64_t)((b - 1) % 16);
  if (e >= 64) return ~0ull;
  return (1ull << e) + (e >= 4 ? j << (e - 4) : (j << e) >> 4);
}

LLVQ_HD int find_class(const int64_t* starts, int n, int64_t index) {
  int lo = 0, hi = n;
  while (lo + 1 < hi) {
    const int mid = (lo + hi) >> 1;
    if ((uint64_t)starts[mid] <= (uint64_t)index) lo = mid; else hi = mid;
  }
  return lo;
}

}  // namespace llvq
