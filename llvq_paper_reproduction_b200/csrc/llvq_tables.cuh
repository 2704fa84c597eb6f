// Table-driven Λ24 decoder, shared by the GPU kernels and a host entry point.
//
// The integer codeword of an index is fixed by its class, its Golay word, its
// even-class sign pattern and, per class part, the lexicographic rank of the
// part's magnitude sequence among the orderings of its multiset (values tried
// in descending order; impl/leech_lattice_vector_quantizer.py:844-867).  The
// arithmetic unranking needs one step per coordinate (24 for an odd class).
// Here a part's sequence comes from a few table lookups instead, keyed by the
// multiset still to place (a "state": the counts of the part's values that
// remain, shared by every class with the same counts):
//   * a tail state (at most kTabTail positions left) lists all its orderings
//     in rank order, so the rest of the sequence is entry `rank`;
//   * a search state lists the orderings of its next h positions (h at most
//     kTabHead) in rank order, each with the rank of its first completion
//     and the state it leaves; a slot table over rank * G / N (N the number
//     of orderings of the state, G a power of two, the slot computed exactly)
//     holds, for a slot inside one entry, that entry itself (one gather), and
//     for a slot that reaches into a second entry the number of the entry
//     holding its first rank (then compared with the following entries).
// A 24-position part is two searches and one tail; a 16-position part one
// search and one tail; 12- and 8-position parts one tail.  Every lane runs
// its searches first (part A's, then part B's; at most tc.max_searches) and
// then its tails, so the lanes of a warp run the same lookup code together.  Sequences are
// nibble strings (value index j of the part in bits 4t..4t+3 for step t).
// The two parts of an even class are then moved onto their positions (the
// word's coordinates and the others) by a nibble-wise bit expand (the
// inverse of compress; H. S. Warren, Hacker's Delight, 2nd ed., section 7-5)
// with move masks precomputed per Golay word, and a byte permute turns value
// indices into magnitudes, four positions at a time.
#pragma once

#include <cstdint>

#include "llvq_device.cuh"

namespace llvq {

constexpr int kTabTail = 12;              // positions a tail state covers
constexpr int kTabHead = 6;               // positions one search covers
constexpr uint32_t kTabEnd = 0xFFFFFFFFu; // no state: the part is empty / finished
constexpr int kTabExpandWords = 40;       // u32 per Golay word in the expand table
constexpr uint32_t kTabTailBit = 1u << 31;
constexpr uint32_t kTabSlotAmbiguous = 1u << 31;
constexpr int kTabMaxStateEntries = 0x10000;

// State record, two uint4:
//   [0] tail:   x = first entry in `tail`, z = kTabTailBit | positions
//       search: x = first entry in `entry`, y = first slot,
//               z = entries | log2 G << 16 | h << 21
//   [1] search: N (u64, x | y << 32), G / N as fp64 bits (z | w << 32)
// Search entry (uint4): {start low, start high, next state, nibbles of the h
// positions}; starts stay below 2^46.  Slot g (uint4) covers the ranks
// ceil(g N / G) .. ceil((g + 1) N / G) - 1: the entry holding all of them, or
// {number of the entry holding the first, kTabSlotAmbiguous, 0, 0}.
//
// Class record, four uint4 (64 bytes):
//   [0] start of the class (u64), permutation count (u64)
//   [1] floor((2^64 - 1) / permutation count), floor((2^64 - 1) / f1 count)
//   [2] values (u64: byte j = value j; even: the |v| = 0 mod 4 part's values,
//       then the |v| = 2 mod 4 part's from byte d0 on), f1 count (u32), meta
//   [3] first word of the class's weight group in weight order (u32), state of
//       part A, state of part B, 0
// meta: odd | word weight << 1 | sign shift << 6 | d0 << 11 | required << 15.
// Part A is the odd class's only part or the even class's |v| = 2 (mod 4)
// part on the word's positions; part B the even class's |v| = 0 (mod 4) part
// on the other positions.
//
// Words are indexed in weight order (lexicographic inside a weight): an even
// class's word is entry wbase + choice; every odd class uses entry 4095 (the
// all-ones word: part A on every position) of the expand table.

#if defined(__CUDA_ARCH__)
template <class T>
__device__ __forceinline__ T tab_ldg(const T* p) { return __ldg(p); }
__device__ __forceinline__ uint32_t tab_prmt(uint32_t a, uint32_t b, uint32_t s) { return __byte_perm(a, b, s); }
__device__ __forceinline__ uint32_t tab_fshl(uint32_t lo, uint32_t hi, int s) { return __funnelshift_l(lo, hi, s); }
__device__ __forceinline__ double tab_bits2d(uint32_t lo, uint32_t hi) {
  return __hiloint2double((int)hi, (int)lo);
}
__device__ __forceinline__ uint64_t tab_mulhi(uint64_t a, uint64_t b) { return __umul64hi(a, b); }
__device__ __forceinline__ int tab_popc(uint32_t v) { return __popc(v); }
__device__ __forceinline__ int tab_msb(uint64_t u) { return 63 - __clzll((long long)u); }
#else
template <class T>
inline T tab_ldg(const T* p) { return *p; }
inline uint32_t tab_prmt(uint32_t a, uint32_t b, uint32_t s) {
  const uint64_t v = ((uint64_t)b << 32) | a;
  uint32_t out = 0;
  for (int i = 0; i < 4; ++i) out |= (uint32_t)((v >> (8 * ((s >> (4 * i)) & 7))) & 0xFF) << (8 * i);
  return out;
}
inline uint32_t tab_fshl(uint32_t lo, uint32_t hi, int s) { return s ? (hi << s) | (lo >> (32 - s)) : hi; }
inline double tab_bits2d(uint32_t lo, uint32_t hi) {
  const uint64_t b = ((uint64_t)hi << 32) | lo;
  double d;
  __builtin_memcpy(&d, &b, 8);
  return d;
}
inline uint64_t tab_mulhi(uint64_t a, uint64_t b) { return (uint64_t)(((unsigned __int128)a * b) >> 64); }
inline int tab_popc(uint32_t v) { return __builtin_popcount(v); }
inline int tab_msb(uint64_t u) { return 63 - __builtin_clzll(u); }
#endif

LLVQ_HD uint64_t tab_u64(uint32_t lo, uint32_t hi) { return ((uint64_t)hi << 32) | lo; }

// Where the decoder reads its tables.  The small ones marked SMEM point to
// shared-memory copies (plain loads) or to global memory (read-only cache
// loads); starts and deposit4 are read with plain loads (shared memory in
// the kernels); the rest is global memory.
struct TabCtx {
  const uint4* srec;          // 2 per state                          (SMEM)
  const uint4* crec;          // 4 per class                          (SMEM)
  const uint16_t* bucket;     // index bucket -> class                (SMEM)
  const uint32_t* words;      // Golay words in weight order          (SMEM)
  const uint32_t* golay;      // Golay words in lexicographic order   (SMEM)
  const int64_t* starts;      // class starts (binary search)         (plain loads)
  const uint8_t* deposit4;    // [m * 16 + s]: the low popc(m) bits of s placed on the set bits of m (plain)
  const uint4* entry;
  const uint4* slot;
  const unsigned long long* tail;
  const uint4* expand;        // kTabExpandWords u32 per word, weight order
  int n_classes;
  int max_searches;           // searches of the longest class (both parts)
  int64_t total;
};

template <bool SMEM, class T>
LLVQ_HD T tab_ldr(const T* p) {
  if constexpr (SMEM) return *p;
  else return tab_ldg(p);
}

// One search from search state s (record r0) with rank r: the nibbles of
// the h positions it covers; s becomes the state left, r the rank within it.
template <bool SMEM>
LLVQ_HD void tab_search(const TabCtx& tc, const uint4& r0, uint32_t& s, uint64_t& r, uint64_t& nib, int& take) {
  const uint4 r1 = tab_ldr<SMEM>(tc.srec + 2 * s + 1);
  const uint32_t n = r0.z & 0x1FFFFu, lg = (r0.z >> 17) & 31u;
  const uint64_t N = tab_u64(r1.x, r1.y), rg = r << lg;
  // slot g = floor(r G / N): an fp64 estimate, corrected exactly (N (G + 1) < 2^64)
  uint64_t g = (uint64_t)((double)r * tab_bits2d(r1.z, r1.w));
  if ((g + 1) * N <= rg) ++g;
  else if (g * N > rg) --g;
  uint4 e = tab_ldg(tc.slot + r0.y + (uint32_t)g);
  if (e.y & kTabSlotAmbiguous) {
    const uint4* ent = tc.entry + r0.x;
    uint32_t j = e.x;
    e = tab_ldg(ent + j);
    while (j + 1 < n) {
      const uint2 nx = tab_ldg(reinterpret_cast<const uint2*>(ent + j + 1));
      if (tab_u64(nx.x, nx.y) > r) break;
      ++j;
      e = tab_ldg(ent + j);
    }
  }
  r -= tab_u64(e.x, e.y);
  s = e.z;
  nib = e.w;
  take = (int)((r0.z >> 22) & 15u);
}

LLVQ_HD void tab_put(uint64_t& lo, uint64_t& hi, uint64_t nib, int t) {
  const int sh = 4 * t;
  if (sh < 64) {
    lo |= nib << sh;
    if (sh) hi |= nib >> (64 - sh);
  } else {
    hi |= nib << (sh - 64);
  }
}

// 96-bit (three u32) shift left by a constant number of bits.
template <int S>
LLVQ_HD void tab_shl96(const uint32_t (&x)[3], uint32_t (&t)[3]) {
  if constexpr (S == 64) {
    t[2] = x[0]; t[1] = 0; t[0] = 0;
  } else if constexpr (S == 32) {
    t[2] = x[1]; t[1] = x[0]; t[0] = 0;
  } else {
    t[2] = tab_fshl(x[1], x[2], S);
    t[1] = tab_fshl(x[0], x[1], S);
    t[0] = x[0] << S;
  }
}

// Expand table layout, per Golay word (weight order), kTabExpandWords u32 as
// five 32-byte stages q = 0..4 (applied in that order; stage q moves nibbles
// by 2^(4-q) positions): {A0, A1, A2, B0}, {B1, B2, M_q, 0}, where A0..A2 /
// B0..B2 are the nibble-wide move masks of the expand by the word / by its
// complement (three u32 covering positions 0-7, 8-15, 16-23) and M_0..M_2
// the word itself widened to nibbles.
//
// Nibble-wise expand of both parts at once: source nibble t of xa goes to
// the t-th position of the word, source nibble t of xb to the t-th position
// outside it; m receives the word's nibble mask.  Positions outside each
// part's mask hold garbage.
LLVQ_HD void tab_expand2(uint32_t (&xa)[3], uint32_t (&xb)[3], const uint4* e, uint32_t (&m)[3]) {
  uint32_t t[3];
#define LLVQ_EXPAND_STAGE(Q, S)                                                           \
  {                                                                                        \
    const uint4 u = tab_ldg(e + 2 * (Q)), v = tab_ldg(e + 2 * (Q) + 1);                     \
    const uint32_t ma[3] = {u.x, u.y, u.z}, mb[3] = {u.w, v.x, v.y};                      \
    if ((Q) < 3) m[(Q) < 3 ? (Q) : 0] = v.z;                                               \
    tab_shl96<S>(xa, t);                                                                   \
    for (int k = 0; k < 3; ++k) xa[k] = (xa[k] & ~ma[k]) | (t[k] & ma[k]);                  \
    tab_shl96<S>(xb, t);                                                                   \
    for (int k = 0; k < 3; ++k) xb[k] = (xb[k] & ~mb[k]) | (t[k] & mb[k]);                  \
  }
  LLVQ_EXPAND_STAGE(0, 64)
  LLVQ_EXPAND_STAGE(1, 32)
  LLVQ_EXPAND_STAGE(2, 16)
  LLVQ_EXPAND_STAGE(3, 8)
  LLVQ_EXPAND_STAGE(4, 4)
#undef LLVQ_EXPAND_STAGE
}

// Magnitudes by position (mag[w], byte i = position 4 w + i) from the two
// parts' states and ranks.  word_slot: the word's entry in the expand table
// (weight order); spread: whether the parts need moving at all (false for
// odd classes and words of weight 0 or 24, whose parts are in position
// order already: their lanes skip the mask loads).
template <bool SMEM>
LLVQ_HD void tab_magnitudes(const TabCtx& tc, uint32_t sa, uint64_t ra, uint32_t sb, uint64_t rb, int word_slot,
                            bool spread, int d0, uint64_t vals, uint32_t (&mag)[6]) {
  uint64_t a_lo = 0, a_hi = 0, b_lo = 0, b_hi = 0;
  int ta = 0, tb = 0;
  // searches: part A's, then part B's, one per iteration
  for (int it = 0; it < tc.max_searches; ++it) {
    uint4 r0 = make_uint4(0, 0, kTabTailBit, 0);
    bool in_b = false;
    if (sa != kTabEnd) r0 = tab_ldr<SMEM>(tc.srec + 2 * sa);
    if (r0.z & kTabTailBit) {
      in_b = true;
      r0 = make_uint4(0, 0, kTabTailBit, 0);
      if (sb != kTabEnd) r0 = tab_ldr<SMEM>(tc.srec + 2 * sb);
    }
    if (r0.z & kTabTailBit) continue;  // both parts are at their tails
    uint32_t s = in_b ? sb : sa;
    uint64_t r = in_b ? rb : ra, nib;
    int take;
    tab_search<SMEM>(tc, r0, s, r, nib, take);
    if (in_b) {
      tab_put(b_lo, b_hi, nib, tb);
      tb += take;
      sb = s;
      rb = r;
    } else {
      tab_put(a_lo, a_hi, nib, ta);
      ta += take;
      sa = s;
      ra = r;
    }
  }
  // tails: the rest of each part is one entry
  if (sa != kTabEnd) {
    const uint4 r0 = tab_ldr<SMEM>(tc.srec + 2 * sa);
    tab_put(a_lo, a_hi, tab_ldg(tc.tail + r0.x + ra), ta);
  }
  if (sb != kTabEnd) {
    const uint4 r0 = tab_ldr<SMEM>(tc.srec + 2 * sb);
    tab_put(b_lo, b_hi, tab_ldg(tc.tail + r0.x + rb), tb);
  }
  // part A value indices follow the d0 part-B values (no nibble overflows:
  // indices stay below 8, and the nibbles past the part's end are dropped by
  // the merge below)
  const uint64_t add = (uint64_t)d0 * 0x1111111111111111ull;
  a_lo += add;
  a_hi += add & 0xFFFFFFFFull;
  uint32_t xa[3] = {(uint32_t)a_lo, (uint32_t)(a_lo >> 32), (uint32_t)a_hi};
  uint32_t xb[3] = {(uint32_t)b_lo, (uint32_t)(b_lo >> 32), (uint32_t)b_hi};
  uint32_t m[3];
  if (spread) {
    tab_expand2(xa, xb, tc.expand + (size_t)word_slot * (kTabExpandWords / 4), m);
  } else {  // part A (odd, or the weight-24 word) everywhere, or part B (weight 0) everywhere
    const uint32_t all = word_slot ? 0xFFFFFFFFu : 0u;
    m[0] = m[1] = m[2] = all;
  }
  const uint32_t vlo = (uint32_t)vals, vhi = (uint32_t)(vals >> 32);
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const uint32_t x = (xa[k] & m[k]) | (xb[k] & ~m[k]);
    mag[2 * k] = tab_prmt(vlo, vhi, x & 0xFFFFu);
    mag[2 * k + 1] = tab_prmt(vlo, vhi, x >> 16);
  }
}

// Signs of a codeword from its magnitudes by position (mag[w], byte i =
// position 4 w + i) and y = the signed integer codeword; false (and y
// undefined) if the even sign rank is out of range for the magnitudes.
//   odd class:  y_d = m_d where m_d = 1 (mod 4) off the word or 3 (mod 4) on
//               it, else -m_d (solve_odd_subclass's signed leader with the
//               word's sign flips, impl/leech_lattice_vector_quantizer.py:649-681);
//   even class: the sign rank's bits on the nonzero coordinates in position
//               order, with the bit at the first word coordinate inserted so
//               that the negative word coordinates have the class's parity
//               (rank_even_signs / apply_even_signs, :804-841).
LLVQ_HD bool tab_signs(const uint32_t (&mag)[6], uint32_t word, bool odd, uint64_t sign, int parity_bit,
                       const uint8_t* deposit4, int (&y)[kDim]) {
  // per-position bits of the magnitudes, four bytes at a time (every
  // magnitude is below 128, so byte + 0x7F carries into bit 7 exactly when it
  // is nonzero; a multiply by 0x01020408 gathers bit 0 of the four bytes into
  // the top nibble)
  uint32_t nzmask = 0, b1mask = 0;
#pragma unroll
  for (int w = 0; w < 6; ++w) {
    const uint32_t t = mag[w];
    nzmask |= (((((t + 0x7F7F7F7Fu) >> 7) & 0x01010101u) * 0x01020408u) >> 24) << (4 * w);
    b1mask |= ((((t >> 1) & 0x01010101u) * 0x01020408u) >> 24) << (4 * w);
  }
  bool ok = true;
  uint32_t neg;
  if (odd) {
    neg = b1mask ^ word;
  } else {
    const int nz = tab_popc(nzmask);
    uint32_t cmask;
    if (word) {
      const int p = tab_popc(nzmask & ((word & (0u - word)) - 1u));
      const uint32_t rr = (uint32_t)sign;
      ok = (sign >> (nz - 1)) == 0;
      cmask = ((rr >> p) << (p + 1)) | (rr & ((1u << p) - 1u));
    } else {
      ok = nz >= 32 || (sign >> nz) == 0;
      cmask = (uint32_t)sign;
    }
    neg = 0;
#pragma unroll
    for (int k = 0; k < kDim / 4; ++k) {
      const uint32_t mm = (nzmask >> (4 * k)) & 15u;
      neg |= (uint32_t)deposit4[mm * 16 + (cmask & 15u)] << (4 * k);
      cmask >>= tab_popc(mm);
    }
    if (word && (tab_popc(neg & word) & 1) != parity_bit) neg ^= word & (0u - word);
  }
#pragma unroll
  for (int d = 0; d < kDim; ++d) {
    const int mv = (int)((mag[d >> 2] >> (8 * (d & 3))) & 0xFFu);
    y[d] = ((neg >> d) & 1u) ? -mv : mv;
  }
  return ok;
}

// a / b for b >= 1 given magic = floor((2^64 - 1) / b): the high half of
// a * magic is floor(a / b) or one less (division by an invariant integer by
// multiplication, Granlund and Montgomery 1994), fixed by one comparison.
LLVQ_HD uint64_t tab_divmod(uint64_t a, uint64_t b, uint64_t magic, uint64_t& rem) {
  uint64_t q = tab_mulhi(a, magic);
  uint64_t r = a - q * b;
  if (r >= b) {
    ++q;
    r -= b;
  }
  rem = r;
  return q;
}

// Class of a valid index: the bucket of its leading bit and next four bits
// narrows the search to the classes between the owners of the bucket's lowest
// index and of the next bucket's.
template <bool SMEM>
LLVQ_HD int tab_find_class(const TabCtx& tc, int64_t v) {
  const uint64_t u = (uint64_t)v;
  int key = 0;
  if (u) {
    const int e = tab_msb(u);
    key = 1 + e * 16 + (int)((e >= 4 ? u >> (e - 4) : u << (4 - e)) & 15u);
  }
  int lo = tab_ldr<SMEM>(tc.bucket + key), hi = tab_ldr<SMEM>(tc.bucket + key + 1) + 1;
  while (lo + 1 < hi) {
    const int mid = (lo + hi) >> 1;
    if (tc.starts[mid] <= v) lo = mid; else hi = mid;
  }
  return lo;
}

// Integer codeword of index v; false and zeros outside the codebook (or for
// a sign rank out of range, which no valid index has).
template <bool SMEM>
LLVQ_HD bool tab_decode(const TabCtx& tc, int64_t v, int (&y)[kDim]) {
  if (!(v >= 0 && v < tc.total)) {
    for (int d = 0; d < kDim; ++d) y[d] = 0;
    return false;
  }
  const int k = tab_find_class<SMEM>(tc, v);
  const uint4* cp = tc.crec + 4 * k;
  const uint4 c0 = tab_ldr<SMEM>(cp), c1 = tab_ldr<SMEM>(cp + 1), c2 = tab_ldr<SMEM>(cp + 2),
              c3 = tab_ldr<SMEM>(cp + 3);
  const uint64_t start = tab_u64(c0.x, c0.y), perm = tab_u64(c0.z, c0.w);
  const uint64_t magic_perm = tab_u64(c1.x, c1.y), magic_f1 = tab_u64(c1.z, c1.w);
  const uint64_t vals = tab_u64(c2.x, c2.y);
  const uint32_t f1p = c2.z, meta = c2.w;
  const bool odd = meta & 1u;
  const int weight = (int)((meta >> 1) & 31u), sshift = (int)((meta >> 6) & 31u), d0 = (int)((meta >> 11) & 15u);
  uint64_t prank;
  const uint64_t cur = tab_divmod((uint64_t)v - start, perm, magic_perm, prank);
  uint32_t word;
  int slot;
  uint64_t sign = 0, ra = prank, rb = 0;
  if (odd) {
    word = tab_ldr<SMEM>(tc.golay + (int)cur);
    slot = kNumGolay - 1;
  } else {
    sign = cur & ((1ull << sshift) - 1);
    slot = (int)c3.x + (int)(cur >> sshift);
    word = tab_ldr<SMEM>(tc.words + slot);
    uint64_t r1;
    rb = tab_divmod(prank, f1p, magic_f1, r1);
    ra = r1;
  }
  uint32_t mag[6];
  tab_magnitudes<SMEM>(tc, c3.y, ra, c3.z, rb, slot, !odd && weight != 0 && weight != kDim, d0, vals, mag);
  const bool ok = tab_signs(mag, word, odd, sign, (int)((meta >> 15) & 1u), tc.deposit4, y);
  if (!ok)
    for (int d = 0; d < kDim; ++d) y[d] = 0;
  return ok;
}

}  // namespace llvq
