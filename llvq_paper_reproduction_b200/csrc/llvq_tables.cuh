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
//   * a tail state (at most kTabTail = 12 positions left) lists all its
//     orderings in rank order, so the rest of the sequence is entry `rank`;
//   * a search state lists the orderings of its next h positions (h =
//     min(kTabHead, positions - kTabTail)) in rank order, each with the rank
//     of its first completion and the state it leaves.  A slot table over
//     g(rank) = umulhi(rank >> s, M) (a monotone 32-bit map onto about four
//     slots per entry) gives, per slot, the entry holding the slot's first
//     rank and the entry after it when one boundary falls inside the slot,
//     so a search is one 32-byte gather and one comparison; the few slots
//     with two or more boundaries inside are marked and scanned.
// Every class part has 0, 8, 12, 16 or 24 positions (Golay word weights), so
// its lookups are fixed by its size: a 24-position part is two searches of 6
// positions and a tail of 12, a 16-position part one search of 4 and a tail
// of 12, 12- and 8-position parts one tail.  That gives four decode shapes
// (kShape*), one per class; one code path covers them all, so lanes of a
// warp holding different shapes run the same lookups.  The 24-position parts
// (odd classes, word weight 0 or 24) store their sequences as nibble strings
// (value index j of the part in bits 4t..4t+3 for step t), already in
// position order.  The two parts of a weight-8/12/16 class (at most four
// values each) store theirs as two bit planes (bit t = bit 0 / bit 1 of the
// value index at step t); the planes are moved onto their positions (the
// word's coordinates and the others) by a bit deposit (the expand of H. S.
// Warren, Hacker's Delight, 2nd ed., section 7-5) with five move masks per
// Golay word and part, one 32-byte load, and then widened to nibbles.  A byte
// permute turns the nibbles into magnitudes, four positions at a time.
#pragma once

#include <cstdint>

#include "llvq_device.cuh"

namespace llvq {

constexpr int kTabTail = 12;              // positions a tail state covers
constexpr int kTabHead = 6;               // positions one search covers
constexpr uint32_t kTabEnd = 0xFFFFFFFFu; // no state: the part is empty / finished
constexpr uint32_t kTabTailBit = 1u << 31;
constexpr uint32_t kTabSlotMulti = 0xFFFFFFFEu;  // "next state" of a slot's second entry: scan the entries
constexpr int kTabSlotsPerEntry = 4;
constexpr int kTabMaxStateEntries = 0x10000;
constexpr int kTabClassRecords = 3;       // uint4 per class record
constexpr int kTabExpand2Words = 8;       // u32 per Golay word in the bit-plane deposit table

// Decode shapes (the lookups and the sign rule an index needs, from its class).
enum : int {
  kShapeOdd24 = 0,    // odd class: one 24-position part, odd signs
  kShapeEven24 = 1,   // even class of word weight 0 or 24: one 24-position part, even signs
  kShapeEven16 = 2,   // even, weight 8 or 16: a 16-position part and an 8-position part
  kShapeEven12 = 3,   // even, weight 12: two 12-position parts
  kShapeInvalid = 4,  // outside the codebook: a zero codeword
  kShapes = 5
};

// State record, two uint4:
//   [0] tail:   x = first entry in `tail`, z = kTabTailBit | positions
//       search: x = first slot, y = M, z = s | h << 8, w = first entry in `entry`
//   [1] N (u64, x | y << 32), z = number of entries (search)
// Search entry (uint4): {start low, start high, next state, nibbles of the h
// positions}; starts stay below 2^46.  Slot g (two uint4) covers the ranks r
// with umulhi(r >> s, M) = g: {E0, E1}, E0 the entry holding the slot's first
// rank, E1 the next entry if it starts inside the slot (else start = all
// ones), or, when two or more entries start inside the slot, {start of the
// next entry, kTabSlotMulti, its index, 0}.
//
// Class record, kTabClassRecords uint4 (48 bytes):
//   [0] start (48 bits) | meta << 48, permutation count (48 bits) | P1 << 48
//   [1] floor((2^64 - 1) / permutation count), values (u64: byte j = value
//       j; even: the |v| = 0 mod 4 part's values, then the |v| = 2 mod 4
//       part's from byte d0 on)
//   [2] (even classes with two parts only) floor((2^64 - 1) / f1 count),
//       f1 count, P2 | first word of the weight group (weight order) << 16 | d0 << 28
// meta: shape | sign shift << 2 | required << 7 | (word weight 24) << 8 | (P1 is part A) << 9.
// P1 is the part that is searched (odd: the only part; weight 0 or 24: the
// non-empty part; weight 8 or 16: the 16-position part; weight 12: part A),
// P2 the other part of a weight-8, 12 or 16 class.  Part A is the odd
// class's only part or the even class's |v| = 2 (mod 4) part on the word's
// positions; part B the even class's |v| = 0 (mod 4) part on the other
// positions.
//
// Words are indexed in weight order (lexicographic inside a weight): an even
// class's word is entry wbase + choice.

#if defined(__CUDA_ARCH__)
template <class T>
__device__ __forceinline__ T tab_ldg(const T* p) { return __ldg(p); }
__device__ __forceinline__ uint32_t tab_prmt(uint32_t a, uint32_t b, uint32_t s) { return __byte_perm(a, b, s); }
__device__ __forceinline__ uint32_t tab_fshl(uint32_t lo, uint32_t hi, int s) { return __funnelshift_l(lo, hi, s); }
__device__ __forceinline__ uint32_t tab_umulhi(uint32_t a, uint32_t b) { return __umulhi(a, b); }
__device__ __forceinline__ uint64_t tab_mulhi(uint64_t a, uint64_t b) { return __umul64hi(a, b); }
__device__ __forceinline__ int tab_popc(uint32_t v) { return __popc(v); }
__device__ __forceinline__ int tab_msb(uint64_t u) { return 63 - __clzll((long long)u); }
// One 32-byte read-only load (p 32-byte aligned): one gather instead of two.
__device__ __forceinline__ void tab_ldg256(const uint4* p, uint4& a, uint4& b) {
  asm("ld.global.nc.v8.u32 {%0, %1, %2, %3, %4, %5, %6, %7}, [%8];"
      : "=r"(a.x), "=r"(a.y), "=r"(a.z), "=r"(a.w), "=r"(b.x), "=r"(b.y), "=r"(b.z), "=r"(b.w)
      : "l"(p));
}
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
inline uint32_t tab_umulhi(uint32_t a, uint32_t b) { return (uint32_t)(((uint64_t)a * b) >> 32); }
inline uint64_t tab_mulhi(uint64_t a, uint64_t b) { return (uint64_t)(((unsigned __int128)a * b) >> 64); }
inline int tab_popc(uint32_t v) { return __builtin_popcount(v); }
inline int tab_msb(uint64_t u) { return 63 - __builtin_clzll(u); }
inline void tab_ldg256(const uint4* p, uint4& a, uint4& b) {
  a = p[0];
  b = p[1];
}
#endif

LLVQ_HD uint64_t tab_u64(uint32_t lo, uint32_t hi) { return ((uint64_t)hi << 32) | lo; }

// Where the decoder reads its tables.  The small ones marked SMEM point to
// shared-memory copies (plain loads) or to global memory (read-only cache
// loads); starts and deposit4 are read with plain loads (shared memory in
// the kernels); the rest is global memory.
struct TabCtx {
  const uint4* srec;          // 2 per state                          (SMEM)
  const uint4* crec;          // kTabClassRecords per class           (SMEM)
  // (the shared copies of srec and crec are stored field-major, record j of
  // state / class k at j * count + k, so that a warp's random records spread
  // over all banks; the global ones record-major, at 2k + j / 3k + j)
  const uint16_t* bucket;     // index bucket -> class                (global / host)
  const uint32_t* bucket2;    // bucket b -> class of b | class of b + 1 << 16 (shared copy)
  const uint32_t* words;      // Golay words in weight order          (SMEM)
  const uint32_t* golay;      // Golay words in lexicographic order   (SMEM)
  const int64_t* starts;      // class starts (binary search)         (plain loads)
  const uint8_t* deposit4;    // [m * 16 + s]: the low popc(m) bits of s placed on the set bits of m (plain)
  const uint4* entry;
  const uint4* slot;          // 2 per slot
  const unsigned long long* tail;  // nibble-string tails (odd and weight-0/24 parts)
  const uint32_t* tail2;          // bit-plane tails (parts of weight-8/12/16 classes)
  const uint4* expand2;       // kTabExpand2Words u32 per word, weight order
  int n_classes;
  int n_states;
  int max_searches;           // searches of the longest class (both parts)
  int64_t total;
};

template <bool SMEM, class T>
LLVQ_HD T tab_ldr(const T* p) {
  if constexpr (SMEM) return *p;
  else return tab_ldg(p);
}

// Record j of class k / state s.
template <bool SMEM>
LLVQ_HD uint4 tab_crec(const TabCtx& tc, int k, int j) {
  return tab_ldr<SMEM>(tc.crec + (SMEM ? j * tc.n_classes + k : kTabClassRecords * k + j));
}
template <bool SMEM>
LLVQ_HD uint4 tab_srec(const TabCtx& tc, uint32_t s, int j) {
  return tab_ldr<SMEM>(tc.srec + (SMEM ? (size_t)j * tc.n_states + s : 2 * (size_t)s + j));
}

// One search from search state s (record r0) with rank r: the nibbles of the
// positions it covers; s becomes the state left, r the rank within it.
template <bool SMEM>
LLVQ_HD uint32_t tab_search(const TabCtx& tc, const uint4& r0, uint32_t& s, uint64_t& r) {
  const uint32_t g = tab_umulhi((uint32_t)(r >> (r0.z & 63u)), r0.y);
  uint4 e0, e1;
  tab_ldg256(tc.slot + 2 * ((size_t)r0.x + g), e0, e1);
  const uint64_t b = tab_u64(e1.x, e1.y);
  const bool up = r >= b;
  uint64_t start = up ? b : tab_u64(e0.x, e0.y);
  uint32_t next = up ? e1.z : e0.z, nib = up ? e1.w : e0.w;
  if (next == kTabSlotMulti) {  // several entries start inside the slot: scan from the second
    const uint4* ent = tc.entry + r0.w;
    const uint32_t n = tab_srec<SMEM>(tc, s, 1).z;
    uint32_t j = nib;
    while (j + 1 < n) {
      const uint2 nx = tab_ldg(reinterpret_cast<const uint2*>(ent + j + 1));
      if (tab_u64(nx.x, nx.y) > r) break;
      ++j;
    }
    const uint4 e = tab_ldg(ent + j);
    start = tab_u64(e.x, e.y);
    next = e.z;
    nib = e.w;
  }
  r -= start;
  s = next;
  return nib;
}

// Bit t (t < 8) of b to bit 4t: three shift-and-mask stages.
LLVQ_HD uint32_t tab_spread8(uint32_t b) {
  uint32_t x = (b & 0xFFu) | ((b & 0xFFu) << 12);
  x &= 0x000F000Fu;
  x = (x | (x << 6)) & 0x03030303u;
  return (x | (x << 3)) & 0x11111111u;
}

// Bit-plane deposit (the expand of Hacker's Delight, section 7-5, with the
// move masks of one Golay word): bit t of a goes to the t-th set bit of the
// word, bit t of b to the t-th clear bit, for both planes of each part; the
// merged planes and the word give each position's byte-permute selector
// (value index bits 0-1, bit 2 = on the word).  e: the word's kTabExpand2Words
// masks (stage i of the word's deposit in m[i] bits 0-23, the complement's
// stage i split over m[i] bits 24-31 and m[5..7]).
LLVQ_HD void tab_deposit_planes(uint32_t a0, uint32_t a1, uint32_t b0, uint32_t b1, uint32_t word, const uint4* e,
                                uint32_t (&x)[3]) {
  uint4 u, v;
  tab_ldg256(e, u, v);
  const uint32_t ma[5] = {u.x, u.y, u.z, u.w, v.x};
  const uint32_t mb[5] = {tab_prmt(u.x, v.y, 0x3543u), tab_prmt(u.y, v.y, 0x3763u), tab_prmt(u.z, v.z, 0x3543u),
                          tab_prmt(u.w, v.z, 0x3763u), tab_prmt(v.x, v.w, 0x3543u)};
#pragma unroll
  for (int i = 4; i >= 0; --i) {
    const int sh = 1 << i;
    a0 = (a0 & ~ma[i]) | ((a0 << sh) & ma[i]);
    a1 = (a1 & ~ma[i]) | ((a1 << sh) & ma[i]);
    b0 = (b0 & ~mb[i]) | ((b0 << sh) & mb[i]);
    b1 = (b1 & ~mb[i]) | ((b1 << sh) & mb[i]);
  }
  const uint32_t p0 = (a0 & word) | (b0 & ~word), p1 = (a1 & word) | (b1 & ~word);
#pragma unroll
  for (int g = 0; g < 3; ++g)
    x[g] = tab_spread8(p0 >> (8 * g)) + 2u * tab_spread8(p1 >> (8 * g)) + 4u * tab_spread8(word >> (8 * g));
}

// Per-position bit masks of magnitudes (mag[w], byte i = position 4w + i;
// every magnitude is below 128): nonzero (byte + 0x7F carries into bit 7
// exactly when the byte is nonzero) and bit 1, both gathered by one multiply
// (0x01020408 moves bit 0 of four bytes into the top nibble; nonzero in bit
// 0 and bit 1 in bit 4 of each byte give nonzero bits 24-27 and bit-1 bits
// 28-31).
LLVQ_HD void tab_magnitude_masks(const uint32_t (&mag)[6], uint32_t& nz, uint32_t& b1) {
  nz = 0;
  b1 = 0;
#pragma unroll
  for (int w = 0; w < 6; ++w) {
    const uint32_t t = mag[w];
    const uint32_t f = ((((t + 0x7F7F7F7Fu) >> 7) & 0x01010101u) | ((t << 3) & 0x10101010u)) * 0x01020408u;
    nz |= ((f >> 24) & 15u) << (4 * w);
    b1 |= (f >> 28) << (4 * w);
  }
}

// Negative coordinates of an even codeword from its nonzero mask and sign
// rank: the rank's bits go to the nonzero coordinates in position order,
// with the bit at the first word coordinate inserted so that the negative
// word coordinates have the class's parity (rank_even_signs /
// apply_even_signs, impl/leech_lattice_vector_quantizer.py:804-841).  False
// when the rank is out of range for the magnitudes (no valid index).
LLVQ_HD bool tab_even_neg(uint32_t nzmask, uint32_t word, uint64_t sign, int parity_bit, const uint8_t* deposit4,
                          uint32_t& neg) {
  const int nz = tab_popc(nzmask);
  bool ok;
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
  uint32_t n = 0;
#pragma unroll
  for (int k = 0; k < kDim / 4; ++k) {
    const uint32_t mm = (nzmask >> (4 * k)) & 15u;
    n |= (uint32_t)deposit4[mm * 16 + (cmask & 15u)] << (4 * k);
    cmask >>= tab_popc(mm);
  }
  if (word && (tab_popc(n & word) & 1) != parity_bit) n ^= word & (0u - word);
  neg = n;
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
  int lo, hi;
  if constexpr (SMEM) {
    const uint32_t bb = tc.bucket2[key];
    lo = (int)(bb & 0xFFFFu);
    hi = (int)(bb >> 16) + 1;
  } else {
    lo = tab_ldg(tc.bucket + key);
    hi = tab_ldg(tc.bucket + key + 1) + 1;
  }
  while (lo + 1 < hi) {
    const int mid = (lo + hi) >> 1;
    if ((uint64_t)tc.starts[mid] <= (uint64_t)v) lo = mid; else hi = mid;
  }
  return lo;
}

// Class and decode shape of an index (kShapeInvalid outside the codebook).
template <bool SMEM>
LLVQ_HD int tab_classify(const TabCtx& tc, int64_t v, int& k) {
  if (!((uint64_t)v < (uint64_t)tc.total)) {
    k = 0;
    return kShapeInvalid;
  }
  k = tab_find_class<SMEM>(tc, v);
  return (int)((tab_crec<SMEM>(tc, k, 0).y >> 16) & 3u);
}

// Magnitudes by position (mag[w], byte i = position 4w + i) and the mask of
// negative coordinates of the valid index v of class k, on one path for every
// decode shape (so the lanes of a warp that hold different shapes diverge
// only around the even-class expand and sign deposit):
//   part P1 (odd and weight 0/24: the 24-position part, two searches;
//   weight 8/16: the 16-position part, one search; weight 12: part A, none)
//   runs its searches and its tail; part P2 (weight 8/16: the 8-position
//   part; weight 12: part B) is one tail.  False for a sign rank out of range
//   (no valid index has one).
template <bool SMEM>
LLVQ_HD bool tab_decode_mn(const TabCtx& tc, int64_t v, int k, uint32_t (&mag)[6], uint32_t& neg) {
  const uint4 c0 = tab_crec<SMEM>(tc, k, 0), c1 = tab_crec<SMEM>(tc, k, 1);
  const uint32_t meta = c0.y >> 16;
  const int shape = (int)(meta & 3u), sshift = (int)((meta >> 2) & 31u);
  uint64_t prank;
  const uint64_t cur = tab_divmod((uint64_t)v - tab_u64(c0.x, c0.y & 0xFFFFu), tab_u64(c0.z, c0.w & 0xFFFFu),
                                  tab_u64(c1.x, c1.y), prank);
  const bool split = shape >= kShapeEven16;
  // primary part P1 and its searches, secondary tail part P2
  uint32_t s1 = c0.w >> 16, s2 = kTabEnd, c2w = 0;
  uint64_t r1 = prank, r2 = 0;
  if (split) {
    const uint4 c2 = tab_crec<SMEM>(tc, k, 2);
    uint64_t ra;
    const uint64_t rb = tab_divmod(prank, c2.z, tab_u64(c2.x, c2.y), ra);
    const bool p1a = (meta >> 9) & 1u;
    r1 = p1a ? ra : rb;
    r2 = p1a ? rb : ra;
    s2 = c2.w & 0xFFFFu;
    c2w = c2.w;
  }
  const int nsearch = shape <= kShapeEven24 ? 2 : shape == kShapeEven16 ? 1 : 0;
  uint32_t t2 = 0;
  if (split) t2 = tab_ldg(tc.tail2 + tab_srec<SMEM>(tc, s2, 0).x + r2);  // independent of P1
  uint32_t nib[2] = {0, 0};
#pragma unroll
  for (int it = 0; it < 2; ++it)
    if (it < nsearch) nib[it] = tab_search<SMEM>(tc, tab_srec<SMEM>(tc, s1, 0), s1, r1);
  const uint32_t tbase = tab_srec<SMEM>(tc, s1, 0).x;
  uint32_t x[3], word;
  if (!split) {
    // one 24-position part: two searches of 6 positions, a tail of 12
    const uint64_t t = tab_ldg(tc.tail + tbase + r1);
    x[0] = nib[0] | (nib[1] << 24);
    x[1] = (nib[1] >> 8) | ((uint32_t)t << 16);
    x[2] = (uint32_t)(t >> 16);
    word = shape == kShapeOdd24 ? tab_ldr<SMEM>(tc.golay + (int)cur) : (((meta >> 8) & 1u) ? kFull24 : 0u);
  } else {
    // two parts as bit planes: P1 (a search of 4 positions and a tail of 12,
    // or a tail of 12) and P2 (a tail of 8 or 12)
    const uint32_t t1 = tab_ldg(tc.tail2 + tbase + r1);
    uint32_t q0 = t1 & 0xFFFu, q1 = t1 >> 12;
    if (shape == kShapeEven16) {
      q0 = (nib[0] & 0xFu) | (q0 << 4);
      q1 = ((nib[0] >> 8) & 0xFu) | (q1 << 4);
    }
    const uint32_t u0 = t2 & 0xFFFu, u1 = t2 >> 12;
    const bool p1a = (meta >> 9) & 1u;
    const int slot = (int)((c2w >> 16) & 0xFFFu) + (int)(cur >> sshift);
    word = tab_ldr<SMEM>(tc.words + slot);
    tab_deposit_planes(p1a ? q0 : u0, p1a ? q1 : u1, p1a ? u0 : q0, p1a ? u1 : q1, word,
                       tc.expand2 + (size_t)slot * (kTabExpand2Words / 4), x);
  }
  const uint32_t vlo = c1.z, vhi = c1.w;
#pragma unroll
  for (int q = 0; q < 3; ++q) {
    mag[2 * q] = tab_prmt(vlo, vhi, x[q] & 0xFFFFu);
    mag[2 * q + 1] = tab_prmt(vlo, vhi, x[q] >> 16);
  }
  uint32_t nzmask, b1mask;
  tab_magnitude_masks(mag, nzmask, b1mask);
  if (shape == kShapeOdd24) {
    // y = m where m = 1 mod 4 off the word or m = 3 mod 4 on it, else -m
    // (solve_odd_subclass's signed leader with the word's sign flips,
    // impl/leech_lattice_vector_quantizer.py:649-681)
    neg = b1mask ^ word;
    return true;
  }
  return tab_even_neg(nzmask, word, cur & ((1ull << sshift) - 1), (int)((meta >> 7) & 1u), tc.deposit4, neg);
}

// Integer codeword of index v; false and zeros outside the codebook (or for
// a sign rank out of range, which no valid index has).
template <bool SMEM>
LLVQ_HD bool tab_decode(const TabCtx& tc, int64_t v, int (&y)[kDim]) {
  int k;
  const int shape = tab_classify<SMEM>(tc, v, k);
  uint32_t mag[6], neg = 0;
  bool ok = shape != kShapeInvalid;
  if (ok) ok = tab_decode_mn<SMEM>(tc, v, k, mag, neg);
#pragma unroll
  for (int d = 0; d < kDim; ++d) {
    const int mv = ok ? (int)((mag[d >> 2] >> (8 * (d & 3))) & 0xFFu) : 0;
    y[d] = ((neg >> d) & 1u) ? -mv : mv;
  }
  return ok;
}

}  // namespace llvq
