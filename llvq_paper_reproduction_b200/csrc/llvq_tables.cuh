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
//     and the state it leaves; a guide table over rank / N, N the number of
//     orderings of the state, finds the entry holding `rank` in one or two
//     probes.
// A 24-position part is two searches and one tail; a 16-position part one
// search and one tail; 12- and 8-position parts one tail.  Sequences are
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

// State record (uint4):
//   tail:   x = first entry in `tail`, w = kTabTailBit | positions
//   search: x = first entry in `entry`, y = first guide slot, z = fp32 bits of
//           G / N (G guide slots, a power of two), w = entries | log2 G << 17
//           | h << 22
// Search entry (uint4): {start low, start high, next state, nibbles of the h
// positions}.  Guide slot g: the entry holding rank ceil(g N / G).
constexpr uint32_t kTabTailBit = 1u << 31;

// Part A is the odd class's only part or the even class's |v| = 2 (mod 4)
// part on the word's positions; part B the even class's |v| = 0 (mod 4) part
// on the other positions.

#if defined(__CUDA_ARCH__)
template <class T>
__device__ __forceinline__ T tab_ld(const T* p) { return __ldg(p); }
__device__ __forceinline__ uint32_t tab_prmt(uint32_t a, uint32_t b, uint32_t s) { return __byte_perm(a, b, s); }
__device__ __forceinline__ uint32_t tab_fshl(uint32_t lo, uint32_t hi, int s) { return __funnelshift_l(lo, hi, s); }
__device__ __forceinline__ uint32_t tab_f2u(float f) { return __float2uint_rz(f); }
__device__ __forceinline__ float tab_u2f(uint64_t v) { return __ull2float_rn(v); }
__device__ __forceinline__ float tab_bits2f(uint32_t b) { return __uint_as_float(b); }
#else
template <class T>
inline T tab_ld(const T* p) { return *p; }
inline uint32_t tab_prmt(uint32_t a, uint32_t b, uint32_t s) {
  const uint64_t v = ((uint64_t)b << 32) | a;
  uint32_t out = 0;
  for (int i = 0; i < 4; ++i) out |= (uint32_t)((v >> (8 * ((s >> (4 * i)) & 7))) & 0xFF) << (8 * i);
  return out;
}
inline uint32_t tab_fshl(uint32_t lo, uint32_t hi, int s) {
  return s ? (hi << s) | (lo >> (32 - s)) : hi;
}
inline uint32_t tab_f2u(float f) { return (uint32_t)f; }
inline float tab_u2f(uint64_t v) { return (float)v; }
inline float tab_bits2f(uint32_t b) {
  float f;
  __builtin_memcpy(&f, &b, 4);
  return f;
}
#endif

// One lookup: from state s with rank r, the nibbles of the positions it
// covers (`take` of them); s becomes the next state (kTabEnd after a tail).
LLVQ_HD void tab_job(const TabView& tv, uint32_t& s, uint64_t& r, uint64_t& nib, int& take) {
  const uint4 rec = tab_ld(tv.state + s);
  if (rec.w & kTabTailBit) {
    nib = tab_ld(tv.tail + rec.x + r);
    take = (int)(rec.w & 31u);
    s = kTabEnd;
    return;
  }
  const uint32_t n = rec.w & 0x1FFFFu, lg = (rec.w >> 17) & 31u;
  uint32_t g = tab_f2u(tab_u2f(r) * tab_bits2f(rec.z));
  const uint32_t gmax = (1u << lg) - 1u;
  g = g < gmax ? g : gmax;
  const uint4* ent = tv.entry + rec.x;
  uint32_t j = tab_ld(tv.guide + rec.y + g);
  uint4 e = tab_ld(ent + j);
  uint64_t st = ((uint64_t)e.y << 32) | e.x;
  // the fp32 slot can be one too high: step back (entry 0 starts at 0)
  while (st > r && j > 0) {
    --j;
    e = tab_ld(ent + j);
    st = ((uint64_t)e.y << 32) | e.x;
  }
  while (j + 1 < n) {
    const uint2 nx = tab_ld(reinterpret_cast<const uint2*>(ent + j + 1));
    const uint64_t ns = ((uint64_t)nx.y << 32) | nx.x;
    if (ns > r) break;
    ++j;
    e = tab_ld(ent + j);
    st = ns;
  }
  r -= st;
  s = e.z;
  nib = e.w;
  take = (int)((rec.w >> 22) & 15u);
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

// Expand table layout, per Golay word (lexicographic index), kTabExpandWords
// u32 as five 32-byte stages q = 0..4 (applied in that order; stage q moves
// nibbles by 2^(4-q) positions): {A0, A1, A2, B0}, {B1, B2, M_q, 0}, where
// A0..A2 / B0..B2 are the nibble-wide move masks of the expand by the word /
// by its complement (three u32 covering positions 0-7, 8-15, 16-23) and
// M_0..M_2 the word itself widened to nibbles.
//
// Nibble-wise expand of both parts at once: source nibble t of xa goes to
// the t-th position of the word, source nibble t of xb to the t-th position
// outside it; m receives the word's nibble mask.  Positions outside each
// part's mask hold garbage.
LLVQ_HD void tab_expand2(uint32_t (&xa)[3], uint32_t (&xb)[3], const uint4* e, uint32_t (&m)[3]) {
  uint32_t t[3];
#define LLVQ_EXPAND_STAGE(Q, S)                                                           \
  {                                                                                        \
    const uint4 u = tab_ld(e + 2 * (Q)), v = tab_ld(e + 2 * (Q) + 1);                       \
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

// Magnitudes by position (mag[w], byte i = position 4 w + i) of a valid
// class-local decomposition: part A rank ra from state sa, part B rank rb
// from state sb, word = lexicographic index of the Golay word whose positions
// part A takes (4095, all positions, for odd classes), d0 = number of part-B
// values (their value indices come first in `vals`), vals = the part-B values
// then the part-A values, one per byte.
LLVQ_HD void tab_magnitudes(const TabView& tv, uint32_t sa, uint64_t ra, uint32_t sb, uint64_t rb, int word_lex,
                            int d0, uint64_t vals, uint32_t (&mag)[6]) {
  uint64_t a_lo = 0, a_hi = 0, b_lo = 0, b_hi = 0;
  bool in_b = sa == kTabEnd;
  uint32_t s = in_b ? sb : sa;
  uint64_t r = in_b ? rb : ra;
  int t = 0;
  for (int job = 0; job < tv.max_jobs; ++job) {
    if (s == kTabEnd) break;
    uint64_t nib;
    int take;
    tab_job(tv, s, r, nib, take);
    if (in_b) tab_put(b_lo, b_hi, nib, t);
    else tab_put(a_lo, a_hi, nib, t);
    t += take;
    if (s == kTabEnd && !in_b) {
      in_b = true;
      s = sb;
      r = rb;
      t = 0;
    }
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
  tab_expand2(xa, xb, tv.expand + (size_t)word_lex * (kTabExpandWords / 4), m);
  const uint32_t vlo = (uint32_t)vals, vhi = (uint32_t)(vals >> 32);
#pragma unroll
  for (int k = 0; k < 3; ++k) {
    const uint32_t x = (xa[k] & m[k]) | (xb[k] & ~m[k]);
    mag[2 * k] = tab_prmt(vlo, vhi, x & 0xFFFFu);
    mag[2 * k + 1] = tab_prmt(vlo, vhi, x >> 16);
  }
}

}  // namespace llvq

namespace llvq {

#if defined(__CUDA_ARCH__)
__device__ __forceinline__ int tab_popc(uint32_t v) { return __popc(v); }
#else
inline int tab_popc(uint32_t v) { return __builtin_popcount(v); }
#endif

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
// deposit4[m * 16 + s]: the low popc(m) bits of s placed on the set bits of m.
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
      const uint32_t m = (nzmask >> (4 * k)) & 15u;
      neg |= (uint32_t)deposit4[m * 16 + (cmask & 15u)] << (4 * k);
      cmask >>= tab_popc(m);
    }
    if (word && (tab_popc(neg & word) & 1) != parity_bit) neg ^= word & (0u - word);
  }
#pragma unroll
  for (int d = 0; d < kDim; ++d) {
    const int m = (int)((mag[d >> 2] >> (8 * (d & 3))) & 0xFFu);
    y[d] = ((neg >> d) & 1u) ? -m : m;
  }
  return ok;
}

}  // namespace llvq
