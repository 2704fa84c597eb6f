// Λ24 nearest-point quantizer for sm_100a: exact, reference-order argmax over
// (Golay word, shell, class) as in LeechLatticeVectorQuantizer.quantize
// (impl/leech_lattice_vector_quantizer.py:282-314), fused with the index
// encoding (encode_codeword, :247-280).
//
// One CTA per 24-D block at a time (persistent grid), 256 threads x 8
// complementary Golay word pairs (c, ~c) each (512 x 4 for the largest
// codebooks).  Per block it stages |x| in
// sorted order, the 3 byte tables that permute a Golay word into that order,
// and the integer image q = rint(|x| * 2^e) with |q| <= 2^19.  Per pair it
// builds the suffix sums of the sorted (sign-flipped) coordinates in
// registers once (the complement's follow from them) and scores every class
// of both words with the generated FFMA chains (one FFMA per distinct leader
// value).  All suffix sums are exact integers in fp32; only the FFMA chain
// rounds, so every approximate score is within a proven bound E of the exact
// real score.
//
// The argmax is then decided exactly.  If a single word holds every pair
// within W = 2E + 4 (q units) of the best approximate score, the search kernel
// hands that word to the finalize kernel (one thread per block), which
// re-scores the word's pairs inside the window with the reference's own fp64
// arithmetic (CPython 3.12 sum(), a Neumaier-compensated sum).  Otherwise the
// whole CTA re-scans all words that way.  Ties go to the earliest (Golay word,
// class) in the reference loop order.  The winning codeword is rebuilt with
// the reference's sort/tie rules (solve_even_subclass / solve_odd_subclass,
// :619-666) and ranked (rank_class_codeword and friends, :692-889).
// best_pair / best_score carry the hand-over between the two kernels.
#include <cuda_runtime.h>

#include <algorithm>
#include <atomic>
#include <cfloat>
#include <climits>
#include <cmath>
#include <cstdint>

#include "llvq_device.cuh"
#include "llvq_internal.h"

__device__ __forceinline__ float llvq_max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

#include "_gen/search_gen.cuh"

namespace llvq {

// CTA shape of the search, per codebook (the generated Spec's kCtaThreads /
// kCtaMinBlocks / kCtaRealign, chosen by the size of its scoring code;
// table-driven codebooks use 256 threads, 3 CTAs): small codes (shells 2..11,
// 13 alone) run 6 CTAs of 128 threads (16 pairs each, <= 85 registers); the
// shells 2..13 and shell 23 codes 3 CTAs of 256 threads (8 pairs each); the
// shell 32 code one CTA of 512 (4 pairs each).  The search is issue-bound and
// the resident warps outweigh a few spilled bytes.  In the larger shapes the
// warps realign at every pair (a barrier per four warps in 256-thread CTAs,
// one for the whole 512-thread CTA), so they run the same stretch of the
// generated scoring code and share the instruction cache: 128 threads
// without the barrier ran 3.6% slower on shells 2..13, 26% slower on shell 23
// and 37% slower on shell 32; on shell 32, 512 threads gain another 44% over
// 256.  On the small codes the barrier costs about 2%.
constexpr int kMaxSearchThreads = 512;
constexpr int kSearchThreads = 256;
constexpr int kSearchMinBlocks = 3;
constexpr long long kTagWord = 1ll << 40;   // low 12 bits: the word
constexpr long long kTagExact = 2ll << 40;  // bits 12..39: class, low 12 bits: word

struct RowShared {
  float x[kDim];
  float aval[kDim];     // |q| in ascending (|x|, position) order
  float lval[48];       // 24 + r -> +aval[r], 23 - r -> -aval[r]
  uint32_t utab[3][256];
  int8_t apos[kDim];    // position at each sorted rank
  int8_t arank[kDim];
  uint32_t negmask;     // x_d < 0
  uint32_t nposA;       // sorted-rank image of ~negmask
  int invalid;
  float scale;          // 2^e
  float K;              // sqrt(8) * 2^e in fp32
  float red[kMaxSearchThreads / 32];
  double xs_best[kMaxSearchThreads];
  long long xs_order[kMaxSearchThreads];
};

// The same block data for one thread (finalize kernel), without the byte tables.
struct RowLocal {
  float x[kDim];
  float aval[kDim];
  float lval[48];
  int8_t apos[kDim];
  int8_t arank[kDim];
  uint32_t negmask;
  uint32_t nposA;
  float scale;
  float K;
};

// ------------------------------------------------------------ row helpers

// Scale exponent: |q| = |rint(x * 2^e)| <= 2^19.  Clamped so sqrt(8)*2^e*shell
// stays finite in fp32; a clamped (tiny) row only loses precision, which the
// exact window pass absorbs.
__device__ __forceinline__ int row_exponent(float maxabs) {
  if (!(maxabs > 0.f)) return 0;
  int E;
  (void)frexpf(maxabs, &E);  // maxabs < 2^E
  int e = kQBits - E;
  if (e > 100) e = 100;
  if (e < -120) e = -120;
  return e;
}

__device__ __forceinline__ float pow2f(int e) { return __int_as_float((e + 127) << 23); }

// Proven bound (q units) on |approximate score - exact real score| for any
// pair, for FFMA chains with window constants (l1max, mg, am): half a unit per
// unit of leader L1 norm from rounding x to q, plus one fp32 rounding per FFMA
// of a partial sum bounded by m*K + sum |coef| * (suffix length) * 2^Q.
__device__ __forceinline__ double window_error(double K, float l1max, float mg, float am) {
  const double u = 1.0 / 16777216.0;  // 2^-24
  return 0.5 * l1max + u * K * mg + u * (double)(1 << kQBits) * am * (1.0 + 1e-6);
}

__device__ __forceinline__ double window_width(float K, const DevBook& b) {
  return 2.0 * window_error((double)K, b.l1max, b.win_mg, b.win_am) + 4.0;
}

// CPython 3.12 sum() of the float products x_d * y_d (Neumaier-compensated),
// then LATTICE_SCALE * proj - shell, every operation separately rounded.
__device__ double reference_projection(const float* x, const int* y) {
  double f = __dadd_rn(0.0, __dmul_rn((double)x[0], (double)y[0]));
  double c = 0.0;
#pragma unroll
  for (int d = 1; d < kDim; ++d) {
    const double xi = __dmul_rn((double)x[d], (double)y[d]);
    const double t = __dadd_rn(f, xi);
    if (fabs(f) >= fabs(xi)) c = __dadd_rn(c, __dadd_rn(__dsub_rn(f, t), xi));
    else c = __dadd_rn(c, __dadd_rn(__dsub_rn(xi, t), f));
    f = t;
  }
  if (c != 0.0 && isfinite(c)) f = __dadd_rn(f, c);
  return f;
}

__device__ double reference_score(const float* x, const int* y, int shell) {
  return __dsub_rn(__dmul_rn(kLatticeScaleD, reference_projection(x, y)), (double)shell);
}

// The exact score a search maximises: the reference's (ANG false), or the
// correlation per unit norm of the multi-shell shape search, proj / |y| =
// proj / sqrt(16 shell) (ANG true; the angular specs of gen_search.py).
template <bool ANG>
__device__ __forceinline__ double exact_score(const float* x, const int* y, int shell) {
  if constexpr (ANG) return __ddiv_rn(reference_projection(x, y), __dsqrt_rn(16.0 * (double)shell));
  else return reference_score(x, y, shell);
}

// The reference's best codeword of class c for Golay word `word`
// (solve_even_subclass / solve_odd_subclass).  apos: positions in ascending
// (|x|, position) order.
__device__ void build_candidate(const float* x, const int8_t* apos, const DevClass& c, uint32_t word, int* y) {
  if (c.parity == 0) {
    int t0 = 0, t1 = 0, first1 = -1;
    for (int r = 0; r < kDim; ++r) {
      const int p = apos[r];
      int m;
      if ((word >> p) & 1u) {
        m = c.asc1[t1++];
        if (first1 < 0) first1 = p;
      } else {
        m = c.asc0[t0++];
      }
      y[p] = x[p] >= 0.f ? m : -m;
    }
    if (c.even_weight > 0) {
      int neg = 0;
      for (int d = 0; d < kDim; ++d) neg += ((word >> d) & 1u) && y[d] < 0;
      if ((neg & 1) != c.required) y[first1] = -y[first1];
    }
  } else {
    float xp[kDim];
    int ord[kDim];
    for (int d = 0; d < kDim; ++d) {
      xp[d] = ((word >> d) & 1u) ? -x[d] : x[d];
      ord[d] = d;
    }
    for (int i = 1; i < kDim; ++i) {  // sort by (x', position), stable
      const int p = ord[i];
      int j = i - 1;
      while (j >= 0 && xp[ord[j]] > xp[p]) {
        ord[j + 1] = ord[j];
        --j;
      }
      ord[j + 1] = p;
    }
    for (int r = 0; r < kDim; ++r) {
      const int p = ord[r];
      const int v = c.asc0[r];
      y[p] = ((word >> p) & 1u) ? -v : v;
    }
  }
}

// ------------------------------------------------------- scoring adapters

// Generated specialisations: everything is a compile-time constant.
template <class S>
struct Ops {
  static constexpr int kThreads = S::kCtaThreads;
  static constexpr int kMinBlocks = S::kCtaMinBlocks;
  static constexpr bool kRealign = S::kCtaRealign;
  static constexpr int kNumShells = S::kNumShells;
  static constexpr int kMinShellC = S::kMinShell;
  static constexpr bool kHasOdd = S::kHasOdd;
  static constexpr bool kAngular = S::kAngular;
  template <int W>
  static constexpr bool has_even() {
    return W == 0 ? S::kHasEven_w0 : W == 8 ? S::kHasEven_w8 : W == 12 ? S::kHasEven_w12
                                                                        : W == 16 ? S::kHasEven_w16 : S::kHasEven_w24;
  }
  template <int W>
  static constexpr int r0max() {
    return W == 0 ? S::kR0Max_w0 : W == 8 ? S::kR0Max_w8 : W == 12 ? S::kR0Max_w12
                                                                   : W == 16 ? S::kR0Max_w16 : S::kR0Max_w24;
  }
  static constexpr bool kPacked = true;  // odd_max2 / even_max2_w12 score c and ~c in one pass
  __device__ static float odd_max(const DevBook&, const float (&R)[25], const float* nmk) { return S::odd_max(R, nmk); }
  __device__ static float2 odd_max2(const DevBook&, const float2 (&Rp)[25], const float* nmk) {
    return S::odd_max2(Rp, nmk);
  }
  __device__ static float2 even_max2_w12(const DevBook&, const float2 (&R0p)[25], const float2 (&R1p)[25], float2 P0p,
                                         float2 P1p, const float* nmk) {
    return S::even_max2_w12(R0p, R1p, P0p, P1p, nmk);
  }
  template <class F>
  __device__ static void odd_cands(const DevBook&, const float (&R)[25], const float* nmk, float thr, F&& f) {
    S::odd_cands(R, nmk, thr, f);
  }
  template <int W>
  __device__ static float even_max(const DevBook&, const float (&R0)[25], const float (&R1)[25], float P0, float P1,
                                   const float* nmk) {
    if constexpr (W == 0) return S::even_max_w0(R0, R1, P0, P1, nmk);
    else if constexpr (W == 8) return S::even_max_w8(R0, R1, P0, P1, nmk);
    else if constexpr (W == 12) return S::even_max_w12(R0, R1, P0, P1, nmk);
    else if constexpr (W == 16) return S::even_max_w16(R0, R1, P0, P1, nmk);
    else return S::even_max_w24(R0, R1, P0, P1, nmk);
  }
  template <int W, class F>
  __device__ static void even_cands(const DevBook&, const float (&R0)[25], const float (&R1)[25], float P0, float P1,
                                    const float* nmk, float thr, F&& f) {
    if constexpr (W == 0) S::even_cands_w0(R0, R1, P0, P1, nmk, thr, f);
    else if constexpr (W == 8) S::even_cands_w8(R0, R1, P0, P1, nmk, thr, f);
    else if constexpr (W == 12) S::even_cands_w12(R0, R1, P0, P1, nmk, thr, f);
    else if constexpr (W == 16) S::even_cands_w16(R0, R1, P0, P1, nmk, thr, f);
    else S::even_cands_w24(R0, R1, P0, P1, nmk, thr, f);
  }
};

// Table-driven scoring for any codebook (no generated code): the same FFMA
// chains read from DevClass::term_*.
struct RuntimeSpec {};
constexpr int kRuntimeShells = 64;

__device__ __forceinline__ float runtime_chain(const DevClass& c, const float* R, const float* R0, const float* R1,
                                               float P0, float P1, const float* nmk, int min_shell) {
  float acc = nmk[c.shell - min_shell];
  for (int t = 0; t < c.nterms; ++t) {
    const int kind = c.term_kind[t], idx = c.term_idx[t];
    const float v = kind == 0 ? R[idx] : kind == 1 ? R0[idx] : kind == 2 ? R1[idx] : kind == 3 ? P0 : P1;
    acc = fmaf(c.term_coef[t], v, acc);
  }
  return acc;
}

template <>
struct Ops<RuntimeSpec> {
  static constexpr int kThreads = kSearchThreads;
  static constexpr int kMinBlocks = kSearchMinBlocks;
  static constexpr bool kRealign = true;
  static constexpr int kNumShells = kRuntimeShells;
  static constexpr int kMinShellC = -1;
  static constexpr bool kHasOdd = true;
  static constexpr bool kAngular = false;
  static constexpr bool kPacked = false;
  template <int W>
  static constexpr bool has_even() { return true; }
  template <int W>
  static constexpr int r0max() { return kDim - W; }
  __device__ static float odd_max(const DevBook& b, const float (&R)[25], const float* nmk) {
    float best = -INFINITY;
    for (int k = 0; k < b.n_classes; ++k) {
      const DevClass& c = b.cls[k];
      if (c.parity != 1) continue;
      best = fmaxf(best, runtime_chain(c, R, nullptr, nullptr, 0.f, 0.f, nmk, b.min_shell));
    }
    return best;
  }
  template <class F>
  __device__ static void odd_cands(const DevBook& b, const float (&R)[25], const float* nmk, float thr, F&& f) {
    for (int k = 0; k < b.n_classes; ++k) {
      const DevClass& c = b.cls[k];
      if (c.parity != 1) continue;
      const float s = runtime_chain(c, R, nullptr, nullptr, 0.f, 0.f, nmk, b.min_shell);
      if (s >= thr) f(k, s);
    }
  }
  template <int W>
  __device__ static float even_max(const DevBook& b, const float (&R0)[25], const float (&R1)[25], float P0, float P1,
                                   const float* nmk) {
    float best = -INFINITY;
    for (int k = 0; k < b.n_classes; ++k) {
      const DevClass& c = b.cls[k];
      if (c.parity != 0 || c.even_weight != W) continue;
      best = fmaxf(best, runtime_chain(c, nullptr, R0, R1, P0, P1, nmk, b.min_shell));
    }
    return best;
  }
  template <int W, class F>
  __device__ static void even_cands(const DevBook& b, const float (&R0)[25], const float (&R1)[25], float P0, float P1,
                                    const float* nmk, float thr, F&& f) {
    for (int k = 0; k < b.n_classes; ++k) {
      const DevClass& c = b.cls[k];
      if (c.parity != 0 || c.even_weight != W) continue;
      const float s = runtime_chain(c, nullptr, R0, R1, P0, P1, nmk, b.min_shell);
      if (s >= thr) f(k, s);
    }
  }
};

// ------------------------------------------------------------ word scoring

// Odd classes: R[t] = sum of the t largest x'_i.  The selected entries of the
// 48-slot sorted list (positives at 24 + rank, negatives at 23 - rank) are
// exactly one per coordinate; the t largest are the top t set bits.
// The walk takes one 32-bit half at a time: the positives (the ranks of
// posA, largest first: lval[24 + r]) until they run out, then the negatives
// (the other ranks, smallest first: bit 23 - r of lo, lval[23 - r]); the two
// sets cover all 24 ranks, so no scan sees zero.  Against one 64-bit mask
// with a 64-bit scan and clear: +4% on shells 2..13 and +11% on shell 11.
// PTR (the small scoring codes) switches a pointer into lval, the others an
// integer offset (each form 2-4% faster than the other on its codebooks).
template <bool PTR, class Row>
__device__ __forceinline__ void odd_sums(const Row& sh, uint32_t cA, float (&R)[25]) {
  const uint32_t posA = cA ^ sh.nposA;
  uint32_t w = posA, lo = __brev(~posA & kFull24) >> 8;
  R[0] = 0.f;
  if constexpr (PTR) {
    const float* base = sh.lval + 24;
#pragma unroll
    for (int t = 1; t <= kDim; ++t) {
      if (w == 0u) {
        w = lo;
        lo = 0u;
        base = sh.lval;
      }
      const int b = 31 - __clz(w);
      R[t] = R[t - 1] + base[b];
      w ^= 1u << b;
    }
  } else {
    int off = 24;
#pragma unroll
    for (int t = 1; t <= kDim; ++t) {
      if (w == 0u) {
        w = lo;
        lo = 0u;
        off = 0;
      }
      const int b = 31 - __clz(w);
      R[t] = R[t - 1] + sh.lval[off + b];
      w ^= 1u << b;
    }
  }
}

// Even classes of word weight W: suffix sums of |q| inside (R1) and outside
// (R0) the word, and the sign-parity penalties.
template <int W, int N0, class Row>
__device__ __forceinline__ void even_sums(const Row& sh, uint32_t c, uint32_t cA, float (&R0)[25],
                                          float (&R1)[25], float& P0, float& P1) {
  uint32_t f1 = cA, f0 = ~cA & kFull24;
  R1[0] = 0.f;
#pragma unroll
  for (int t = 1; t <= W; ++t) {
    const int j = 31 - __clz(f1);
    R1[t] = R1[t - 1] + sh.aval[j];
    f1 ^= 1u << j;
  }
  R0[0] = 0.f;
#pragma unroll
  for (int t = 1; t <= N0; ++t) {
    const int j = 31 - __clz(f0);
    R0[t] = R0[t - 1] + sh.aval[j];
    f0 ^= 1u << j;
  }
  const float qmin1 = W ? sh.aval[__ffs(cA) - 1] : 0.f;
  const int negpar = __popc(c & sh.negmask) & 1;
  P0 = negpar ? qmin1 : 0.f;  // penalty for classes that need an even count of negatives
  P1 = negpar ? 0.f : qmin1;  // ... and for those that need an odd count
}

template <class S, int W, class Row, class F>
__device__ __forceinline__ void even_cands_word(const DevBook& b, const Row& sh, uint32_t c, uint32_t cA,
                                                const float* nmk, float thr, F&& f) {
  if constexpr (Ops<S>::template has_even<W>()) {
    float R0[25], R1[25], P0, P1;
    even_sums<W, Ops<S>::template r0max<W>()>(sh, c, cA, R0, R1, P0, P1);
    Ops<S>::template even_cands<W>(b, R0, R1, P0, P1, nmk, thr, f);
  }
}

__device__ __forceinline__ uint32_t permute_word(const RowShared& sh, uint32_t c) {
  return sh.utab[0][c & 255u] | sh.utab[1][(c >> 8) & 255u] | sh.utab[2][c >> 16];
}

__device__ __forceinline__ uint32_t permute_word(const RowLocal& r, uint32_t c) {
  uint32_t u = 0;
#pragma unroll
  for (int d = 0; d < kDim; ++d)
    if ((c >> d) & 1u) u |= 1u << r.arank[d];
  return u;
}

template <class S, class Row, class F>
__device__ __forceinline__ void word_cands(const DevBook& b, const Row& sh, uint32_t c, const float* nmk,
                                           float thr, F&& f) {
  const uint32_t cA = permute_word(sh, c);
  if constexpr (Ops<S>::kHasOdd) {
    float R[25];
    odd_sums<!Ops<S>::kRealign>(sh, cA, R);
    Ops<S>::odd_cands(b, R, nmk, thr, f);
  }
  switch (__popc(c)) {
    case 8: even_cands_word<S, 8>(b, sh, c, cA, nmk, thr, f); break;
    case 12: even_cands_word<S, 12>(b, sh, c, cA, nmk, thr, f); break;
    case 16: even_cands_word<S, 16>(b, sh, c, cA, nmk, thr, f); break;
    case 0: even_cands_word<S, 0>(b, sh, c, cA, nmk, thr, f); break;
    default: even_cands_word<S, 24>(b, sh, c, cA, nmk, thr, f); break;
  }
}

// ------------------------------------------- complementary word pairs
//
// The all-ones word is a Golay word, so the words pair up as (c, ~c), and
// one walk over the sorted coordinates serves both.  Odd classes: x' of ~c
// is -x' of c, so R_~c[t] = R_c[24 - t] - R_c[24] (exact: integers below
// 2^24 in fp32).  Even classes: the in-word and off-word suffix sums swap,
// so walking both completely (24 steps) gives both words' sums.  Each
// complement sum is bounded like the sum it replaces, so the window constants
// of the scoring chains hold for both words.
//
// Generated codebooks score both words of a pair in one pass wherever they
// run the same classes (every odd class; the even classes of a 12/12 pair):
// lane x of float2 operands holds c's sums, lane y ~c's, and every chain step
// below a trie root is one FFMA2 (fma.rn.f32x2: each lane rounds exactly like
// the scalar FFMA, so the scores and the window are unchanged).  On shells
// 2..13 this took the search from 6.70 to 7.1 M blocks/s; on shell 32 (3.0
// bits/dim shape-gain) from 1.28 to 1.61 M.  8/16 and 0/24 pairs run different
// even classes on their two words and stay scalar.

// Even sums of c (weight W) and of ~c (weight 24 - W): R1 over c's W
// positions, R0 over the others, the sign-parity penalties of both words.
template <int W, class Row>
__device__ __forceinline__ void even_sums_pair(const Row& sh, uint32_t c, uint32_t cA, float (&R0)[25],
                                               float (&R1)[25], float& P0, float& P1, float& Q0, float& Q1) {
  uint32_t f1 = cA, f0 = ~cA & kFull24;
  R1[0] = 0.f;
#pragma unroll
  for (int t = 1; t <= W; ++t) {
    const int j = 31 - __clz(f1);
    R1[t] = R1[t - 1] + sh.aval[j];
    f1 ^= 1u << j;
  }
  R0[0] = 0.f;
#pragma unroll
  for (int t = 1; t <= kDim - W; ++t) {
    const int j = 31 - __clz(f0);
    R0[t] = R0[t - 1] + sh.aval[j];
    f0 ^= 1u << j;
  }
  const float qc = W ? sh.aval[__ffs(cA) - 1] : 0.f;
  const float qn = W < kDim ? sh.aval[__ffs(~cA & kFull24) - 1] : 0.f;
  const int nc = __popc(c & sh.negmask) & 1, nn = __popc(~c & kFull24 & sh.negmask) & 1;
  P0 = nc ? qc : 0.f;
  P1 = nc ? 0.f : qc;
  Q0 = nn ? qn : 0.f;
  Q1 = nn ? 0.f : qn;
}

template <class S, int W, class Row>
__device__ __forceinline__ void even_pair_max(const DevBook& b, const Row& sh, uint32_t c, uint32_t cA,
                                              const float* nmk, float& bc, float& bn) {
  constexpr int WC = kDim - W;
  if constexpr (W == WC && Ops<S>::kPacked) {
    if constexpr (Ops<S>::template has_even<W>()) {
      // both words weigh 12: lane x scores c, lane y scores ~c, whose in-word
      // and off-word sums are c's off-word and in-word sums
      float R0[25], R1[25], P0, P1, Q0, Q1;
      even_sums_pair<W>(sh, c, cA, R0, R1, P0, P1, Q0, Q1);
      float2 R0p[25], R1p[25];
#pragma unroll
      for (int t = 0; t <= W; ++t) {
        R0p[t] = make_float2(R0[t], R1[t]);
        R1p[t] = make_float2(R1[t], R0[t]);
      }
      const float2 v = Ops<S>::even_max2_w12(b, R0p, R1p, make_float2(P0, Q0), make_float2(P1, Q1), nmk);
      bc = fmaxf(bc, v.x);
      bn = fmaxf(bn, v.y);
    }
  } else if constexpr (W == WC) {
    if constexpr (Ops<S>::template has_even<W>()) {
      // both words weigh 12: one copy of the scoring code, run twice with
      // the in-word and off-word sums swapped in between (the generated code
      // is large; two inlined copies would not stay in the instruction cache)
      float R0[25], R1[25], P0, P1, Q0, Q1;
      even_sums_pair<W>(sh, c, cA, R0, R1, P0, P1, Q0, Q1);
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const float v = Ops<S>::template even_max<W>(b, R0, R1, P0, P1, nmk);
        if (h == 0) {
          bc = fmaxf(bc, v);
#pragma unroll
          for (int t = 0; t <= W; ++t) {
            const float x = R0[t];
            R0[t] = R1[t];
            R1[t] = x;
          }
          P0 = Q0;
          P1 = Q1;
        } else {
          bn = fmaxf(bn, v);
        }
      }
    }
  } else if constexpr (Ops<S>::template has_even<W>() || Ops<S>::template has_even<WC>()) {
    float R0[25], R1[25], P0, P1, Q0, Q1;
    even_sums_pair<W>(sh, c, cA, R0, R1, P0, P1, Q0, Q1);
    if constexpr (Ops<S>::template has_even<W>()) bc = fmaxf(bc, Ops<S>::template even_max<W>(b, R0, R1, P0, P1, nmk));
    if constexpr (Ops<S>::template has_even<WC>())
      bn = fmaxf(bn, Ops<S>::template even_max<WC>(b, R1, R0, Q0, Q1, nmk));
  }
}

// Best approximate scores of c and of ~c (c: weight 0, 8 or 12).
template <class S, class Row>
__device__ __forceinline__ void pair_max(const DevBook& b, const Row& sh, uint32_t c, const float* nmk, float& bc,
                                         float& bn) {
  const uint32_t cA = permute_word(sh, c);
  bc = -INFINITY;
  bn = -INFINITY;
  if constexpr (Ops<S>::kHasOdd && Ops<S>::kPacked) {
    float R[25];
    odd_sums<!Ops<S>::kRealign>(sh, cA, R);
    float2 R2[25];
#pragma unroll
    for (int t = 0; t <= kDim; ++t) R2[t] = make_float2(R[t], R[kDim - t] - R[kDim]);
    const float2 v = Ops<S>::odd_max2(b, R2, nmk);
    bc = v.x;
    bn = v.y;
  } else if constexpr (Ops<S>::kHasOdd) {
    float R[25];
    odd_sums<!Ops<S>::kRealign>(sh, cA, R);
    const float r24 = R[kDim];
#pragma unroll 1
    for (int h = 0; h < 2; ++h) {  // one copy of the odd scoring code for both words
      const float v = Ops<S>::odd_max(b, R, nmk);
      if (h == 0) {
        bc = v;
#pragma unroll
        for (int t = 0; t <= kDim / 2; ++t) {  // in place: R[t] <- R[24 - t] - R[24]
          const float lo = R[t], hi = R[kDim - t];
          R[t] = hi - r24;
          R[kDim - t] = lo - r24;
        }
      } else {
        bn = v;
      }
    }
  }
  switch (__popc(c)) {
    case 8: even_pair_max<S, 8>(b, sh, c, cA, nmk, bc, bn); break;
    case 0: even_pair_max<S, 0>(b, sh, c, cA, nmk, bc, bn); break;
    default: even_pair_max<S, 12>(b, sh, c, cA, nmk, bc, bn); break;
  }
}

// ------------------------------------------------------------- the search

// Exact-pass handler for one candidate pair: the reference's codeword and fp64
// score, kept if it beats (score desc, loop order asc).  Not inlined: the
// generated scoring code calls it from every class site.
template <bool ANG>
__device__ __noinline__ void consider_exact(const float* x, const int8_t* apos, const DevBook& book, uint32_t word,
                                            int lex, int k, double* best, long long* order) {
  int y[kDim];
  const DevClass& cls = book.cls[k];
  build_candidate(x, apos, cls, word, y);
  const double s = exact_score<ANG>(x, y, cls.shell);
  const long long o = (long long)lex * book.n_classes + k;
  if (s > *best || (s == *best && o < *order)) {
    *best = s;
    *order = o;
  }
}

// Gain code of the winning codeword for shape-gain quantization (gc.thr
// null: none).  g = <x, y> / |y| (the projection is the reference score's
// compensated fp64 sum; |y| = sqrt(16 shell)), divided by gc.sigma[row /
// gc.bpr] when given; the code is the number of thresholds below g.
__device__ __forceinline__ int gain_code(const GainCode& gc, const float* x, const int* y, int shell, int64_t row) {
  double g = __ddiv_rn(reference_projection(x, y), __dsqrt_rn(16.0 * (double)shell));
  if (gc.sigma) g = __ddiv_rn(g, (double)__ldg(gc.sigma + row / gc.bpr));
  int lo = 0, hi = gc.nthr;  // first threshold >= g
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if (__ldg(gc.thr + mid) < g) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// Rebuild the winning codeword, its fp64 reference score and its index (and
// its gain code).
template <bool ANG>
__device__ __noinline__ void write_winner(const float* x, const int8_t* apos, const DevBook& book, long long order,
                                          int64_t row, long long* index_out, long long* pair_out, float* score_out,
                                          GainCode gc) {
  const int lex = (int)(order / book.n_classes), k = (int)(order % book.n_classes);
  const DevClass& c = book.cls[k];
  const uint32_t word = book.golay[lex];
  int y[kDim];
  build_candidate(x, apos, c, word, y);
  const double s = exact_score<ANG>(x, y, c.shell);
  const int choice = c.parity ? lex : (int)book.golay_wrank[lex];
  long long idx = rank_codeword(c, y, word, choice);
  if (gc.thr) {
    const int g = gain_code(gc, x, y, c.shell, row);
    if (gc.gain_out) gc.gain_out[row] = g;
    if (gc.pack) idx = (idx << gc.bits) | g;
  }
  index_out[row] = idx;
  pair_out[row] = (long long)k * kNumGolay + lex;
  score_out[row] = (float)s;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

// Stage one block: x, validity, scale, sorted |x| order and the word tables.
// The row's 24 values come from warp 0 (lane d holds x[row, d], loaded one
// row ahead by the caller so that the load's latency overlaps the previous
// row's search).
__device__ void stage_row(float v, RowShared& sh) {
  const int tid = threadIdx.x, lane = tid & 31;
  if (tid < 32) {
    if (lane < kDim) sh.x[lane] = v;
    const unsigned bad = __ballot_sync(0xffffffffu, lane < kDim && !isfinite(v));
    const unsigned neg = __ballot_sync(0xffffffffu, lane < kDim && v < 0.f);
    const float mx = warp_max(fabsf(v));
    if (lane == 0) {
      sh.invalid = bad != 0;
      sh.negmask = neg & kFull24;
      sh.scale = pow2f(row_exponent(mx));
      sh.K = kSqrt8F * sh.scale;
    }
  }
  __syncthreads();
  if (tid < kDim && !sh.invalid) {
    const float ai = fabsf(sh.x[tid]);
    int r = 0;
#pragma unroll
    for (int j = 0; j < kDim; ++j) {
      const float aj = fabsf(sh.x[j]);
      r += (aj < ai) || (aj == ai && j < tid);
    }
    const float q = rintf(ai * sh.scale);
    sh.arank[tid] = (int8_t)r;
    sh.apos[r] = (int8_t)tid;
    sh.aval[r] = q;
    sh.lval[24 + r] = q;
    sh.lval[23 - r] = -q;
  }
  __syncthreads();
  if (!sh.invalid) {
    for (int i = tid; i < 3 * 256; i += blockDim.x) {
      const int t = i >> 8, v = i & 255;
      uint32_t u = 0;
#pragma unroll
      for (int bit = 0; bit < 8; ++bit)
        if ((v >> bit) & 1) u |= 1u << sh.arank[8 * t + bit];
      sh.utab[t][v] = u;
    }
    if (tid == 0) {
      const uint32_t pos = ~sh.negmask & kFull24;
      uint32_t u = 0;
      for (int d = 0; d < kDim; ++d)
        if ((pos >> d) & 1u) u |= 1u << sh.arank[d];
      sh.nposA = u;
    }
  }
  __syncthreads();
}

template <class S>
__global__ void __launch_bounds__(Ops<S>::kThreads, Ops<S>::kMinBlocks) search_kernel(const float* __restrict__ x, int64_t n, DevBook book,
                                                                long long* tag_out, float* m_out) {
  __shared__ RowShared sh;
  constexpr int T = Ops<S>::kThreads;
  constexpr int kWordsPerThread = kNumGolay / T;
  constexpr int kPairsPerThread = kWordsPerThread / 2;
  static_assert(T <= kMaxSearchThreads && kNumGolay % (2 * T) == 0, "CTA shape");
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  constexpr int NS = Ops<S>::kNumShells;
  const int min_shell = Ops<S>::kMinShellC >= 0 ? Ops<S>::kMinShellC : book.min_shell;
  float xv = (tid < kDim && blockIdx.x < n) ? x[(int64_t)blockIdx.x * kDim + tid] : 0.f;
  for (int64_t row = blockIdx.x; row < n; row += gridDim.x) {
    stage_row(xv, sh);
    if (tid < kDim && row + gridDim.x < n) xv = x[(row + gridDim.x) * kDim + tid];  // next row
    if (sh.invalid) {
      if (tid == 0) {
        tag_out[row] = -1;
        m_out[row] = NAN;
      }
      __syncthreads();
      continue;
    }
    float nmk[NS];
#pragma unroll
    for (int s = 0; s < NS; ++s) nmk[s] = -(float)(min_shell + s) * sh.K;

    // best score (b1) and word (lex w1) of this thread's words, and the best
    // score of its other words (b2)
    float b1 = -INFINITY, b2 = -INFINITY;
    int w1 = -1;
    auto take = [&](float bw, int lex) {
      if (bw > b1) {
        b2 = b1;
        b1 = bw;
        w1 = lex;
      } else {
        b2 = fmaxf(b2, bw);
      }
    };
    for (int i = 0; i < kPairsPerThread; ++i) {
      // realign the warps (instruction cache): 256-thread CTAs in two groups
      // of four warps (named barriers 1 and 2; +2% on shells 2..13 over one
      // barrier for all eight), 512-thread CTAs all together (groups of four
      // ran 15% slower on shell 32)
      if constexpr (Ops<S>::kRealign) {
        if constexpr (T == 256) asm volatile("bar.sync %0, 128;" ::"r"(1 + (warp >> 2)) : "memory");
        else __syncthreads();
      }
      const int j = i * T + tid;
      const uint32_t c = __ldg(book.plist_word + j);
      const int lex = __ldg(book.plist_lex + j);
      float bc, bn;
      pair_max<S>(book, sh, c, nmk, bc, bn);
      take(bc, lex);
      take(bn, kNumGolay - 1 - lex);
    }
    const float wm = warp_max(b1);
    if (lane == 0) sh.red[warp] = wm;
    __syncthreads();
    float M = sh.red[0];
#pragma unroll
    for (int w = 1; w < T / 32; ++w) M = fmaxf(M, sh.red[w]);
    const float thr = __double2float_rd((double)M - window_width(sh.K, book));
    const int contenders = __syncthreads_count(b1 >= thr);
    const int second = __syncthreads_or(b2 >= thr);
    if (contenders == 1 && !second) {
      if (b1 >= thr) {
        tag_out[row] = kTagWord | (long long)w1;
        m_out[row] = M;
      }
    } else {
      // Exact pass: every pair inside the window, scored with the reference
      // arithmetic; ties go to the earliest (Golay word, class) in loop order.
      double best = -INFINITY;
      long long order = LLONG_MAX;
      for (int i = 0; i < kWordsPerThread; ++i) {
        const int j = i * T + tid;
        const uint32_t c = __ldg(book.wlist_word + j);
        const int lex = __ldg(book.wlist_lex + j);
        word_cands<S>(book, sh, c, nmk, thr,
                      [&](int k, float) {
                        consider_exact<Ops<S>::kAngular>(sh.x, sh.apos, book, c, lex, k, &best, &order);
                      });
      }
      sh.xs_best[tid] = best;
      sh.xs_order[tid] = order;
      __syncthreads();
      if (tid == 0) {
        for (int t = 1; t < T; ++t) {
          if (sh.xs_best[t] > best || (sh.xs_best[t] == best && sh.xs_order[t] < order)) {
            best = sh.xs_best[t];
            order = sh.xs_order[t];
          }
        }
        tag_out[row] = kTagExact | ((order % book.n_classes) << 12) | (order / book.n_classes);
        m_out[row] = (float)best;
      }
    }
    __syncthreads();
  }
}

// ------------------------------------------------------------- finalize

// One thread per block: rebuild the block's sorted data, re-score the handed
// word's pairs inside the window with the generated code and decide them in
// fp64, then write index, pair and score.
template <class S>
__global__ void __launch_bounds__(128) finalize_kernel(const float* __restrict__ x, int64_t n, DevBook book,
                                                       const long long* tag_in, const float* m_in,
                                                       long long* index_out, long long* pair_out, float* score_out,
                                                       GainCode gc) {
  const int64_t row = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (row >= n) return;
  const long long tag = tag_in[row];
  if (tag < 0) {
    index_out[row] = -1;
    pair_out[row] = -1;
    score_out[row] = NAN;
    if (gc.gain_out) gc.gain_out[row] = -1;
    return;
  }
  RowLocal r;
  float mx = 0.f;
  r.negmask = 0;
#pragma unroll
  for (int d = 0; d < kDim; ++d) {
    r.x[d] = x[row * kDim + d];
    mx = fmaxf(mx, fabsf(r.x[d]));
    r.negmask |= (uint32_t)(r.x[d] < 0.f) << d;
  }
  r.scale = pow2f(row_exponent(mx));
  r.K = kSqrt8F * r.scale;
#pragma unroll
  for (int i = 0; i < kDim; ++i) {
    const float ai = fabsf(r.x[i]);
    int rk = 0;
#pragma unroll
    for (int j = 0; j < kDim; ++j) {
      const float aj = fabsf(r.x[j]);
      rk += (aj < ai) || (aj == ai && j < i);
    }
    r.arank[i] = (int8_t)rk;
  }
  for (int i = 0; i < kDim; ++i) {
    const int rk = r.arank[i];
    const float q = rintf(fabsf(r.x[i]) * r.scale);
    r.apos[rk] = (int8_t)i;
    r.aval[rk] = q;
    r.lval[24 + rk] = q;
    r.lval[23 - rk] = -q;
  }
  {
    const uint32_t pos = ~r.negmask & kFull24;
    uint32_t u = 0;
    for (int d = 0; d < kDim; ++d)
      if ((pos >> d) & 1u) u |= 1u << r.arank[d];
    r.nposA = u;
  }
  long long order;
  if (tag & kTagExact) {
    order = (tag & 4095) * book.n_classes + ((tag >> 12) & ((1ll << 28) - 1));
  } else {
    constexpr int NS = Ops<S>::kNumShells;
    const int min_shell = Ops<S>::kMinShellC >= 0 ? Ops<S>::kMinShellC : book.min_shell;
    float nmk[NS];
#pragma unroll
    for (int s = 0; s < NS; ++s) nmk[s] = -(float)(min_shell + s) * r.K;
    const float thr = __double2float_rd((double)m_in[row] - window_width(r.K, book));
    const int lex = (int)(tag & 4095);
    const uint32_t c = __ldg(book.golay + lex);
    double best = -INFINITY;
    order = LLONG_MAX;
    // Collect the window's classes first and score them afterwards in one
    // loop, so the lanes of a warp run the fp64 scoring together instead of
    // one by one at each generated class site.
    constexpr int kMaxCands = 8;
    int cand[kMaxCands];
    int nc = 0;
    word_cands<S>(book, r, c, nmk, thr, [&](int k, float) {
      if (nc < kMaxCands) cand[nc++] = k;
      else consider_exact<Ops<S>::kAngular>(r.x, r.apos, book, c, lex, k, &best, &order);
    });
    for (int i = 0; i < nc; ++i) consider_exact<Ops<S>::kAngular>(r.x, r.apos, book, c, lex, cand[i], &best, &order);
    if (order == LLONG_MAX) {  // cannot happen for a finite row
      index_out[row] = -1;
      pair_out[row] = -1;
      score_out[row] = NAN;
      if (gc.gain_out) gc.gain_out[row] = -1;
      return;
    }
  }
  write_winner<Ops<S>::kAngular>(r.x, r.apos, book, order, row, index_out, pair_out, score_out, gc);
}

// ------------------------------------------------------------- launchers

template <class S>
static cudaError_t launch_search(const float* x, int64_t n, const DevBook& book, long long* index, long long* pair,
                                 float* score, const GainCode& gc, cudaStream_t stream) {
  // persistent grid: SMs x resident CTAs, looked up once per device (host
  // threads that race here compute the same value)
  static std::atomic<int> grid_cap[kMaxDevices];
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  if (dev < 0 || dev >= kMaxDevices) return cudaErrorInvalidDevice;
  int cap = grid_cap[dev].load(std::memory_order_relaxed);
  if (cap <= 0) {
    int sms = 0, blocks_per_sm = 0;
    e = cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (e != cudaSuccess) return e;
    e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&blocks_per_sm, search_kernel<S>, Ops<S>::kThreads, 0);
    if (e != cudaSuccess) return e;
    cap = sms * std::max(blocks_per_sm, 1);
    grid_cap[dev].store(cap, std::memory_order_relaxed);
  }
  const int64_t grid = std::min<int64_t>(n, (int64_t)cap);
  search_kernel<S><<<(unsigned)grid, Ops<S>::kThreads, 0, stream>>>(x, n, book, pair, score);
  cudaError_t err = cudaGetLastError();
  if (err != cudaSuccess) return err;
  finalize_kernel<S><<<(unsigned)((n + 127) / 128), 128, 0, stream>>>(x, n, book, pair, score, index, pair, score,
                                                                      gc);
  return cudaGetLastError();
}

#define LLVQ_SPEC_ENTRY(NAME)                                                                     \
  {gen::kSig_##NAME, &launch_search<gen::Spec_##NAME>, #NAME, (float)gen::Spec_##NAME::kL1Max, \
   (float)gen::Spec_##NAME::kWinMG, (float)gen::Spec_##NAME::kWinAM, gen::Spec_##NAME::kAngular},
static const SpecEntry kSpecs[] = {LLVQ_FOR_EACH_SPEC(LLVQ_SPEC_ENTRY)};

const SpecEntry* spec_table(int* count) {
  *count = (int)(sizeof(kSpecs) / sizeof(kSpecs[0]));
  return kSpecs;
}

cudaError_t quantize_launch(const Codebook& cb, const float* x, int64_t n, long long* index, long long* pair,
                            float* score, cudaStream_t stream, bool force_runtime, const GainCode& gc, bool angular) {
  if (n <= 0) return cudaSuccess;
  DevBook book = cb.dev;
  SearchLauncher launch;
  if (angular) {  // generated code only
    if (!cb.spec_ang) return cudaErrorNotSupported;
    launch = cb.spec_ang->launch;
    book.l1max = cb.spec_ang->l1max;
    book.win_mg = cb.spec_ang->win_mg;
    book.win_am = cb.spec_ang->win_am;
  } else if (cb.spec && !force_runtime) {
    launch = cb.spec->launch;
    book.l1max = cb.spec->l1max;
    book.win_mg = cb.spec->win_mg;
    book.win_am = cb.spec->win_am;
  } else {
    launch = &launch_search<RuntimeSpec>;
    book.l1max = cb.rt_l1max;
    book.win_mg = cb.rt_mg;
    book.win_am = cb.rt_am;
  }
  return launch(x, n, book, index, pair, score, gc, stream);
}

}  // namespace llvq
