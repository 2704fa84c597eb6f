// Host-side codebook builder and the C ABI (include/llvq_b200.h).
//
// The builder turns a class list (shell, parity, leader) into the device
// tables: per-class counts and rank data, the Golay word tables and the
// FFMA chains of the table-driven search.  Counts follow
// build_local_structure (impl/leech_lattice_vector_quantizer_gpu.py:570-601)
// and the offsets LeechLatticeVectorQuantizerGpu._build_*_offsets (:520-537).
#include <cuda_runtime.h>

#include <algorithm>
#include <climits>
#include <cmath>
#include <cstdio>
#include <cstring>
#include <new>
#include <string>

#include "../../include/llvq_b200.h"
#include "llvq_device.cuh"
#include "llvq_internal.h"
#include "llvq_tables.cuh"

struct llvq_codebook {
  llvq::Codebook cb;
};

namespace {

thread_local std::string g_last_error;

int fail(int status, const std::string& msg) {
  g_last_error = msg;
  return status;
}

int cuda_fail(cudaError_t e, const char* where) {
  if (e == cudaErrorMemoryAllocation) return fail(LLVQ_ERR_OUT_OF_MEMORY, std::string(where) + ": out of device memory");
  return fail(LLVQ_ERR_CUDA, std::string(where) + ": " + cudaGetErrorName(e) + " (" + cudaGetErrorString(e) + ")");
}

using u128 = unsigned __int128;

// Extended Golay code in the reference's order: cyclic [23,12,7] code of
// g(x) = x^11+x^9+x^7+x^6+x^5+x+1, parity appended, sorted as 0/1 tuples with
// coordinate 0 first (extended_golay_codewords, _gpu.py:1048-1067).
std::vector<uint32_t> golay_lex() {
  const uint32_t g = 0b101011100011u;
  std::vector<uint32_t> keys(llvq::kNumGolay);
  for (uint32_t msg = 0; msg < (uint32_t)llvq::kNumGolay; ++msg) {
    uint32_t c = 0;
    for (int b = 0; b < 12; ++b)
      if ((msg >> b) & 1u) c ^= g << b;
    c &= 0x7FFFFFu;
    const uint32_t word = c | ((uint32_t)(__builtin_popcount(c) & 1) << 23);
    uint32_t key = 0;  // coordinate 0 most significant
    for (int d = 0; d < llvq::kDim; ++d) key |= ((word >> d) & 1u) << (23 - d);
    keys[msg] = key;
  }
  std::sort(keys.begin(), keys.end());
  std::vector<uint32_t> out(llvq::kNumGolay);
  for (int i = 0; i < llvq::kNumGolay; ++i) {
    uint32_t w = 0;
    for (int d = 0; d < llvq::kDim; ++d) w |= ((keys[i] >> (23 - d)) & 1u) << d;
    out[i] = w;
  }
  return out;
}

u128 multinomial(const int32_t* mult, int nv) {
  u128 out = 1;
  int rem = 0;
  for (int j = 0; j < nv; ++j) rem += mult[j];
  for (int j = 0; j < nv; ++j) {
    u128 c = 1;
    for (int k = 1; k <= mult[j]; ++k) c = c * (u128)(rem - mult[j] + k) / (u128)k;
    out *= c;
    rem -= mult[j];
  }
  return out;
}

void distinct_desc(const int* vals, int n, int32_t* v, int32_t* m, int* nv) {
  *nv = 0;
  for (int i = 0; i < n; ++i) {
    if (*nv && v[*nv - 1] == vals[i]) {
      m[*nv - 1]++;
    } else {
      if (*nv == llvq::kMaxVals + 1) return;  // caller rejects nv > kMaxVals
      v[*nv] = vals[i];
      m[*nv] = 1;
      (*nv)++;
    }
  }
}

// FFMA chain of a class for the table-driven search, in the natural order
// (the window constants below are computed for exactly this order).
void build_chain(llvq::DevClass& c, const int* leader) {
  c.nterms = 0;
  auto add = [&](float coef, int kind, int idx) {
    c.term_coef[c.nterms] = coef;
    c.term_kind[c.nterms] = (int8_t)kind;
    c.term_idx[c.nterms] = (int8_t)idx;
    c.nterms++;
  };
  if (c.parity == 1) {
    int s[llvq::kDim];
    for (int d = 0; d < llvq::kDim; ++d) s[d] = (leader[d] % 4 == 1) ? leader[d] : -leader[d];
    std::sort(s, s + llvq::kDim, [](int a, int b) { return a > b; });
    int32_t v[llvq::kMaxVals + 1], m[llvq::kMaxVals + 1];
    int nv;
    distinct_desc(s, llvq::kDim, v, m, &nv);
    int cum = 0;
    for (int j = 0; j < nv; ++j) {
      cum += m[j];
      add((float)(j + 1 < nv ? v[j] - v[j + 1] : v[j]), 0, cum);
    }
  } else {
    int cum = 0;
    for (int j = 0; j < c.nv0; ++j) {
      cum += c.m0[j];
      const int nxt = j + 1 < c.nv0 ? c.v0[j + 1] : 0;
      if (c.v0[j] - nxt) add((float)(c.v0[j] - nxt), 1, cum);
    }
    cum = 0;
    for (int j = 0; j < c.nv1; ++j) {
      cum += c.m1[j];
      const int nxt = j + 1 < c.nv1 ? c.v1[j + 1] : 0;
      add((float)(c.v1[j] - nxt), 2, cum);
    }
    if (c.even_weight) add((float)(-2 * c.v1[c.nv1 - 1]), 3 + c.required, 0);
  }
}

// The class search's bucket table stores class numbers in 16 bits.
constexpr int kMaxClasses = 65536;

int build(llvq::Codebook& cb, int32_t n, const int32_t* shell, const int32_t* parity, const int32_t* leader) {
  using namespace llvq;
  if (n <= 0 || !shell || !parity || !leader) return fail(LLVQ_ERR_INVALID_ARGUMENT, "empty class list");
  if (n > kMaxClasses) return fail(LLVQ_ERR_UNSUPPORTED, "more than 65536 classes");
  cb.golay = golay_lex();
  int nww[25] = {0};
  cb.golay_wrank.resize(kNumGolay);
  for (int i = 0; i < kNumGolay; ++i) {
    const int w = __builtin_popcount(cb.golay[i]);
    cb.golay_wrank[i] = (uint16_t)nww[w]++;
  }
  int acc = 0;
  for (int w = 0; w <= 24; ++w) {
    cb.weight_start[w] = acc;
    acc += nww[w];
  }
  cb.by_weight.resize(kNumGolay);
  cb.wlist_word.resize(kNumGolay);
  cb.wlist_lex.resize(kNumGolay);
  {
    int fill[25];
    std::copy(cb.weight_start, cb.weight_start + 25, fill);
    for (int i = 0; i < kNumGolay; ++i) {
      const int w = __builtin_popcount(cb.golay[i]);
      const int j = fill[w]++;
      cb.by_weight[j] = (uint16_t)i;
      cb.wlist_lex[j] = (uint16_t)i;
      cb.wlist_word[j] = cb.golay[i];
    }
  }
  // Complementary pairs (the all-ones word is in the code, and complementing
  // reverses the lexicographic order, so lex(~c) = 4095 - lex(c)): keep the
  // lighter word of each pair (bit 0 clear when both weigh 12), ordered by
  // weight (0, 8, 12) then lex, so warps of the search run one weight's code.
  cb.plist_word.clear();
  cb.plist_lex.clear();
  for (int w : {0, 8, 12}) {
    for (int i = 0; i < kNumGolay; ++i) {
      const uint32_t c = cb.golay[i];
      if (__builtin_popcount(c) != w || (w == 12 && (c & 1u))) continue;
      if (cb.golay[kNumGolay - 1 - i] != (~c & kFull24)) return fail(LLVQ_ERR_UNSUPPORTED, "golay order broken");
      cb.plist_word.push_back(c);
      cb.plist_lex.push_back((uint16_t)i);
    }
  }
  if ((int)cb.plist_word.size() != kNumGolay / 2) return fail(LLVQ_ERR_UNSUPPORTED, "golay pairs broken");
  cb.cls.assign(n, DevClass{});
  cb.class_start.assign(n, 0);
  u128 cursor = 0;
  cb.min_shell = shell[0];
  cb.max_shell = shell[n - 1];
  for (int k = 0; k < n; ++k) {
    const int* L = leader + (size_t)k * kDim;
    DevClass& c = cb.cls[k];
    c.shell = shell[k];
    c.parity = parity[k];
    if (c.parity != 0 && c.parity != 1) return fail(LLVQ_ERR_INVALID_ARGUMENT, "parity must be 0 (even) or 1 (odd)");
    if (k && shell[k] < shell[k - 1]) return fail(LLVQ_ERR_INVALID_ARGUMENT, "classes must be in shell order");
    if (c.shell < 2 || c.shell - cb.min_shell >= 64) return fail(LLVQ_ERR_UNSUPPORTED, "shell out of range");
    long sq = 0;
    int l1 = 0, nonzero = 0;
    for (int d = 0; d < kDim; ++d) {
      if (L[d] < 0 || L[d] > 127 || (d && L[d] > L[d - 1]))
        return fail(LLVQ_ERR_INVALID_ARGUMENT, "leader must be non-negative and descending");
      if ((L[d] & 1) != c.parity) return fail(LLVQ_ERR_INVALID_ARGUMENT, "leader parity mismatch");
      sq += (long)L[d] * L[d];
      l1 += L[d];
      nonzero += L[d] != 0;
    }
    if (sq != 16L * c.shell) return fail(LLVQ_ERR_INVALID_ARGUMENT, "leader norm is not 16 * shell");
    c.l1 = l1;
    int32_t vt[kMaxVals + 1], mt[kMaxVals + 1];
    if (c.parity == 1) {
      int nv;
      distinct_desc(L, kDim, vt, mt, &nv);
      if (nv > kMaxVals) return fail(LLVQ_ERR_UNSUPPORTED, "too many distinct magnitudes in a class");
      std::copy(vt, vt + nv, c.v0);
      std::copy(mt, mt + nv, c.m0);
      c.nv0 = nv;
      c.nv1 = 0;
      int s[kDim];
      for (int d = 0; d < kDim; ++d) s[d] = (L[d] % 4 == 1) ? L[d] : -L[d];
      std::sort(s, s + kDim);
      for (int d = 0; d < kDim; ++d) c.asc0[d] = (int8_t)s[d];
      const u128 perm = multinomial(c.m0, c.nv0);
      c.golay_count = kNumGolay;
      c.sign_count = 1;
      c.sign_shift = 0;
      c.f1_perm = 1;
      if (perm >> 58) return fail(LLVQ_ERR_UNSUPPORTED, "class too large for 64-bit ranks");
      c.perm_count = (uint64_t)perm;
    } else {
      int f0[kDim], f1[kDim], n0 = 0, n1 = 0;
      for (int d = 0; d < kDim; ++d) {
        if (L[d] % 4 == 2) f1[n1++] = L[d];
        else f0[n0++] = L[d];
      }
      int nv0, nv1;
      distinct_desc(f0, n0, vt, mt, &nv0);
      if (nv0 > kMaxVals) return fail(LLVQ_ERR_UNSUPPORTED, "too many distinct magnitudes");
      std::copy(vt, vt + nv0, c.v0);
      std::copy(mt, mt + nv0, c.m0);
      distinct_desc(f1, n1, vt, mt, &nv1);
      if (nv1 > kMaxVals) return fail(LLVQ_ERR_UNSUPPORTED, "too many distinct magnitudes");
      std::copy(vt, vt + nv1, c.v1);
      std::copy(mt, mt + nv1, c.m1);
      c.nv0 = nv0;
      c.nv1 = nv1;
      for (int i = 0; i < n0; ++i) c.asc0[i] = (int8_t)f0[n0 - 1 - i];
      for (int i = 0; i < n1; ++i) c.asc1[i] = (int8_t)f1[n1 - 1 - i];
      c.even_weight = n1;
      c.required = (l1 % 8) / 4;
      c.golay_count = nww[n1];
      if (!c.golay_count) return fail(LLVQ_ERR_INVALID_ARGUMENT, "even class weight is not a Golay weight");
      if (n1 == 0 && l1 % 8) return fail(LLVQ_ERR_INVALID_ARGUMENT, "empty even class (no valid sign pattern)");
      const int sign_shift = n1 == 0 ? nonzero : nonzero - 1;
      c.sign_shift = sign_shift;
      c.sign_count = 1ull << sign_shift;
      const u128 p0 = multinomial(c.m0, c.nv0), p1 = multinomial(c.m1, c.nv1);
      if ((p0 * p1) >> 58) return fail(LLVQ_ERR_UNSUPPORTED, "class too large for 64-bit ranks");
      if (p1 >> 32) return fail(LLVQ_ERR_UNSUPPORTED, "class too large for 32-bit sub-ranks");
      c.f1_perm = (uint64_t)p1;
      c.perm_count = (uint64_t)(p0 * p1);
    }
    const u128 count = (u128)c.golay_count * (u128)c.sign_count * (u128)c.perm_count;
    c.start = (int64_t)cursor;
    cb.class_start[k] = c.start;
    cursor += count;
    // indices are unsigned 64-bit (stored as the two's-complement int64
    // image above 2^63); all ones stays the invalid index
    if (cursor >= ((u128)1 << 64) - 1) return fail(LLVQ_ERR_UNSUPPORTED, "codebook has 2^64 - 1 or more codewords");
    build_chain(c, L);
  }
  cb.total = (int64_t)(uint64_t)cursor;
  // window constants of the table-driven chains
  float l1max = 0, mg = 0, am = 0;
  for (const DevClass& c : cb.cls) {
    l1max = std::max(l1max, (float)c.l1);
    double a = 0, tot = 0;
    for (int t = 0; t < c.nterms; ++t) {
      const double bound = c.term_kind[t] >= 3 ? 1.0 : (double)c.term_idx[t];
      a += std::fabs((double)c.term_coef[t]) * bound;
      tot += a;
    }
    mg = std::max(mg, (float)(c.shell * (c.nterms + 2)));
    am = std::max(am, (float)tot);
  }
  cb.rt_l1max = l1max;
  cb.rt_mg = mg;
  cb.rt_am = am;
  // generated code for exactly this class list?
  int nspec = 0;
  const SpecEntry* specs = spec_table(&nspec);
  for (int s = 0; s < nspec; ++s) {
    const int* sig = specs[s].sig;
    if (sig[0] != n) continue;
    bool same = true;
    for (int k = 0; k < n && same; ++k) {
      const int* e = sig + 1 + k * (2 + kDim);
      same = e[0] == shell[k] && e[1] == parity[k] && std::equal(e + 2, e + 2 + kDim, leader + (size_t)k * kDim);
    }
    if (same) {
      if (specs[s].angular) {
        if (!cb.spec_ang) cb.spec_ang = &specs[s];
      } else if (!cb.spec) {
        cb.spec = &specs[s];
      }
    }
  }
  return LLVQ_OK;
}

size_t align256(size_t v) { return (v + 255) & ~size_t(255); }

// The decoder's fast path (fully unrolled, 32-bit after the first step) needs
// every part to have at most four distinct values and N < 2^32 from the
// second step of each part on: N only shrinks, so it suffices that N after
// the first step (at most N * c_max / positions) and the N of a part that
// starts after step 0 (the f0 part of a word of weight > 0) are below 2^32.
bool fast_decode_ok(const llvq::DevClass& c) {
  using u128 = unsigned __int128;
  const u128 lim = (u128)1 << 32;
  auto cmax = [](const int32_t* m, int nv) {
    int32_t best = 0;
    for (int j = 0; j < nv; ++j) best = std::max(best, m[j]);
    return (u128)best;
  };
  if (c.nv0 > 4 || c.nv1 > 4) return false;
  if (c.parity) return (u128)c.perm_count * cmax(c.m0, c.nv0) / llvq::kDim < lim;
  const int w = c.even_weight;
  const u128 f1 = c.f1_perm, f0 = c.perm_count / c.f1_perm;
  if (w > 0 && f1 * cmax(c.m1, c.nv1) / (u128)w >= lim) return false;
  if (w == 0) return f0 * cmax(c.m0, c.nv0) / llvq::kDim < lim;
  return f0 < lim;
}

// The decoder's eight-value variant: every part has at most kMaxVals distinct
// values and a multinomial below 2^59, so N * C for any cumulative count C
// (at most 24) stays below 2^64 in its 64-bit steps.
bool wide_decode_ok(const llvq::DevClass& c) {
  using u128 = unsigned __int128;
  const u128 lim = (u128)1 << 59;
  if (c.nv0 > llvq::kMaxVals || c.nv1 > llvq::kMaxVals) return false;
  if (c.parity) return (u128)c.perm_count < lim;
  const u128 f1 = c.f1_perm, f0 = c.perm_count / c.f1_perm;
  return f1 < lim && f0 < lim;
}

// The decoder's tail table (llvq_device.cuh, kTailLen): for every count
// vector over four values summing to 8, its sequences in lexicographic order.
void build_tail_tables(std::vector<uint32_t>& off, std::vector<uint16_t>& seq) {
  using namespace llvq;
  off.assign(kTailKeys, 0);
  seq.clear();
  int cnt[4];
  uint32_t cur = 0;
  auto emit = [&](auto&& self, int pos) -> void {
    if (pos == kTailLen) {
      seq.push_back((uint16_t)cur);
      return;
    }
    for (int v = 0; v < 4; ++v) {
      if (!cnt[v]) continue;
      --cnt[v];
      cur = (cur & ~(3u << (2 * pos))) | ((uint32_t)v << (2 * pos));
      self(self, pos + 1);
      ++cnt[v];
    }
  };
  for (int n0 = 0; n0 <= kTailLen; ++n0)
    for (int n1 = 0; n0 + n1 <= kTailLen; ++n1)
      for (int n2 = 0; n0 + n1 + n2 <= kTailLen; ++n2) {
        const int n3 = kTailLen - n0 - n1 - n2;
        off[n0 * 81 + (n0 + n1) * 9 + (n0 + n1 + n2)] = (uint32_t)seq.size();
        cnt[0] = n0;
        cnt[1] = n1;
        cnt[2] = n2;
        cnt[3] = n3;
        cur = 0;
        emit(emit, 0);
      }
}

int upload(llvq::Codebook& cb, int device) {
  using namespace llvq;
  const size_t n = cb.cls.size();
  size_t off = 0;
  const size_t o_cls = off; off = align256(off + n * sizeof(DevClass));
  const size_t o_start = off; off = align256(off + n * sizeof(int64_t));
  const size_t o_golay = off; off = align256(off + kNumGolay * sizeof(uint32_t));
  const size_t o_wrank = off; off = align256(off + kNumGolay * sizeof(uint16_t));
  const size_t o_wword = off; off = align256(off + kNumGolay * sizeof(uint32_t));
  const size_t o_wlex = off; off = align256(off + kNumGolay * sizeof(uint16_t));
  const size_t o_byw = off; off = align256(off + kNumGolay * sizeof(uint16_t));
  const size_t o_dcls = off; off = align256(off + n * sizeof(DecodeClass));
  const size_t o_bucket = off; off = align256(off + (kBuckets + 1) * sizeof(uint16_t));
  const size_t o_pword = off; off = align256(off + (kNumGolay / 2) * sizeof(uint32_t));
  const size_t o_plex = off; off = align256(off + (kNumGolay / 2) * sizeof(uint16_t));
  const size_t o_toff = off; off = align256(off + kTailKeys * sizeof(uint32_t));
  const size_t o_tseq = off; off = align256(off + kTailSeqs * sizeof(uint16_t));
  const TabHost& tb = cb.tab;
  const size_t o_tstate = off; off = align256(off + tb.state.size() * sizeof(uint4));
  const size_t o_tcrec = off; off = align256(off + tb.crec.size() * sizeof(uint4));
  const size_t o_tentry = off; off = align256(off + tb.entry.size() * sizeof(uint4));
  const size_t o_tslot = off; off = align256(off + tb.slot.size() * sizeof(uint4));
  const size_t o_ttail = off; off = align256(off + tb.tail.size() * sizeof(unsigned long long));
  const size_t o_ttail2 = off; off = align256(off + tb.tail2.size() * sizeof(uint32_t));
  const size_t o_texp2 = off; off = align256(off + tb.expand2.size() * sizeof(uint32_t));
  std::vector<unsigned char> host(off, 0);
  if (tb.ok) {
    std::memcpy(host.data() + o_tstate, tb.state.data(), tb.state.size() * sizeof(uint4));
    std::memcpy(host.data() + o_tcrec, tb.crec.data(), tb.crec.size() * sizeof(uint4));
    std::memcpy(host.data() + o_tentry, tb.entry.data(), tb.entry.size() * sizeof(uint4));
    std::memcpy(host.data() + o_tslot, tb.slot.data(), tb.slot.size() * sizeof(uint4));
    std::memcpy(host.data() + o_ttail, tb.tail.data(), tb.tail.size() * sizeof(unsigned long long));
    std::memcpy(host.data() + o_ttail2, tb.tail2.data(), tb.tail2.size() * sizeof(uint32_t));
    std::memcpy(host.data() + o_texp2, tb.expand2.data(), tb.expand2.size() * sizeof(uint32_t));
  }
  {
    std::vector<DecodeClass> dc(n);
    for (size_t k = 0; k < n; ++k) {
      const DevClass& c = cb.cls[k];
      DecodeClass& d = dc[k];
      d.start = c.start;
      d.perm_count = c.perm_count;
      d.magic_perm = ~0ull / c.perm_count;
      d.f0_perm = c.perm_count / c.f1_perm;
      d.f1_perm = (uint32_t)c.f1_perm;
      d.magic_f1 = ~0ull / c.f1_perm;
      d.meta = (uint32_t)c.parity | ((uint32_t)c.even_weight << 1) | ((uint32_t)c.sign_shift << 6) |
               ((uint32_t)c.nv0 << 11) | ((uint32_t)c.nv1 << 15) | ((uint32_t)c.required << 19) |
               (fast_decode_ok(c) ? kMetaFast | kMetaWide : 0u) | (wide_decode_ok(c) ? kMetaWide : 0u);
      d.golay_base = (uint32_t)cb.weight_start[c.even_weight];
      d.pad = 0;
      d.v0 = d.m0 = d.v1 = d.m1 = 0;
      for (int j = 0; j < kMaxVals; ++j) {
        d.v0 |= (uint64_t)(uint8_t)(j < c.nv0 ? c.v0[j] : 0) << (8 * j);
        d.m0 |= (uint64_t)(uint8_t)(j < c.nv0 ? c.m0[j] : 0) << (8 * j);
        d.v1 |= (uint64_t)(uint8_t)(j < c.nv1 ? c.v1[j] : 0) << (8 * j);
        d.m1 |= (uint64_t)(uint8_t)(j < c.nv1 ? c.m1[j] : 0) << (8 * j);
      }
    }
    std::memcpy(host.data() + o_dcls, dc.data(), n * sizeof(DecodeClass));
    // owner class of each bucket's lowest index (the last class past the end)
    std::vector<uint16_t> bucket(kBuckets + 1);
    for (int b = 0; b <= kBuckets; ++b) {
      const uint64_t lo = bucket_low(b);
      bucket[b] = (uint16_t)(lo >= (uint64_t)cb.total ? n - 1
                                                      : find_class(cb.class_start.data(), (int)n, (int64_t)lo));
    }
    std::memcpy(host.data() + o_bucket, bucket.data(), bucket.size() * sizeof(uint16_t));
  }
  std::memcpy(host.data() + o_cls, cb.cls.data(), n * sizeof(DevClass));
  std::memcpy(host.data() + o_start, cb.class_start.data(), n * sizeof(int64_t));
  std::memcpy(host.data() + o_golay, cb.golay.data(), kNumGolay * sizeof(uint32_t));
  std::memcpy(host.data() + o_wrank, cb.golay_wrank.data(), kNumGolay * sizeof(uint16_t));
  std::memcpy(host.data() + o_wword, cb.wlist_word.data(), kNumGolay * sizeof(uint32_t));
  std::memcpy(host.data() + o_wlex, cb.wlist_lex.data(), kNumGolay * sizeof(uint16_t));
  std::memcpy(host.data() + o_byw, cb.by_weight.data(), kNumGolay * sizeof(uint16_t));
  std::memcpy(host.data() + o_pword, cb.plist_word.data(), (kNumGolay / 2) * sizeof(uint32_t));
  std::memcpy(host.data() + o_plex, cb.plist_lex.data(), (kNumGolay / 2) * sizeof(uint16_t));
  {
    std::vector<uint32_t> toff;
    std::vector<uint16_t> tseq;
    build_tail_tables(toff, tseq);
    if ((int)tseq.size() != kTailSeqs) return fail(LLVQ_ERR_UNSUPPORTED, "tail table broken");
    std::memcpy(host.data() + o_toff, toff.data(), kTailKeys * sizeof(uint32_t));
    std::memcpy(host.data() + o_tseq, tseq.data(), kTailSeqs * sizeof(uint16_t));
  }
  int prev = -1;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (prev != device && (e = cudaSetDevice(device)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  void* mem = nullptr;
  e = cudaMalloc(&mem, off);
  if (e == cudaSuccess) e = cudaMemcpy(mem, host.data(), off, cudaMemcpyHostToDevice);
  if (prev != device) cudaSetDevice(prev);
  if (e != cudaSuccess) {
    if (mem) cudaFree(mem);
    return e == cudaErrorMemoryAllocation ? fail(LLVQ_ERR_OUT_OF_MEMORY, "codebook tables") : cuda_fail(e, "upload");
  }
  unsigned char* base = static_cast<unsigned char*>(mem);
  cb.dev_alloc = mem;
  cb.dev_bytes = off;
  cb.device = device;
  DevBook& d = cb.dev;
  d.cls = reinterpret_cast<const DevClass*>(base + o_cls);
  d.class_start = reinterpret_cast<const int64_t*>(base + o_start);
  d.golay = reinterpret_cast<const uint32_t*>(base + o_golay);
  d.golay_wrank = reinterpret_cast<const uint16_t*>(base + o_wrank);
  d.wlist_word = reinterpret_cast<const uint32_t*>(base + o_wword);
  d.wlist_lex = reinterpret_cast<const uint16_t*>(base + o_wlex);
  d.by_weight = reinterpret_cast<const uint16_t*>(base + o_byw);
  d.dcls = reinterpret_cast<const DecodeClass*>(base + o_dcls);
  d.bucket = reinterpret_cast<const uint16_t*>(base + o_bucket);
  d.plist_word = reinterpret_cast<const uint32_t*>(base + o_pword);
  d.plist_lex = reinterpret_cast<const uint16_t*>(base + o_plex);
  d.tail_off = reinterpret_cast<const uint32_t*>(base + o_toff);
  d.tail_seq = reinterpret_cast<const uint16_t*>(base + o_tseq);
  d.tab = TabView{};
  if (tb.ok) {
    d.tab.state = reinterpret_cast<const uint4*>(base + o_tstate);
    d.tab.crec = reinterpret_cast<const uint4*>(base + o_tcrec);
    d.tab.entry = reinterpret_cast<const uint4*>(base + o_tentry);
    d.tab.slot = reinterpret_cast<const uint4*>(base + o_tslot);
    d.tab.tail = reinterpret_cast<const unsigned long long*>(base + o_ttail);
    d.tab.tail2 = reinterpret_cast<const uint32_t*>(base + o_ttail2);
    d.tab.expand2 = reinterpret_cast<const uint4*>(base + o_texp2);
    d.tab.n_states = (int)(tb.state.size() / 2);
    d.tab.max_searches = tb.max_searches;
  }
  std::copy(cb.weight_start, cb.weight_start + 25, d.weight_start);
  d.n_classes = (int32_t)n;
  d.min_shell = cb.min_shell;
  d.max_shell = cb.max_shell;
  d.total = cb.total;
  return LLVQ_OK;
}

// Decoded-weight staging of the large-batch GEMM: up to 256 MiB, so the
// Llama-size matrices (up to 16k x 8k) are decoded in one chunk and every
// tile of the matrix is available to the SMs at once.
constexpr int64_t kGemmStagingBudget = 256ll << 20;

// Runs `fn` with the codebook's device current, restoring the caller's device.
template <class F>
int on_device(const llvq_codebook* h, F&& fn) {
  if (!h) return fail(LLVQ_ERR_INVALID_ARGUMENT, "null codebook");
  if (h->cb.device < 0) return fail(LLVQ_ERR_INVALID_ARGUMENT, "host-only codebook has no device tables");
  int prev = -1;
  cudaError_t e = cudaGetDevice(&prev);
  if (e != cudaSuccess) return cuda_fail(e, "cudaGetDevice");
  if (prev != h->cb.device && (e = cudaSetDevice(h->cb.device)) != cudaSuccess) return cuda_fail(e, "cudaSetDevice");
  e = fn();
  if (prev != h->cb.device) cudaSetDevice(prev);
  if (e != cudaSuccess) return cuda_fail(e, "kernel launch");
  return LLVQ_OK;
}

}  // namespace

extern "C" {

int llvq_codebook_create(int32_t n_classes, const int32_t* shell, const int32_t* parity, const int32_t* leader,
                         int device, llvq_codebook** out) {
  if (!out) return fail(LLVQ_ERR_INVALID_ARGUMENT, "null output pointer");
  *out = nullptr;
  llvq_codebook* h = new (std::nothrow) llvq_codebook();
  if (!h) return fail(LLVQ_ERR_OUT_OF_MEMORY, "codebook");
  int st = build(h->cb, n_classes, shell, parity, leader);
  if (st == LLVQ_OK && !llvq::build_decode_tables(h->cb, h->cb.tab, &h->cb.tab_why) && h->cb.tab_why.empty())
    h->cb.tab_why = "tables not built";
  if (st == LLVQ_OK && device >= 0) st = upload(h->cb, device);
  if (st != LLVQ_OK) {
    delete h;
    return st;
  }
  *out = h;
  return LLVQ_OK;
}

void llvq_codebook_destroy(llvq_codebook* h) {
  if (!h) return;
  if (h->cb.dev_alloc) {
    int prev = -1;
    cudaGetDevice(&prev);
    if (prev != h->cb.device) cudaSetDevice(h->cb.device);
    cudaFree(h->cb.dev_alloc);
    if (prev != h->cb.device && prev >= 0) cudaSetDevice(prev);
  }
  delete h;
}

int llvq_codeword_batch_host(const llvq_codebook* h, const int64_t* indices, int64_t n, int32_t* out, int64_t* bad) {
  if (!h) return fail(LLVQ_ERR_INVALID_ARGUMENT, "null codebook");
  if (n < 0 || (n > 0 && (!indices || !out))) return fail(LLVQ_ERR_INVALID_ARGUMENT, "bad codeword arguments");
  if (!h->cb.tab.ok) return fail(LLVQ_ERR_UNSUPPORTED, "codebook has no decoder tables: " + h->cb.tab_why);
  int64_t nbad = 0;
  for (int64_t i = 0; i < n; ++i)
    if (!llvq::decode_index_tables_host(h->cb, indices[i], out + i * llvq::kDim)) ++nbad;
  if (bad) *bad = nbad;
  return LLVQ_OK;
}

int llvq_codebook_tables(const llvq_codebook* h, int32_t* tabulated, int64_t* table_bytes, int32_t* max_lookups) {
  if (!h) return fail(LLVQ_ERR_INVALID_ARGUMENT, "null codebook");
  const llvq::TabHost& t = h->cb.tab;
  if (tabulated) *tabulated = t.ok ? 1 : 0;
  if (table_bytes)
    *table_bytes = (int64_t)(t.state.size() * 16 + t.crec.size() * 16 + t.entry.size() * 16 + t.slot.size() * 16 +
                             t.tail.size() * 8 + t.tail2.size() * 4 + t.expand2.size() * 4);
  if (max_lookups) *max_lookups = t.max_searches + 2;  // searches, then one tail per part
  return LLVQ_OK;
}

int llvq_codebook_info(const llvq_codebook* h, int64_t* total_count, int32_t* n_classes, int32_t* min_shell,
                       int32_t* max_shell, int32_t* specialized) {
  if (!h) return fail(LLVQ_ERR_INVALID_ARGUMENT, "null codebook");
  if (total_count) *total_count = h->cb.total;
  if (n_classes) *n_classes = (int32_t)h->cb.cls.size();
  if (min_shell) *min_shell = h->cb.min_shell;
  if (max_shell) *max_shell = h->cb.max_shell;
  if (specialized) *specialized = h->cb.spec != nullptr;
  return LLVQ_OK;
}

int llvq_quantize_ex(const llvq_codebook* h, const float* x, int64_t n, int64_t* indices, int64_t* best_pair,
                     float* best_score, uint32_t flags, void* stream) {
  if (n < 0 || (n > 0 && (!x || !indices || !best_pair || !best_score)))
    return fail(LLVQ_ERR_INVALID_ARGUMENT, "bad quantize arguments");
  return on_device(h, [&] {
    return llvq::quantize_launch(h->cb, x, n, reinterpret_cast<long long*>(indices),
                                 reinterpret_cast<long long*>(best_pair), best_score, (cudaStream_t)stream,
                                 (flags & LLVQ_FLAG_TABLE_DRIVEN) != 0);
  });
}

int llvq_quantize_gain(const llvq_codebook* h, const float* x, int64_t n, int64_t* indices, int64_t* best_pair,
                       float* best_score, const double* gain_thresholds, int32_t gain_bits, const float* row_sigma,
                       int64_t blocks_per_row, int32_t* gain_index, uint32_t flags, void* stream) {
  const bool pack = (flags & LLVQ_GAIN_PACK) != 0, angular = (flags & LLVQ_GAIN_ANGULAR) != 0;
  if (n < 0 || (n > 0 && (!x || !indices || !best_pair || !best_score || !gain_thresholds)))
    return fail(LLVQ_ERR_INVALID_ARGUMENT, "bad quantize arguments");
  if (gain_bits < 1 || gain_bits > 16 || (row_sigma && blocks_per_row <= 0))
    return fail(LLVQ_ERR_INVALID_ARGUMENT, "gain code: need 1 <= gain_bits <= 16 and blocks_per_row > 0");
  if (!h) return fail(LLVQ_ERR_INVALID_ARGUMENT, "null codebook");
  if (pack && ((uint64_t)h->cb.total > 1 ? 64 - __builtin_clzll((unsigned long long)h->cb.total - 1ull) : 1) +
                      gain_bits > 63)
    return fail(LLVQ_ERR_UNSUPPORTED, "packed shape-gain index exceeds 63 bits");
  llvq::GainCode gc;
  gc.thr = gain_thresholds;
  gc.nthr = (1 << gain_bits) - 1;
  gc.bits = gain_bits;
  gc.sigma = row_sigma;
  gc.bpr = row_sigma ? blocks_per_row : 1;
  gc.gain_out = gain_index;
  gc.pack = pack;
  if (angular && !h->cb.spec_ang)
    return fail(LLVQ_ERR_UNSUPPORTED, "no angular (multi-shell shape) search code for this class list");
  return on_device(h, [&] {
    return llvq::quantize_launch(h->cb, x, n, reinterpret_cast<long long*>(indices),
                                 reinterpret_cast<long long*>(best_pair), best_score, (cudaStream_t)stream, false, gc,
                                 angular);
  });
}

int llvq_quantize(const llvq_codebook* h, const float* x, int64_t n, int64_t* indices, int64_t* best_pair,
                  float* best_score, void* stream) {
  return llvq_quantize_ex(h, x, n, indices, best_pair, best_score, 0u, stream);
}

int llvq_dequantize_lattice(const llvq_codebook* h, const int64_t* indices, int64_t n, int64_t* out,
                            int32_t* error_count, void* stream) {
  if (n < 0 || (n > 0 && (!indices || !out))) return fail(LLVQ_ERR_INVALID_ARGUMENT, "bad dequantize arguments");
  return on_device(h, [&] {
    return llvq::dequantize_launch(h->cb, {indices, 8}, n, out, 0, nullptr, 1, error_count, (cudaStream_t)stream);
  });
}

int llvq_dequantize(const llvq_codebook* h, const int64_t* indices, int64_t n, float* out, int32_t kind,
                    int32_t* error_count, void* stream) {
  if (n < 0 || (n > 0 && (!indices || !out))) return fail(LLVQ_ERR_INVALID_ARGUMENT, "bad dequantize arguments");
  if (kind != LLVQ_OUT_F32 && kind != LLVQ_OUT_F32_DOUBLE) return fail(LLVQ_ERR_INVALID_ARGUMENT, "bad output kind");
  return on_device(h, [&] {
    return llvq::dequantize_launch(h->cb, {indices, 8}, n, out, kind, nullptr, 1, error_count, (cudaStream_t)stream);
  });
}

int llvq_dequantize_bf16(const llvq_codebook* h, const int64_t* indices, int64_t n, const uint16_t* row_scale_f16,
                         int64_t blocks_per_row, uint16_t* out_bf16, int32_t* error_count, void* stream) {
  if (n < 0 || blocks_per_row <= 0 || (n > 0 && (!indices || !out_bf16 || !row_scale_f16)))
    return fail(LLVQ_ERR_INVALID_ARGUMENT, "bad dequantize arguments");
  return on_device(h, [&] {
    return llvq::dequantize_launch(h->cb, {indices, 8}, n, out_bf16, 3, row_scale_f16, blocks_per_row, error_count,
                                   (cudaStream_t)stream);
  });
}

}  // extern "C"

namespace {

// Shared by llvq_gemm and llvq_gemm_packed.
int gemm_impl(const llvq_codebook* h, llvq::IndexSource src, int64_t n_out, int64_t blocks_per_row,
              const uint16_t* row_scale_f16, const uint16_t* a_bf16, int64_t m, int64_t k, float* y,
              int32_t* error_flag, void* stream) {
  if (m < 0 || n_out < 0 || blocks_per_row <= 0 || k <= 0 || k % 8 || k > 24 * blocks_per_row)
    return fail(LLVQ_ERR_INVALID_ARGUMENT, "gemm shapes: need k % 8 == 0 and 0 < k <= 24 * blocks_per_row");
  if (m > 0 && n_out > 0 && (!src.ptr || !a_bf16 || !y || (reinterpret_cast<uintptr_t>(a_bf16) & 15)))
    return fail(LLVQ_ERR_INVALID_ARGUMENT, "gemm pointers: null, or activations not 16-byte aligned");
  if (m > (int64_t)INT32_MAX || n_out > (int64_t)INT32_MAX || blocks_per_row > (int64_t)INT32_MAX)
    return fail(LLVQ_ERR_INVALID_ARGUMENT, "gemm shapes exceed 32-bit extents");
  if (m == 0 || n_out == 0) return LLVQ_OK;
  return on_device(h, [&] {
    if (m <= llvq::kGemvMaxM)  // decoded in registers: no staging
      return llvq::gemv_decode_launch(h->cb, src, n_out, blocks_per_row, row_scale_f16, a_bf16, m, k, y,
                                      (cudaStream_t)stream);
    if (llvq::gemm_fused_ok(h->cb, m)) {  // decoded into shared memory: a small partial-sum workspace only
      int sms = 0;
      cudaError_t e = llvq::device_sms(&sms);
      if (e != cudaSuccess) return e;
      const int64_t bytes = llvq::gemm_fused_workspace_bytes(n_out, blocks_per_row, m, sms);
      cudaMemPool_t pool;
      e = llvq::gemm_staging_pool(&pool);
      if (e != cudaSuccess) return e;
      void* ws = nullptr;
      e = cudaMallocFromPoolAsync(&ws, (size_t)bytes, pool, (cudaStream_t)stream);
      if (e != cudaSuccess) return e;
      e = llvq::gemm_fused_launch(h->cb, src, n_out, blocks_per_row, row_scale_f16, a_bf16, m, k, y, error_flag, ws,
                                  bytes, sms, (cudaStream_t)stream);
      const cudaError_t ef = cudaFreeAsync(ws, (cudaStream_t)stream);
      return e != cudaSuccess ? e : ef;
    }
    // stream-ordered staging buffer from the library's pool, released on the
    // same stream after the GEMM
    const int64_t bytes = llvq::gemm_staging_bytes(n_out, blocks_per_row, kGemmStagingBudget);
    cudaMemPool_t pool;
    cudaError_t e = llvq::gemm_staging_pool(&pool);
    if (e != cudaSuccess) return e;
    void* staging = nullptr;
    e = cudaMallocFromPoolAsync(&staging, (size_t)bytes, pool, (cudaStream_t)stream);
    if (e != cudaSuccess) return e;
    e = llvq::gemm_staged_launch(h->cb, src, n_out, blocks_per_row, row_scale_f16, a_bf16, m, k, y, error_flag,
                                 staging, bytes, (cudaStream_t)stream);
    const cudaError_t ef = cudaFreeAsync(staging, (cudaStream_t)stream);
    return e != cudaSuccess ? e : ef;
  });
}

// Packed indices of `index_bytes` bytes must leave the all-ones value free
// for the invalid index.
int check_index_bytes(const llvq_codebook* h, int32_t index_bytes) {
  if (!h) return fail(LLVQ_ERR_INVALID_ARGUMENT, "null codebook");
  if (index_bytes < 1 || index_bytes > 8) return fail(LLVQ_ERR_INVALID_ARGUMENT, "index_bytes must be 1..8");
  if (index_bytes < 8 && (uint64_t)h->cb.total > (~0ull >> (64 - 8 * index_bytes)))
    return fail(LLVQ_ERR_INVALID_ARGUMENT, "index_bytes too small for this codebook's index range");
  return LLVQ_OK;
}

}  // namespace

extern "C" {

int llvq_gemm(const llvq_codebook* h, const int64_t* indices, int64_t n_out, int64_t blocks_per_row,
              const uint16_t* row_scale_f16, const uint16_t* a_bf16, int64_t m, int64_t k, float* y,
              int32_t* error_flag, void* stream) {
  return gemm_impl(h, {indices, 8}, n_out, blocks_per_row, row_scale_f16, a_bf16, m, k, y, error_flag, stream);
}

int llvq_gemm_packed(const llvq_codebook* h, const uint8_t* packed, int32_t index_bytes, int64_t n_out,
                     int64_t blocks_per_row, const uint16_t* row_scale_f16, const uint16_t* a_bf16, int64_t m,
                     int64_t k, float* y, int32_t* error_flag, void* stream) {
  const int st = check_index_bytes(h, index_bytes);
  if (st != LLVQ_OK) return st;
  return gemm_impl(h, {packed, index_bytes}, n_out, blocks_per_row, row_scale_f16, a_bf16, m, k, y, error_flag,
                   stream);
}

int llvq_dequantize_packed(const llvq_codebook* h, const uint8_t* packed, int32_t index_bytes, int64_t n, void* out,
                           int32_t kind, const uint16_t* row_scale_f16, int64_t blocks_per_row,
                           int32_t* error_count, void* stream) {
  const int st = check_index_bytes(h, index_bytes);
  if (st != LLVQ_OK) return st;
  if (n < 0 || (n > 0 && (!packed || !out))) return fail(LLVQ_ERR_INVALID_ARGUMENT, "bad dequantize arguments");
  if (kind < LLVQ_OUT_INT64 || kind > LLVQ_OUT_BF16_ROWSCALE) return fail(LLVQ_ERR_INVALID_ARGUMENT, "bad output kind");
  if (kind == LLVQ_OUT_BF16_ROWSCALE && (blocks_per_row <= 0 || (n > 0 && !row_scale_f16)))
    return fail(LLVQ_ERR_INVALID_ARGUMENT, "bf16 output needs row scales and blocks_per_row > 0");
  return on_device(h, [&] {
    return llvq::dequantize_launch(h->cb, {packed, index_bytes}, n, out, kind, row_scale_f16,
                                   kind == LLVQ_OUT_BF16_ROWSCALE ? blocks_per_row : 1, error_count,
                                   (cudaStream_t)stream);
  });
}

int llvq_pack_indices(const int64_t* indices, int64_t n, int32_t index_bytes, uint8_t* packed, int32_t* error_count,
                      void* stream) {
  if (index_bytes < 1 || index_bytes > 8) return fail(LLVQ_ERR_INVALID_ARGUMENT, "index_bytes must be 1..8");
  if (n < 0 || (n > 0 && (!indices || !packed))) return fail(LLVQ_ERR_INVALID_ARGUMENT, "bad pack arguments");
  const cudaError_t e = llvq::pack_indices_launch(indices, n, index_bytes, packed, error_count, (cudaStream_t)stream);
  return e == cudaSuccess ? LLVQ_OK : cuda_fail(e, "pack launch");
}

int llvq_unpack_indices(const uint8_t* packed, int64_t n, int32_t index_bytes, int64_t* indices, void* stream) {
  if (index_bytes < 1 || index_bytes > 8) return fail(LLVQ_ERR_INVALID_ARGUMENT, "index_bytes must be 1..8");
  if (n < 0 || (n > 0 && (!indices || !packed))) return fail(LLVQ_ERR_INVALID_ARGUMENT, "bad unpack arguments");
  const cudaError_t e = llvq::unpack_indices_launch(packed, n, index_bytes, indices, (cudaStream_t)stream);
  return e == cudaSuccess ? LLVQ_OK : cuda_fail(e, "unpack launch");
}

static_assert(LLVQ_GEMM_NOALLOC_STAGING_BYTES == llvq::kNoAllocStagingBytes, "staging size mismatch");
static_assert(128 * ((24 * LLVQ_GEMM_NOALLOC_MAX_BLOCKS_PER_ROW + 63) / 64 * 64) * 2 <= llvq::kNoAllocStagingBytes,
              "one 128-row tile of the widest rows must fit the static staging buffer");

int llvq_gemm_noalloc(const llvq_codebook* h, const int64_t* indices, int64_t n_out, int64_t blocks_per_row,
                      const uint16_t* row_scale_f16, const uint16_t* a_bf16, int64_t m, int64_t k, float* y,
                      int32_t* error_flag, void* stream) {
  if (m < 0 || n_out < 0 || blocks_per_row <= 0 || k <= 0 || k % 8 || k > 24 * blocks_per_row)
    return fail(LLVQ_ERR_INVALID_ARGUMENT, "gemm shapes: need k % 8 == 0 and 0 < k <= 24 * blocks_per_row");
  if (m > llvq::kGemvMaxM && blocks_per_row > LLVQ_GEMM_NOALLOC_MAX_BLOCKS_PER_ROW)
    return fail(LLVQ_ERR_INVALID_ARGUMENT,
                "gemm_noalloc: blocks_per_row > 2730 (rows wider than 65536 columns) does not fit the 16 MiB "
                "static staging buffer when m > 4; use llvq_gemm");
  if (m > 0 && n_out > 0 && (!indices || !a_bf16 || !y || (reinterpret_cast<uintptr_t>(a_bf16) & 15)))
    return fail(LLVQ_ERR_INVALID_ARGUMENT, "gemm pointers: null, or activations not 16-byte aligned");
  if (m > (int64_t)INT32_MAX || n_out > (int64_t)INT32_MAX)
    return fail(LLVQ_ERR_INVALID_ARGUMENT, "gemm shapes exceed 32-bit extents");
  return on_device(h, [&] {  // setup runs even for empty shapes, so a first empty call prepares the device
    void* staging = nullptr;
    cudaError_t e = llvq::noalloc_staging(&staging);  // first call on a device: loads the array's module
    if (e != cudaSuccess) return e;
    if (llvq::gemm_fused_ok(h->cb, m)) {  // the fused path's partial sums fit the array: use it as workspace
      int sms = 0;
      e = llvq::device_sms(&sms);
      if (e != cudaSuccess) return e;
      if (llvq::gemm_fused_workspace_bytes(n_out, blocks_per_row, m, sms) <= llvq::kNoAllocStagingBytes)
        return llvq::gemm_fused_launch(h->cb, {indices, 8}, n_out, blocks_per_row, row_scale_f16, a_bf16, m, k, y,
                                       error_flag, staging, llvq::kNoAllocStagingBytes, sms, (cudaStream_t)stream);
    }
    return llvq::gemm_staged_launch(h->cb, {indices, 8}, n_out, blocks_per_row, row_scale_f16, a_bf16, m, k, y,
                                    error_flag, staging, llvq::kNoAllocStagingBytes, (cudaStream_t)stream);
  });
}

int llvq_rotate_scale(const uint16_t* in_f16, int64_t rows, int64_t cols, int64_t ld, int32_t block,
                      const int8_t* signs, float* out, uint16_t* row_scale_out, void* stream) {
  if (rows < 0 || cols <= 0 || ld < cols || block < 2 || block > 4096 || (block & (block - 1)) || cols % block ||
      cols * 4 > 200 * 1024)
    return fail(LLVQ_ERR_INVALID_ARGUMENT, "rotate_scale: block a power of two <= 4096 dividing cols, ld >= cols, "
                                           "cols <= 51200");
  if (rows > 0 && (!in_f16 || !signs || !out || !row_scale_out))
    return fail(LLVQ_ERR_INVALID_ARGUMENT, "rotate_scale: null pointer");
  const cudaError_t e = llvq::rotate_scale_launch(in_f16, rows, cols, ld, block, signs, out, row_scale_out,
                                                  (cudaStream_t)stream);
  return e == cudaSuccess ? LLVQ_OK : cuda_fail(e, "rotate_scale launch");
}

int llvq_hadamard_ex(const void* in, int32_t in_type, void* out, int32_t out_type, int64_t rows, int64_t cols,
                     int32_t block, const int8_t* signs, int32_t inverse, void* stream) {
  if (rows < 0 || cols <= 0 || block < 1 || block > 4096 || (block & (block - 1)) || cols % block)
    return fail(LLVQ_ERR_INVALID_ARGUMENT, "hadamard: block must be a power of two <= 4096 dividing cols");
  if (in_type < LLVQ_DT_F32 || in_type > LLVQ_DT_BF16 || (out_type != LLVQ_DT_F32 && out_type != LLVQ_DT_BF16))
    return fail(LLVQ_ERR_INVALID_ARGUMENT, "hadamard: bad element type");
  if (rows > 0 && (!in || !out || !signs)) return fail(LLVQ_ERR_INVALID_ARGUMENT, "hadamard: null pointer");
  const cudaError_t e = llvq::hadamard_launch(in, in_type, out, out_type, rows, cols, block, signs, inverse,
                                              (cudaStream_t)stream);
  return e == cudaSuccess ? LLVQ_OK : cuda_fail(e, "hadamard launch");
}

int llvq_hadamard(const void* in, int32_t in_is_half, float* out, int64_t rows, int64_t cols, int32_t block,
                  const int8_t* signs, int32_t inverse, void* stream) {
  return llvq_hadamard_ex(in, in_is_half ? LLVQ_DT_F16 : LLVQ_DT_F32, out, LLVQ_DT_F32, rows, cols, block, signs,
                          inverse, stream);
}

int llvq_codeword_host(const llvq_codebook* h, int64_t index, int32_t* out24) {
  if (!h || !out24) return fail(LLVQ_ERR_INVALID_ARGUMENT, "null argument");
  const llvq::Codebook& cb = h->cb;
  if ((uint64_t)index >= (uint64_t)cb.total) return fail(LLVQ_ERR_INDEX_RANGE, "index outside codebook range");
  const int k = llvq::find_class(cb.class_start.data(), (int)cb.cls.size(), index);
  const llvq::DevClass& c = cb.cls[k];
  int y[llvq::kDim];
  const int wbase = cb.weight_start[c.even_weight];
  const bool ok = llvq::unrank_codeword(
      c, (uint64_t)index - (uint64_t)c.start,
      [&](int g) { return c.parity ? cb.golay[g] : cb.golay[cb.by_weight[wbase + g]]; }, y);
  if (!ok) return fail(LLVQ_ERR_INDEX_RANGE, "index does not decode");
  for (int d = 0; d < llvq::kDim; ++d) out24[d] = y[d];
  return LLVQ_OK;
}

int llvq_encode_host(const llvq_codebook* h, const int32_t* v, int64_t* index) {
  using namespace llvq;
  if (!h || !v || !index) return fail(LLVQ_ERR_INVALID_ARGUMENT, "null argument");
  const Codebook& cb = h->cb;
  long sq = 0;
  int nodd = 0;
  int y[kDim], key[kDim];
  for (int d = 0; d < kDim; ++d) {
    y[d] = v[d];
    sq += (long)y[d] * y[d];
    nodd += (y[d] & 1) != 0;
    key[d] = y[d] < 0 ? -y[d] : y[d];
  }
  if (sq % 16) return fail(LLVQ_ERR_NOT_A_CODEWORD, "squared norm is not a Leech shell norm");
  const int shell = (int)(sq / 16);
  if (shell < cb.min_shell || shell > cb.max_shell) return fail(LLVQ_ERR_NOT_A_CODEWORD, "shell outside codebook");
  if (nodd != 0 && nodd != kDim) return fail(LLVQ_ERR_NOT_A_CODEWORD, "coordinates must be all even or all odd");
  const int parity = nodd ? 1 : 0;
  std::sort(key, key + kDim, [](int a, int b) { return a > b; });
  uint32_t word = 0;
  for (int d = 0; d < kDim; ++d) {
    const int r = ((y[d] % 4) + 4) % 4;
    const int a = y[d] < 0 ? -y[d] : y[d];
    if (parity ? r == 3 : a % 4 == 2) word |= 1u << d;
  }
  const auto it = std::find(cb.golay.begin(), cb.golay.end(), word);
  if (it == cb.golay.end()) return fail(LLVQ_ERR_NOT_A_CODEWORD, "congruence pattern is not a Golay codeword");
  const int lex = (int)(it - cb.golay.begin());
  for (size_t k = 0; k < cb.cls.size(); ++k) {
    const DevClass& c = cb.cls[k];
    if (c.shell != shell || c.parity != parity) continue;
    int lead[kDim], n0 = 0;
    if (parity) {
      for (int j = 0; j < c.nv0; ++j)
        for (int t = 0; t < c.m0[j]; ++t) lead[n0++] = c.v0[j];
    } else {
      for (int i = 0; i < c.even_weight; ++i) lead[n0++] = c.asc1[i];
      for (int i = 0; i < kDim - c.even_weight; ++i) lead[n0++] = c.asc0[i];
      std::sort(lead, lead + kDim, [](int a, int b) { return a > b; });
    }
    if (!std::equal(lead, lead + kDim, key)) continue;
    if (!parity && __builtin_popcount(word) != c.even_weight)
      return fail(LLVQ_ERR_NOT_A_CODEWORD, "Golay codeword is not compatible with this class");
    const int choice = parity ? lex : (int)cb.golay_wrank[lex];
    const int64_t r = rank_codeword(c, y, word, choice);
    if (r == -1) return fail(LLVQ_ERR_NOT_A_CODEWORD, "sign pattern is outside the class");
    *index = r;
    return LLVQ_OK;
  }
  return fail(LLVQ_ERR_NOT_A_CODEWORD, "no class matches this leader");
}

const char* llvq_status_string(int status) {
  switch (status) {
    case LLVQ_OK: return "ok";
    case LLVQ_ERR_INVALID_ARGUMENT: return "invalid argument";
    case LLVQ_ERR_CUDA: return "CUDA error";
    case LLVQ_ERR_UNSUPPORTED: return "unsupported codebook";
    case LLVQ_ERR_OUT_OF_MEMORY: return "out of memory";
    case LLVQ_ERR_INDEX_RANGE: return "index out of range";
    case LLVQ_ERR_NOT_A_CODEWORD: return "not a codeword";
    default: return "unknown status";
  }
}

const char* llvq_last_error(void) { return g_last_error.c_str(); }

int llvq_version(void) { return 1; }

}  // extern "C"
