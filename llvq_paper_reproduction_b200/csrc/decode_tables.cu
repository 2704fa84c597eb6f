// Host builder of the table-driven decoder's tables (llvq_tables.cuh) and the
// host batch decoder that uses them.
//
// States are count vectors of a class part's values still to place (value
// index j = the j-th largest value of the part, the order in which the
// reference's multiset rank tries values, impl/leech_lattice_vector_quantizer.py
// :870-889).  From every class part's full multiset the builder walks the
// states the decoder can reach: a state with at most kTabTail positions left
// becomes a tail (all its orderings, in rank order); a larger one a search
// over its next h = min(kTabHead, positions - kTabTail) positions (every
// h-prefix in rank order with the rank where its completions start and the
// state it leaves), with a slot table.  States are keyed by their counts
// alone, so classes with equal part multisets share them.
#include <cuda_runtime.h>

#include <algorithm>
#include <cmath>
#include <cstring>
#include <string>
#include <unordered_map>
#include <vector>

#include "llvq_internal.h"
#include "llvq_tables.cuh"

namespace llvq {

namespace {

using u128 = unsigned __int128;

constexpr int kTabMaxVals = 8;                    // value indices must fit a byte-permute selector
constexpr size_t kTabMaxEntries = 1u << 24;       // search entries (16 B each)
constexpr size_t kTabMaxTail = 3u << 23;          // tail entries (8 B each): at most 192 MiB

u128 multinomial_counts(const int* c) {
  u128 out = 1;
  int rem = 0;
  for (int j = 0; j < kTabMaxVals; ++j) {
    for (int k = 1; k <= c[j]; ++k) {
      ++rem;
      out = out * (u128)rem / (u128)k;
    }
  }
  return out;
}

uint64_t pack_counts(const int* c) {
  uint64_t k = 0;
  for (int j = 0; j < kTabMaxVals; ++j) k |= (uint64_t)c[j] << (5 * j);
  return k;
}

void unpack_counts(uint64_t k, int* c) {
  for (int j = 0; j < kTabMaxVals; ++j) c[j] = (int)((k >> (5 * j)) & 31u);
}

struct Builder {
  TabHost& t;
  std::unordered_map<uint64_t, uint32_t> ids;
  std::vector<uint64_t> keys;
  std::vector<int> depth;  // lookups from a state to the end of its part
  std::string why;

  explicit Builder(TabHost& tab) : t(tab) {}

  // States are keyed by their counts and their entry format: value-index
  // nibbles (the parts of odd and weight-0/24 classes) or two bit planes
  // (the parts of weight-8/12/16 classes, at most four values).
  uint32_t get(const int* c, bool planes) {
    const uint64_t key = pack_counts(c) | (planes ? 1ull << 63 : 0ull);
    auto it = ids.find(key);
    if (it != ids.end()) return it->second;
    const uint32_t id = (uint32_t)keys.size();
    ids.emplace(key, id);
    keys.push_back(key);
    return id;
  }

  // Every ordering of the remaining counts, in rank order (value index
  // ascending at each position): as nibble strings, or as bit planes (bit t
  // of the low 12 bits = bit 0 of the value index at step t, bit 12 + t =
  // its bit 1).
  void tail_state(int* c, int rem, uint64_t prefix, int pos, bool planes, std::vector<uint64_t>& out) {
    if (pos == rem) {
      out.push_back(prefix);
      return;
    }
    for (int j = 0; j < kTabMaxVals; ++j) {
      if (!c[j]) continue;
      --c[j];
      const uint64_t add = planes ? (((uint64_t)(j & 1) << pos) | ((uint64_t)((j >> 1) & 1) << (kTabTail + pos)))
                                  : (uint64_t)j << (4 * pos);
      tail_state(c, rem, prefix | add, pos + 1, planes, out);
      ++c[j];
    }
  }

  struct Prefix {
    u128 start;
    uint32_t next;
    uint32_t nib;
  };

  // Search prefixes: nibbles, or bit planes (bit t = bit 0 of step t, bit
  // 8 + t = bit 1).
  void search_state(int* c, int h, int pos, uint32_t nib, bool planes, u128& cursor, std::vector<Prefix>& out) {
    if (pos == h) {
      const uint32_t nx = get(c, planes);
      out.push_back({cursor, nx, nib});
      cursor += multinomial_counts(c);
      return;
    }
    for (int j = 0; j < kTabMaxVals; ++j) {
      if (!c[j]) continue;
      --c[j];
      const uint32_t add = planes ? (((uint32_t)(j & 1) << pos) | ((uint32_t)((j >> 1) & 1) << (8 + pos)))
                                  : (uint32_t)j << (4 * pos);
      search_state(c, h, pos + 1, nib | add, planes, cursor, out);
      ++c[j];
    }
  }

  bool run() {
    // states are processed in creation order; children are created while
    // their parent is processed, so the vector grows behind the cursor
    for (size_t s = 0; s < keys.size(); ++s) {
      int c[kTabMaxVals];
      const bool planes = keys[s] >> 63;
      unpack_counts(keys[s] & ~(1ull << 63), c);
      int rem = 0;
      for (int j = 0; j < kTabMaxVals; ++j) rem += c[j];
      const u128 n = multinomial_counts(c);
      if (n >> 46) return fail("a part has 2^46 or more orderings");
      uint4 r0{0, 0, 0, 0}, r1{0, 0, 0, 0};
      if (rem <= kTabTail) {
        if (planes) {
          if (t.tail2.size() + (size_t)n > kTabMaxTail) return fail("tail tables too large");
          r0.x = (uint32_t)t.tail2.size();
          std::vector<uint64_t> seqs;
          tail_state(c, rem, 0, 0, true, seqs);
          for (uint64_t q : seqs) t.tail2.push_back((uint32_t)q);
        } else {
          if (t.tail.size() + (size_t)n > kTabMaxTail) return fail("tail tables too large");
          r0.x = (uint32_t)t.tail.size();
          std::vector<uint64_t> seqs;
          tail_state(c, rem, 0, 0, false, seqs);
          t.tail.insert(t.tail.end(), seqs.begin(), seqs.end());
        }
        r0.z = kTabTailBit | (uint32_t)rem;
      } else {
        const int h = std::min(kTabHead, rem - kTabTail);
        std::vector<Prefix> pre;
        u128 cursor = 0;
        search_state(c, h, 0, 0, planes, cursor, pre);
        if (cursor != n) return fail("prefix counts do not add up");
        if (pre.size() >= (size_t)kTabMaxStateEntries) return fail("a search state has too many prefixes");
        if (t.entry.size() + pre.size() > kTabMaxEntries) return fail("search tables too large");
        // slot function g(r) = umulhi((u32)(r >> s), M): s makes r >> s fit
        // 32 bits, M spreads the ranks over about kTabSlotsPerEntry slots per
        // entry (M <= G 2^32 / (qmax + 1) keeps g below G)
        const uint64_t n64 = (uint64_t)n;
        int sh = 0;
        while (((n64 - 1) >> sh) >> 32) ++sh;
        const uint64_t qmax = (n64 - 1) >> sh;
        uint64_t want = 1;
        while (want < (uint64_t)kTabSlotsPerEntry * pre.size()) want <<= 1;
        const u128 mw = ((u128)want << 32) / (u128)(qmax + 1);
        const uint32_t M = mw > 0xFFFFFFFFu ? 0xFFFFFFFFu : (mw ? (uint32_t)mw : 1u);
        auto gof = [&](uint64_t r) { return (uint32_t)(((uint64_t)(uint32_t)(r >> sh) * M) >> 32); };
        const uint32_t slots = gof(n64 - 1) + 1;
        if (t.slot.size() / 2 + slots > kTabMaxEntries) return fail("slot tables too large");
        r0.x = (uint32_t)(t.slot.size() / 2);
        r0.y = M;
        r0.z = (uint32_t)sh | ((uint32_t)h << 8);
        r0.w = (uint32_t)t.entry.size();
        r1 = make_uint4((uint32_t)n64, (uint32_t)(n64 >> 32), (uint32_t)pre.size(), 0);
        const size_t e0 = t.entry.size();
        for (const Prefix& p : pre)
          t.entry.push_back({(uint32_t)(uint64_t)p.start, (uint32_t)((uint64_t)p.start >> 32), p.next, p.nib});
        auto entry_of = [&](uint64_t rank) {
          size_t lo = 0, hi = pre.size();
          while (lo + 1 < hi) {
            const size_t mid = (lo + hi) / 2;
            if ((uint64_t)pre[mid].start <= rank) lo = mid; else hi = mid;
          }
          return lo;
        };
        // first rank of slot g: the smallest q with umulhi(q, M) >= g, shifted back
        auto first_rank = [&](uint32_t g) -> uint64_t {
          const uint64_t q = (uint64_t)((((u128)g << 32) + M - 1) / M);
          return q << sh;
        };
        for (uint32_t g = 0; g < slots; ++g) {
          const uint64_t lo = first_rank(g);
          const uint64_t hi = g + 1 < slots ? first_rank(g + 1) : n64;
          if (lo >= hi || gof(lo) != g || (lo && gof(lo - 1) >= g)) return fail("slot function is not monotone");
          const size_t j = entry_of(lo);
          size_t inside = 0;
          for (size_t e = j + 1; e < pre.size() && (uint64_t)pre[e].start < hi; ++e) ++inside;
          t.slot.push_back(t.entry[e0 + j]);
          if (inside == 0) {
            t.slot.push_back(make_uint4(0xFFFFFFFFu, 0xFFFFFFFFu, 0, 0));
          } else if (inside == 1) {
            t.slot.push_back(t.entry[e0 + j + 1]);
          } else {
            const uint4& nx = t.entry[e0 + j + 1];
            t.slot.push_back(make_uint4(nx.x, nx.y, kTabSlotMulti, (uint32_t)(j + 1)));
          }
        }
      }
      t.state.push_back(r0);
      t.state.push_back(r1);
    }
    // lookups to the end of a part from each state (children come later in
    // creation order, so walk backwards)
    depth.assign(keys.size(), 1);
    for (size_t s = keys.size(); s-- > 0;) {
      const uint4& r0 = t.state[2 * s];
      if (r0.z & kTabTailBit) continue;
      int d = 0;
      for (uint32_t e = 0; e < t.state[2 * s + 1].z; ++e) d = std::max(d, depth[t.entry[r0.w + e].z]);
      depth[s] = 1 + d;
    }
    return true;
  }

  bool fail(const char* msg) {
    why = msg;
    return false;
  }
};

// Move masks of the bit-wise expand by mask m (Hacker's Delight, section 7-5,
// the inverse of compress): stage i moves the bits marked in mv[i] left by
// 2^i positions, applied for i = 4 down to 0.
void expand_masks(uint32_t m, uint32_t mv[5]) {
  uint32_t mk = ~m << 1;
  for (int i = 0; i < 5; ++i) {
    uint32_t mp = mk ^ (mk << 1);
    mp ^= mp << 2;
    mp ^= mp << 4;
    mp ^= mp << 8;
    mp ^= mp << 16;
    const uint32_t v = mp & m;
    mv[i] = v;
    m = (m ^ v) | (v >> (1 << i));
    mk &= ~mp;
  }
}

}  // namespace

bool build_decode_tables(const Codebook& cb, TabHost& t, std::string* why_out) {
  t = TabHost{};
  Builder b(t);
  auto bad = [&](const std::string& msg) {
    t = TabHost{};
    if (why_out) *why_out = msg;
    return false;
  };
  const size_t n = cb.cls.size();
  std::vector<uint2> parts(n);
  for (size_t k = 0; k < n; ++k) {
    const DevClass& c = cb.cls[k];
    if (c.nv0 + c.nv1 > kTabMaxVals) return bad("a class has more than 8 distinct magnitudes");
    int a[kTabMaxVals] = {0}, z[kTabMaxVals] = {0};
    if (c.parity) {
      for (int j = 0; j < c.nv0; ++j) a[j] = c.m0[j];
      parts[k] = make_uint2(b.get(a, false), kTabEnd);
    } else {
      for (int j = 0; j < c.nv1; ++j) a[j] = c.m1[j];
      for (int j = 0; j < c.nv0; ++j) z[j] = c.m0[j];
      // two parts (weight 8, 12, 16): bit-plane entries, at most four values a part
      const bool planes = c.even_weight > 0 && c.even_weight < kDim;
      if (planes && (c.nv0 > 4 || c.nv1 > 4)) return bad("a two-part class has a part of more than four values");
      parts[k] = make_uint2(c.even_weight > 0 ? b.get(a, planes) : kTabEnd,
                            c.even_weight < kDim ? b.get(z, planes) : kTabEnd);
    }
  }
  if (!b.run()) return bad(b.why);
  if ((uint64_t)cb.total >> 48) return bad("the codebook has 2^48 or more codewords");
  if (b.keys.size() >= 0xFFFFu) return bad("more than 65534 decoder states");
  t.crec.assign(kTabClassRecords * n, uint4{0, 0, 0, 0});
  for (size_t k = 0; k < n; ++k) {
    const DevClass& c = cb.cls[k];
    const uint2 st = parts[k];
    // searches before each part's tail (depth counts the tail too)
    t.max_searches = std::max(t.max_searches, (st.x != kTabEnd ? b.depth[st.x] - 1 : 0) +
                                                  (st.y != kTabEnd ? b.depth[st.y] - 1 : 0));
    // values by selector: odd and weight 0/24: the one part's values from
    // byte 0; weight 8/12/16: part B's values in bytes 0-3, part A's in 4-7
    uint64_t vals = 0;
    int d0 = 0;
    if (c.parity) {
      for (int j = 0; j < c.nv0; ++j) vals |= (uint64_t)(uint8_t)c.v0[j] << (8 * j);
    } else {
      d0 = c.even_weight > 0 && c.even_weight < kDim ? 4 : c.nv0;
      for (int j = 0; j < c.nv0; ++j) vals |= (uint64_t)(uint8_t)c.v0[j] << (8 * j);
      for (int j = 0; j < c.nv1; ++j) vals |= (uint64_t)(uint8_t)c.v1[j] << (8 * (d0 + j));
    }
    int shape = kShapeOdd24;
    if (!c.parity)
      shape = c.even_weight == 0 || c.even_weight == kDim ? kShapeEven24
              : c.even_weight == 12                        ? kShapeEven12
                                                           : kShapeEven16;
    // the part that is searched (P1) and the tail-only part (P2)
    const bool p1a = shape == kShapeOdd24 || shape == kShapeEven12 || c.even_weight >= 16;
    const uint32_t s1 = p1a ? st.x : st.y, s2 = shape >= kShapeEven16 ? (p1a ? st.y : st.x) : 0xFFFFu;
    const uint64_t start = (uint64_t)c.start, perm = c.perm_count;
    const uint64_t mp = ~0ull / perm, mf = ~0ull / c.f1_perm;
    const uint32_t meta = (uint32_t)shape | ((uint32_t)c.sign_shift << 2) | ((uint32_t)c.required << 7) |
                          ((uint32_t)(c.even_weight == kDim) << 8) | ((uint32_t)p1a << 9);
    uint4* r = t.crec.data() + kTabClassRecords * k;
    r[0] = make_uint4((uint32_t)start, (uint32_t)(start >> 32) | (meta << 16), (uint32_t)perm,
                      (uint32_t)(perm >> 32) | (s1 << 16));
    r[1] = make_uint4((uint32_t)mp, (uint32_t)(mp >> 32), (uint32_t)vals, (uint32_t)(vals >> 32));
    const uint32_t wbase = c.parity ? 0u : (uint32_t)cb.weight_start[c.even_weight];
    r[2] = make_uint4((uint32_t)mf, (uint32_t)(mf >> 32), (uint32_t)c.f1_perm,
                      (s2 & 0xFFFFu) | (wbase << 16) | ((uint32_t)d0 << 28));
  }
  t.bucket.assign(kBuckets + 1, 0);
  for (int bk = 0; bk <= kBuckets; ++bk) {  // owner class of each bucket's lowest index
    const uint64_t lo = bucket_low(bk);
    t.bucket[bk] = (uint16_t)(lo >= (uint64_t)cb.total ? n - 1
                                                        : find_class(cb.class_start.data(), (int)n, (int64_t)lo));
  }
  // bit-plane deposit masks per word (weight order): stage i moves bits by
  // 2^i; m[i] = stage i of the word's deposit | low byte of the complement's
  // stage i << 24, m[5..7] the complement's upper 16 bits, two per word
  t.expand2.assign((size_t)kNumGolay * kTabExpand2Words, 0);
  for (int gi = 0; gi < kNumGolay; ++gi) {
    uint32_t mva[5], mvb[5];
    expand_masks(cb.wlist_word[gi], mva);
    expand_masks(~cb.wlist_word[gi] & kFull24, mvb);
    uint32_t* m = t.expand2.data() + (size_t)gi * kTabExpand2Words;
    for (int i = 0; i < 5; ++i) m[i] = mva[i] | ((mvb[i] & 0xFFu) << 24);
    m[5] = (mvb[0] >> 8) | ((mvb[1] >> 8) << 16);
    m[6] = (mvb[2] >> 8) | ((mvb[3] >> 8) << 16);
    m[7] = mvb[4] >> 8;
  }
  t.ok = true;
  return true;
}

namespace {

// deposit4[m * 16 + s]: the low popc(m) bits of s placed on the set bits of m.
const uint8_t* host_deposit4() {
  static uint8_t table[256];
  static bool ready = false;
  if (!ready) {
    for (int i = 0; i < 256; ++i) {
      const uint32_t m = i >> 4;
      uint32_t src = i & 15, dep = 0;
      for (int bit = 0; bit < 4; ++bit)
        if ((m >> bit) & 1u) {
          dep |= (src & 1u) << bit;
          src >>= 1;
        }
      table[i] = (uint8_t)dep;
    }
    ready = true;
  }
  return table;
}

}  // namespace

TabCtx host_tab_ctx(const Codebook& cb) {
  const TabHost& t = cb.tab;
  TabCtx tc{};
  tc.srec = t.state.data();
  tc.crec = t.crec.data();
  tc.bucket = t.bucket.data();
  tc.words = cb.wlist_word.data();
  tc.golay = cb.golay.data();
  tc.starts = cb.class_start.data();
  tc.deposit4 = host_deposit4();
  tc.entry = t.entry.data();
  tc.slot = t.slot.data();
  tc.tail = t.tail.data();
  tc.tail2 = t.tail2.data();
  tc.expand2 = reinterpret_cast<const uint4*>(t.expand2.data());
  tc.n_classes = (int)cb.cls.size();
  tc.n_states = (int)(t.state.size() / 2);
  tc.max_searches = t.max_searches;
  tc.total = cb.total;
  return tc;
}

// Host decode of one index with the tables (the same tab_* code the kernels
// run); false and zeros outside the codebook.
bool decode_index_tables_host(const Codebook& cb, int64_t v, int32_t* out) {
  for (int d = 0; d < kDim; ++d) out[d] = 0;
  if (!cb.tab.ok) return false;
  const TabCtx tc = host_tab_ctx(cb);
  int y[kDim];
  const bool ok = tab_decode<false>(tc, v, y);
  for (int d = 0; d < kDim; ++d) out[d] = y[d];
  return ok;
}

}  // namespace llvq
