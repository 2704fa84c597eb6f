/*
 * llvq_oracle.c -- CPU restatement of the reference Leech-lattice (Λ24)
 * quantizer, used ONLY as test infrastructure (parity checker, CPU baseline).
 * Nothing in the product library links or calls this file.
 *
 * It restates, function by function, the pure-Python reference
 * impl/leech_lattice_vector_quantizer.py of dmnunez1993/llvq-paper-reproduction:
 *
 *   golay_words()            extended_golay_codewords          :914-933
 *   gen_leaders()            generate_shell_class_leaders      :501-554
 *   local_structure()        build_local_structure             :386-417
 *   class sort / offsets     LeechLatticeVectorQuantizer.__init__ :163-185, :336-353
 *   theta check              _validate + leech_shell_counts    :370-383, :936-999
 *   solve_even()             solve_even_subclass               :619-646
 *   solve_odd()              solve_odd_subclass                :649-666
 *   ref_projection()         dot_product (CPython 3.12 sum)    :904-905
 *   oracle_quantize()        quantize                          :282-314
 *   oracle_encode()          encode_codeword + rank_*          :247-280, :692-771, :819-841, :870-889
 *   oracle_codeword()        codeword + unrank_*               :196-245, :774-816, :844-867
 *
 * Floating point: the reference runs on CPython >= 3.12 (.python-version:1
 * pins 3.12).  There `sum()` over floats is Neumaier-compensated, so the
 * projection x.y is NOT a naive left-to-right sum; ref_projection() restates
 * CPython 3.12's builtin_sum float loop exactly.  Build with
 * -ffp-contract=off so no product/add pair is fused into an FMA.
 *
 * Quantize modes: mode 0 sorts inside every (Golay word, class) pair exactly as
 * the reference does; mode 1 hoists the per-word sorts out of the class loop
 * (the orderings depend only on x and the Golay word, never on the class), so
 * both modes return identical results; mode 1 is just faster.
 */
#include <math.h>
#include <pthread.h>
#include <stdint.h>
#include <stdio.h>
#include <stdlib.h>
#include <string.h>

#define DIM 24
#define NGOLAY 4096

typedef unsigned __int128 u128;
typedef __int128 i128;

static const double LATTICE_SCALE = 0.35355339059327373; /* 1.0/sqrt(8.0) as CPython computes it */

typedef struct {
    int shell;
    int parity;        /* 0 even, 1 odd */
    int leader[DIM];   /* magnitudes, descending (ClassLeader.leader) */
    int nval;          /* distinct magnitudes */
    int val[DIM];      /* distinct magnitudes, descending */
    int mult[DIM];     /* their multiplicities */
    int even_weight;   /* #coords with |v| = 2 mod 4 (even classes) */
    int nonzero;
    int leader_sum;
    uint64_t count;
    uint64_t sign_count;
    uint64_t perm_count;
    uint64_t f1_perm;  /* multinomial of the f1 multiplicities (even), 1 for odd */
    int golay_count;
    int64_t start;     /* global index of the class's first codeword */
    /* solver tables */
    int f0_len, f1_len;
    int f0_asc[DIM];   /* _ascending_multiset(f0) */
    int f1_asc[DIM];   /* _ascending_multiset(f1) */
    int odd_signed_asc[DIM]; /* sorted(_odd_signed_leader_values) */
    int required;      /* (sum(leader) % 8) // 4 */
} ocls;

typedef struct {
    int min_shell, max_shell;
    int ncls;
    ocls* cls;
    int64_t shell_offset[64];
    uint64_t shell_count[64];
    uint64_t total;
    uint32_t golay[NGOLAY];     /* lex order, bit d = coordinate d */
    int golay_weight[NGOLAY];
    int golay_rank_in_weight[NGOLAY]; /* position among words of equal weight, lex order */
    int words_by_weight[25][NGOLAY];
    int nwords_weight[25];
} oracle_book;

/* ------------------------------------------------------------------ Golay */

/* extended_golay_codewords(): cyclic [23,12,7] code from
 * g(x)=x^11+x^9+x^7+x^6+x^5+x+1, parity bit appended, sorted as 24-tuples
 * (coordinate 0 compared first). */
static void golay_words(uint32_t out[NGOLAY]) {
    const uint32_t gen = (1u << 11) | (1u << 9) | (1u << 7) | (1u << 6) | (1u << 5) | (1u << 1) | 1u;
    uint32_t keys[NGOLAY];
    for (uint32_t msg = 0; msg < NGOLAY; ++msg) {
        uint32_t code23 = 0;
        for (int b = 0; b < 12; ++b)
            if ((msg >> b) & 1u) code23 ^= gen << b;
        int par = __builtin_popcount(code23 & 0x7FFFFFu) & 1;
        uint32_t word = (code23 & 0x7FFFFFu) | ((uint32_t)par << 23); /* bit d = coord d */
        /* lexicographic key: coordinate 0 is the most significant */
        uint32_t key = 0;
        for (int d = 0; d < DIM; ++d) key |= ((word >> d) & 1u) << (23 - d);
        keys[msg] = key;
    }
    /* sort keys ascending */
    for (int i = 1; i < NGOLAY; ++i) {
        uint32_t k = keys[i];
        int j = i - 1;
        while (j >= 0 && keys[j] > k) { keys[j + 1] = keys[j]; --j; }
        keys[j + 1] = k;
    }
    for (int i = 0; i < NGOLAY; ++i) {
        uint32_t w = 0;
        for (int d = 0; d < DIM; ++d) w |= ((keys[i] >> (23 - d)) & 1u) << d;
        out[i] = w;
    }
}

/* ------------------------------------------------------------ combinatorics */

/* multiset_permutation_count(): n! / prod(c_i!) -- exact for n <= 24 in 128 bits
 * by multiplying binomials. */
static u128 multinomial(const int* counts, int n) {
    int total = 0;
    for (int i = 0; i < n; ++i) total += counts[i];
    u128 out = 1;
    int rem = total;
    for (int i = 0; i < n; ++i) {
        /* C(rem, counts[i]) */
        u128 c = 1;
        for (int k = 1; k <= counts[i]; ++k) c = c * (u128)(rem - counts[i] + k) / (u128)k;
        out *= c;
        rem -= counts[i];
    }
    return out;
}

/* --------------------------------------------------------------- classes */

static void class_finish(ocls* c) {
    /* distinct magnitudes, descending */
    c->nval = 0;
    for (int d = 0; d < DIM; ++d) {
        int v = c->leader[d];
        if (c->nval && c->val[c->nval - 1] == v) c->mult[c->nval - 1]++;
        else { c->val[c->nval] = v; c->mult[c->nval] = 1; c->nval++; }
    }
    c->nonzero = 0; c->leader_sum = 0; c->even_weight = 0;
    for (int d = 0; d < DIM; ++d) {
        c->leader_sum += c->leader[d];
        if (c->leader[d]) c->nonzero++;
        if (c->leader[d] % 4 == 2) c->even_weight++;
    }
    c->required = (c->leader_sum % 8) / 4;
    /* ascending multisets */
    c->f0_len = c->f1_len = 0;
    for (int d = DIM - 1; d >= 0; --d) {
        int v = c->leader[d];
        if (c->parity == 0) {
            if (v % 4 == 0) c->f0_asc[c->f0_len++] = v;
            else c->f1_asc[c->f1_len++] = v;
        }
    }
    if (c->parity == 1) {
        int s[DIM];
        for (int d = 0; d < DIM; ++d) s[d] = (c->leader[d] % 4 == 1) ? c->leader[d] : -c->leader[d];
        /* sort ascending */
        for (int i = 1; i < DIM; ++i) {
            int k = s[i], j = i - 1;
            while (j >= 0 && s[j] > k) { s[j + 1] = s[j]; --j; }
            s[j + 1] = k;
        }
        memcpy(c->odd_signed_asc, s, sizeof s);
    }
}

/* build_local_structure(): number of compatible Golay words, sign count,
 * permutation count.  Returns 0 when the class is empty. */
static int local_structure(ocls* c, const int nwords_weight[25]) {
    if (c->parity == 0) {
        int f0c[DIM], f1c[DIM], n0 = 0, n1 = 0;
        for (int i = 0; i < c->nval; ++i) {
            if (c->val[i] % 4 == 0) f0c[n0++] = c->mult[i];
            else f1c[n1++] = c->mult[i];
        }
        int w = c->even_weight;
        c->golay_count = nwords_weight[w];
        u128 f0 = multinomial(f0c, n0), f1 = multinomial(f1c, n1);
        u128 sign;
        if (w == 0 && c->leader_sum % 8 != 0) sign = 0;
        else sign = (u128)1 << (w == 0 ? c->nonzero : c->nonzero - 1);
        u128 perm = f0 * f1;
        u128 count = (u128)c->golay_count * sign * perm;
        if (count >> 63) return -1;
        c->sign_count = (uint64_t)sign;
        c->perm_count = (uint64_t)perm;
        c->f1_perm = (uint64_t)f1;
        c->count = (uint64_t)count;
    } else {
        c->golay_count = NGOLAY;
        u128 perm = multinomial(c->mult, c->nval);
        u128 count = (u128)NGOLAY * perm;
        if (count >> 63) return -1;
        c->sign_count = 1;
        c->perm_count = (uint64_t)perm;
        c->f1_perm = 1;
        c->count = (uint64_t)count;
    }
    return c->count ? 1 : 0;
}

static int leader_cmp(const ocls* a, const ocls* b) {
    for (int d = 0; d < DIM; ++d)
        if (a->leader[d] != b->leader[d]) return a->leader[d] < b->leader[d] ? -1 : 1;
    if (a->parity != b->parity) return a->parity < b->parity ? -1 : 1;
    if (a->count != b->count) return a->count < b->count ? -1 : 1;
    return 0;
}

typedef struct {
    ocls* buf;
    int n, cap;
    int shell, parity;
    int mags[16];
    int nmags;
    int counts[16];
    const int* nww;
    int overflow;
} gen_state;

static void gen_emit(gen_state* s) {
    ocls c;
    memset(&c, 0, sizeof c);
    c.shell = s->shell;
    c.parity = s->parity;
    int d = 0;
    for (int i = s->nmags - 1; i >= 0; --i)
        for (int k = 0; k < s->counts[i]; ++k) c.leader[d++] = s->mags[i];
    if (d != DIM) return;
    class_finish(&c);
    int r = local_structure(&c, s->nww);
    if (r < 0) { s->overflow = 1; return; }
    if (r == 0) return;
    if (s->n == s->cap) {
        s->cap = s->cap ? 2 * s->cap : 64;
        s->buf = (ocls*)realloc(s->buf, (size_t)s->cap * sizeof(ocls));
    }
    s->buf[s->n++] = c;
}

/* _multiplicity_solutions(): all count vectors over `mags` with
 * sum(counts) = slots and sum(count*mag^2) = square_sum. */
static void gen_rec(gen_state* s, int idx, int slots, int sq) {
    if (idx < 0) {
        if (slots == 0 && sq == 0) gen_emit(s);
        return;
    }
    int m = s->mags[idx];
    int m2 = m * m;
    int maxc = (m2 == 0) ? slots : (slots < sq / m2 ? slots : sq / m2);
    for (int c = maxc; c >= 0; --c) {
        s->counts[idx] = c;
        gen_rec(s, idx - 1, slots - c, sq - c * m2);
    }
    s->counts[idx] = 0;
}

static int cmp_cls(const void* a, const void* b) { return leader_cmp((const ocls*)a, (const ocls*)b); }

/* ---------------------------------------------------------------- theta */

static void theta_counts(int max_shell, i128* out) {
    /* leech_shell_counts(): E4^3 - 720 * Delta, truncated at max_shell */
    int n = max_shell;
    i128* e4 = calloc((size_t)n + 1, sizeof(i128));
    e4[0] = 1;
    for (int k = 1; k <= n; ++k) {
        i128 s = 0;
        for (int dv = 1; dv <= k; ++dv)
            if (k % dv == 0) s += (i128)dv * dv * dv;
        e4[k] = 240 * s;
    }
    i128* e2 = calloc((size_t)n + 1, sizeof(i128));
    i128* e3 = calloc((size_t)n + 1, sizeof(i128));
    for (int i = 0; i <= n; ++i)
        for (int j = 0; i + j <= n; ++j) e2[i + j] += e4[i] * e4[j];
    for (int i = 0; i <= n; ++i)
        for (int j = 0; i + j <= n; ++j) e3[i + j] += e2[i] * e4[j];
    /* Delta = q * prod_{k>=1} (1-q^k)^24 */
    i128* co = calloc((size_t)n + 1, sizeof(i128));
    i128* tmp = calloc((size_t)n + 1, sizeof(i128));
    co[0] = 1;
    i128 binom24[25];
    for (int k = 0; k <= 24; ++k) {
        i128 b = 1;
        for (int t = 1; t <= k; ++t) b = b * (24 - k + t) / t;
        binom24[k] = b;
    }
    for (int kk = 1; kk <= n; ++kk) {
        memset(tmp, 0, ((size_t)n + 1) * sizeof(i128));
        for (int i = 0; i <= n; ++i) {
            if (!co[i]) continue;
            for (int k = 0; k <= 24 && i + kk * k <= n; ++k) {
                i128 f = (k & 1) ? -binom24[k] : binom24[k];
                tmp[i + kk * k] += co[i] * f;
            }
        }
        memcpy(co, tmp, ((size_t)n + 1) * sizeof(i128));
    }
    for (int m = 0; m <= n; ++m) {
        i128 delta = m >= 1 ? co[m - 1] : 0;
        out[m] = e3[m] - 720 * delta;
    }
    free(e4); free(e2); free(e3); free(co); free(tmp);
}

/* ----------------------------------------------------------------- book */

void oracle_destroy(oracle_book* b) {
    if (!b) return;
    free(b->cls);
    free(b);
}

/* Build the implicit codebook for shells [min_shell, max_shell]
 * (the reference always uses min_shell = 2).  Returns NULL when the total
 * codeword count does not fit a signed 64-bit index or the theta check fails. */
oracle_book* oracle_create(int min_shell, int max_shell) {
    if (min_shell < 2 || max_shell < min_shell || max_shell > 60) return NULL;
    oracle_book* b = (oracle_book*)calloc(1, sizeof(oracle_book));
    b->min_shell = min_shell;
    b->max_shell = max_shell;
    golay_words(b->golay);
    for (int i = 0; i < NGOLAY; ++i) {
        int w = __builtin_popcount(b->golay[i]);
        b->golay_weight[i] = w;
        b->golay_rank_in_weight[i] = b->nwords_weight[w];
        b->words_by_weight[w][b->nwords_weight[w]++] = i;
    }
    i128* theta = calloc((size_t)max_shell + 1, sizeof(i128));
    theta_counts(max_shell, theta);
    uint64_t cursor = 0;
    u128 total = 0;
    gen_state s;
    memset(&s, 0, sizeof s);
    s.nww = b->nwords_weight;
    for (int m = min_shell; m <= max_shell; ++m) {
        int first = s.n;
        int target = 16 * m;
        int max_abs = (int)sqrt((double)target);
        while ((max_abs + 1) * (max_abs + 1) <= target) ++max_abs;
        while (max_abs * max_abs > target) --max_abs;
        for (int parity = 0; parity < 2; ++parity) {
            s.shell = m;
            s.parity = parity;
            s.nmags = 0;
            for (int v = parity; v <= max_abs; v += 2) s.mags[s.nmags++] = v;
            memset(s.counts, 0, sizeof s.counts);
            gen_rec(&s, s.nmags - 1, DIM, target);
        }
        if (s.overflow) break;
        qsort(s.buf + first, (size_t)(s.n - first), sizeof(ocls), cmp_cls);
        u128 shell_total = 0;
        for (int k = first; k < s.n; ++k) {
            s.buf[k].start = (int64_t)(cursor + (uint64_t)shell_total);
            shell_total += s.buf[k].count;
        }
        if ((i128)shell_total != theta[m]) { s.overflow = 2; break; }
        b->shell_offset[m] = (int64_t)cursor;
        b->shell_count[m] = (uint64_t)shell_total;
        total += shell_total;
        /* indices are unsigned 64-bit (two's-complement int64 images above
           2^63); all ones stays free for "no index" */
        if (total >= ((u128)1 << 64) - 1) { s.overflow = 1; break; }
        cursor = (uint64_t)total;
    }
    free(theta);
    if (s.overflow) { free(s.buf); free(b); return NULL; }
    b->cls = s.buf;
    b->ncls = s.n;
    b->total = (uint64_t)total;
    return b;
}

int oracle_num_classes(const oracle_book* b) { return b->ncls; }
uint64_t oracle_total(const oracle_book* b) { return b->total; }
void oracle_golay_words(uint32_t out[NGOLAY]) { golay_words(out); }

int oracle_class_info(const oracle_book* b, int k, int32_t* shell, int32_t* parity, int32_t leader[DIM],
                      uint64_t* count, uint64_t* sign_count, uint64_t* perm_count, int32_t* golay_count,
                      int64_t* start) {
    if (k < 0 || k >= b->ncls) return -1;
    const ocls* c = &b->cls[k];
    *shell = c->shell; *parity = c->parity;
    for (int d = 0; d < DIM; ++d) leader[d] = c->leader[d];
    *count = c->count; *sign_count = c->sign_count; *perm_count = c->perm_count;
    *golay_count = c->golay_count; *start = c->start;
    return 0;
}

/* --------------------------------------------------------------- search */

/* CPython 3.12 builtin sum() over the float products x_d*y_d:
 * the first item enters through int 0 + float, the rest through the
 * Neumaier-compensated float loop, and the compensation is added at the end
 * when it is non-zero and finite. */
static double ref_projection(const double* x, const int* y) {
    double f = 0.0 + x[0] * (double)y[0];
    double c = 0.0;
    for (int d = 1; d < DIM; ++d) {
        double xi = x[d] * (double)y[d];
        double t = f + xi;
        if (fabs(f) >= fabs(xi)) c += (f - t) + xi;
        else c += (xi - t) + f;
        f = t;
    }
    if (c != 0.0 && isfinite(c)) f += c;
    return f;
}

/* sorted(positions, key=lambda p: (key[p], p)) */
static void sort_positions(int* pos, int n, const double* key) {
    for (int i = 1; i < n; ++i) {
        int p = pos[i], j = i - 1;
        while (j >= 0 && (key[pos[j]] > key[p] || (key[pos[j]] == key[p] && pos[j] > p))) {
            pos[j + 1] = pos[j];
            --j;
        }
        pos[j + 1] = p;
    }
}

typedef struct {
    int f0[DIM], f1[DIM], n0, n1; /* ordered_f0 / ordered_f1 */
    int odd[DIM];                 /* ordered positions of x' */
} word_orders;

static void compute_orders(const double* x, uint32_t word, word_orders* o, int want_even, int want_odd) {
    if (want_even) {
        double ax[DIM];
        o->n0 = o->n1 = 0;
        for (int d = 0; d < DIM; ++d) {
            ax[d] = fabs(x[d]);
            if ((word >> d) & 1u) o->f1[o->n1++] = d;
            else o->f0[o->n0++] = d;
        }
        sort_positions(o->f0, o->n0, ax);
        sort_positions(o->f1, o->n1, ax);
    }
    if (want_odd) {
        double xp[DIM];
        for (int d = 0; d < DIM; ++d) {
            xp[d] = ((word >> d) & 1u) ? -x[d] : x[d];
            o->odd[d] = d;
        }
        sort_positions(o->odd, DIM, xp);
    }
}

/* solve_even_subclass() */
static void solve_even(const double* x, const ocls* c, const word_orders* o, int* y) {
    memset(y, 0, DIM * sizeof(int));
    for (int i = 0; i < o->n0; ++i) {
        int p = o->f0[i], m = c->f0_asc[i];
        y[p] = x[p] >= 0 ? m : -m;
    }
    for (int i = 0; i < o->n1; ++i) {
        int p = o->f1[i], m = c->f1_asc[i];
        y[p] = x[p] >= 0 ? m : -m;
    }
    if (c->f1_len) {
        int neg = 0;
        for (int i = 0; i < o->n1; ++i) neg += y[o->f1[i]] < 0;
        if ((neg % 2) != c->required) y[o->f1[0]] = -y[o->f1[0]];
    }
}

/* solve_odd_subclass() */
static void solve_odd(const ocls* c, uint32_t word, const word_orders* o, int* y) {
    int yp[DIM];
    for (int r = 0; r < DIM; ++r) yp[o->odd[r]] = c->odd_signed_asc[r];
    for (int d = 0; d < DIM; ++d) y[d] = ((word >> d) & 1u) ? -yp[d] : yp[d];
}

/* quantize(): argmax over (Golay word lex order, shell asc, class asc) of
 * LATTICE_SCALE*proj - shell with strict '>'.  Returns the index, or -1 if no
 * candidate exists (all scores NaN).
 * mode bit 0: hoist the per-word sorts (same result, faster).
 * mode bit 1: angular search for the multi-shell shape of shape-gain
 * quantization (no reference counterpart): the score is proj / |y| =
 * proj / sqrt(16 shell) in fp64 instead, the same loop order and strict '>'.
 * Within one class the best codeword of a word is the same for both scores
 * (every codeword of a class has the same norm). */
int64_t oracle_encode(const oracle_book* b, const int32_t* y);

int64_t oracle_quantize(const oracle_book* b, const double* x, int mode, int32_t* best_golay, int32_t* best_class,
                        double* best_score_out, int32_t* best_y) {
    double best = -INFINITY;
    int found = 0, bg = -1, bk = -1;
    int by[DIM] = {0}, y[DIM];
    word_orders o;
    for (int g = 0; g < NGOLAY; ++g) {
        uint32_t word = b->golay[g];
        int wt = b->golay_weight[g];
        const int hoist = mode & 1, angular = mode & 2;
        if (hoist) compute_orders(x, word, &o, 1, 1);
        for (int k = 0; k < b->ncls; ++k) {
            const ocls* c = &b->cls[k];
            if (c->parity == 0) {
                if (wt != c->even_weight) continue;
                if (!hoist) compute_orders(x, word, &o, 1, 0);
                solve_even(x, c, &o, y);
            } else {
                if (!hoist) compute_orders(x, word, &o, 0, 1);
                solve_odd(c, word, &o, y);
            }
            double proj = ref_projection(x, y);
            double score = angular ? proj / sqrt(16.0 * (double)c->shell)
                                   : LATTICE_SCALE * proj - (double)c->shell;
            if (score > best) {
                best = score;
                found = 1;
                bg = g;
                bk = k;
                memcpy(by, y, sizeof by);
            }
        }
    }
    if (best_golay) *best_golay = bg;
    if (best_class) *best_class = bk;
    if (best_score_out) *best_score_out = best;
    if (!found) return -1;
    if (best_y) for (int d = 0; d < DIM; ++d) best_y[d] = by[d];
    return oracle_encode(b, by);
}

/* ----------------------------------------------------------- rank/unrank */

static int class_of(const oracle_book* b, int shell, const int* sorted_abs, int parity) {
    for (int k = 0; k < b->ncls; ++k) {
        const ocls* c = &b->cls[k];
        if (c->shell != shell || c->parity != parity) continue;
        if (memcmp(c->leader, sorted_abs, DIM * sizeof(int)) == 0) return k;
    }
    return -1;
}

static int golay_index_of(const oracle_book* b, uint32_t word) {
    for (int i = 0; i < NGOLAY; ++i)
        if (b->golay[i] == word) return i;
    return -1;
}

/* rank_multiset_sequence(): lexicographic rank with values tried in
 * descending order. */
static u128 rank_multiset(const int* seq, int n, const int* vals, const int* mult0, int nv, int* ok) {
    int cnt[DIM];
    memcpy(cnt, mult0, (size_t)nv * sizeof(int));
    u128 rank = 0;
    *ok = 1;
    for (int i = 0; i < n; ++i) {
        int a = seq[i], ai = -1;
        for (int j = 0; j < nv; ++j) if (vals[j] == a) ai = j;
        if (ai < 0 || cnt[ai] == 0) { *ok = 0; return 0; }
        for (int j = 0; j < nv; ++j) {
            if (j == ai) break;
            if (cnt[j] == 0) continue;
            cnt[j]--;
            rank += multinomial(cnt, nv);
            cnt[j]++;
        }
        cnt[ai]--;
    }
    return rank;
}

/* unrank_multiset_sequence() */
static int unrank_multiset(u128 rank, const int* vals, const int* mult0, int nv, int n, int* out) {
    int cnt[DIM];
    memcpy(cnt, mult0, (size_t)nv * sizeof(int));
    if (rank >= multinomial(cnt, nv)) return -1;
    for (int i = 0; i < n; ++i) {
        int placed = 0;
        for (int j = 0; j < nv; ++j) {
            if (cnt[j] == 0) continue;
            cnt[j]--;
            u128 br = multinomial(cnt, nv);
            if (rank < br) { out[i] = vals[j]; placed = 1; break; }
            rank -= br;
            cnt[j]++;
        }
        if (!placed) return -1;
    }
    return 0;
}

/* Number of sign assignments of `mags` (lower nonzero positions) whose signed
 * sum is congruent to `target` mod 8: a residue DP over the positions. */
static u128 lower_sign_count(const int* mags, int n, int target) {
    u128 dp[8] = {0}, nd[8];
    dp[0] = 1;
    for (int i = 0; i < n; ++i) {
        memset(nd, 0, sizeof nd);
        for (int r = 0; r < 8; ++r) {
            if (!dp[r]) continue;
            nd[(r + mags[i]) & 7] += dp[r];
            nd[(r - mags[i]) & 7] += dp[r];
        }
        memcpy(dp, nd, sizeof dp);
    }
    return dp[target & 7];
}

/* rank_even_signs(): the rank of the negative-mask among all masks (bit i =
 * i-th nonzero coordinate) whose signed sum is 0 mod 8, in increasing mask
 * order.  Counted bit by bit from the top: for each set bit, the masks that
 * agree above it, clear it, and are free below it. */
static u128 rank_even_signs(const int* y, int* ok) {
    int sum = 0;
    for (int d = 0; d < DIM; ++d) sum += y[d];
    if (((sum % 8) + 8) % 8 != 0) { *ok = 0; return 0; }
    int mags[DIM], neg[DIM], nz = 0;
    for (int d = 0; d < DIM; ++d)
        if (y[d]) { mags[nz] = abs(y[d]); neg[nz] = y[d] < 0; nz++; }
    u128 rank = 0;
    int high = 0; /* signed sum of the positions above the current bit */
    for (int i = nz - 1; i >= 0; --i) {
        if (neg[i]) {
            /* masks with bit i clear: position i positive */
            int need = (-(high + mags[i])) & 7;
            rank += lower_sign_count(mags, i, need);
            high -= mags[i];
        } else {
            high += mags[i];
        }
    }
    *ok = 1;
    return rank;
}

/* Enumerating form of rank_even_signs (reference :819-841), usable when the
 * vector has few nonzeros; kept to cross-check the counting form. */
int64_t oracle_rank_even_signs_enumerate(const int32_t* y) {
    int sum = 0, pos[DIM], nz = 0;
    for (int d = 0; d < DIM; ++d) sum += y[d];
    if (((sum % 8) + 8) % 8 != 0) return -1;
    for (int d = 0; d < DIM; ++d) if (y[d]) pos[nz++] = d;
    if (nz > 22) return -2;
    uint32_t target = 0;
    for (int i = 0; i < nz; ++i) if (y[pos[i]] < 0) target |= 1u << i;
    int64_t rank = 0;
    for (uint32_t mask = 0; mask < (1u << nz); ++mask) {
        int s = 0;
        for (int i = 0; i < nz; ++i) {
            int v = abs(y[pos[i]]);
            s += ((mask >> i) & 1u) ? -v : v;
        }
        if (((s % 8) + 8) % 8 != 0) continue;
        if (mask == target) return rank;
        rank++;
    }
    return -1;
}

int64_t oracle_rank_even_signs(const int32_t* y) {
    int ok;
    int yy[DIM];
    for (int d = 0; d < DIM; ++d) yy[d] = y[d];
    u128 r = rank_even_signs(yy, &ok);
    return ok ? (int64_t)r : -1;
}

/* encode_codeword(): exact index of a Leech codeword, or -1 if the vector is
 * not a codeword of this book. */
int64_t oracle_encode(const oracle_book* b, const int32_t* yin) {
    int y[DIM];
    long sq = 0;
    for (int d = 0; d < DIM; ++d) { y[d] = yin[d]; sq += (long)y[d] * y[d]; }
    if (sq % 16) return -1;
    int shell = (int)(sq / 16);
    if (shell < b->min_shell || shell > b->max_shell) return -1;
    int nodd = 0;
    for (int d = 0; d < DIM; ++d) nodd += (y[d] & 1) != 0;
    if (nodd != 0 && nodd != DIM) return -1;
    int parity = nodd ? 1 : 0;
    int key[DIM];
    for (int d = 0; d < DIM; ++d) key[d] = abs(y[d]);
    for (int i = 1; i < DIM; ++i) { /* descending */
        int k = key[i], j = i - 1;
        while (j >= 0 && key[j] < k) { key[j + 1] = key[j]; --j; }
        key[j + 1] = k;
    }
    int ci = class_of(b, shell, key, parity);
    if (ci < 0) return -1;
    const ocls* c = &b->cls[ci];
    u128 local;
    if (parity == 0) {
        uint32_t word = 0;
        for (int d = 0; d < DIM; ++d) if (abs(y[d]) % 4 == 2) word |= 1u << d;
        int g = golay_index_of(b, word);
        if (g < 0 || b->golay_weight[g] != c->even_weight) return -1;
        int gchoice = b->golay_rank_in_weight[g];
        int s0[DIM], s1[DIM], n0 = 0, n1 = 0;
        for (int d = 0; d < DIM; ++d) {
            if ((word >> d) & 1u) s1[n1++] = abs(y[d]);
            else s0[n0++] = abs(y[d]);
        }
        int v0[DIM], m0[DIM], nv0 = 0, v1[DIM], m1[DIM], nv1 = 0;
        for (int i = 0; i < c->nval; ++i) {
            if (c->val[i] % 4 == 0) { v0[nv0] = c->val[i]; m0[nv0++] = c->mult[i]; }
            else { v1[nv1] = c->val[i]; m1[nv1++] = c->mult[i]; }
        }
        int ok0, ok1, oks;
        u128 r0 = rank_multiset(s0, n0, v0, m0, nv0, &ok0);
        u128 r1 = rank_multiset(s1, n1, v1, m1, nv1, &ok1);
        if (!ok0 || !ok1) return -1;
        u128 perm = r0 * (u128)c->f1_perm + r1;
        u128 sign = rank_even_signs(y, &oks);
        if (!oks || sign >= c->sign_count) return -1;
        local = ((u128)gchoice * c->sign_count + sign) * c->perm_count + perm;
    } else {
        uint32_t word = 0;
        for (int d = 0; d < DIM; ++d) {
            int r = ((y[d] % 4) + 4) % 4;
            if (r == 3) word |= 1u << d;
            else if (r != 1) return -1;
        }
        int g = golay_index_of(b, word);
        if (g < 0) return -1;
        int mags[DIM];
        for (int d = 0; d < DIM; ++d) mags[d] = abs(y[d]);
        int ok;
        u128 perm = rank_multiset(mags, DIM, c->val, c->mult, c->nval, &ok);
        if (!ok) return -1;
        local = (u128)g * c->perm_count + perm;
    }
    return (int64_t)((uint64_t)c->start + (uint64_t)local);
}

/* apply_even_signs(): the sign_rank-th valid sign mask in increasing mask
 * order, found bit by bit from the top with the same residue counts. */
static int apply_even_signs(int* v, u128 rank) {
    int mags[DIM], pos[DIM], nz = 0;
    for (int d = 0; d < DIM; ++d) if (v[d]) { mags[nz] = v[d]; pos[nz++] = d; }
    int high = 0;
    for (int i = nz - 1; i >= 0; --i) {
        int need = (-(high + mags[i])) & 7;
        u128 zero = lower_sign_count(mags, i, need);
        if (rank < zero) {
            high += mags[i];
        } else {
            rank -= zero;
            high -= mags[i];
            v[pos[i]] = -mags[i];
        }
    }
    return (rank == 0 && ((high % 8) + 8) % 8 == 0) ? 0 : -1;
}

/* codeword(): index -> integer Leech vector (before the 1/sqrt(8) scale). */
int oracle_codeword(const oracle_book* b, int64_t index, int32_t* out) {
    const uint64_t u = (uint64_t)index;  /* unsigned: codebooks past 2^63 use the full range */
    if (u >= b->total) return -1;
    int ci = -1;
    for (int k = 0; k < b->ncls; ++k)
        if ((uint64_t)b->cls[k].start <= u) ci = k;
    const ocls* c = &b->cls[ci];
    u128 local = (u128)(u - (uint64_t)c->start);
    u128 perm = local % c->perm_count;
    u128 cur = local / c->perm_count;
    u128 sign = cur % c->sign_count;
    u128 gchoice = cur / c->sign_count;
    int v[DIM];
    if (c->parity == 0) {
        if (gchoice >= (u128)c->golay_count) return -1;
        int g = b->words_by_weight[c->even_weight][(int)gchoice];
        uint32_t word = b->golay[g];
        int v0[DIM], m0[DIM], nv0 = 0, v1[DIM], m1[DIM], nv1 = 0;
        for (int i = 0; i < c->nval; ++i) {
            if (c->val[i] % 4 == 0) { v0[nv0] = c->val[i]; m0[nv0++] = c->mult[i]; }
            else { v1[nv1] = c->val[i]; m1[nv1++] = c->mult[i]; }
        }
        u128 r1 = perm % c->f1_perm, r0 = perm / c->f1_perm;
        int s0[DIM], s1[DIM];
        int n0 = DIM - c->even_weight, n1 = c->even_weight;
        if (unrank_multiset(r0, v0, m0, nv0, n0, s0) || unrank_multiset(r1, v1, m1, nv1, n1, s1)) return -1;
        int i0 = 0, i1 = 0;
        for (int d = 0; d < DIM; ++d) v[d] = ((word >> d) & 1u) ? s1[i1++] : s0[i0++];
        if (apply_even_signs(v, sign)) return -1;
    } else {
        uint32_t word = b->golay[(int)gchoice];
        int mags[DIM];
        if (unrank_multiset(perm, c->val, c->mult, c->nval, DIM, mags)) return -1;
        for (int d = 0; d < DIM; ++d) {
            int target = ((word >> d) & 1u) ? 3 : 1;
            v[d] = (mags[d] % 4 == target) ? mags[d] : -mags[d];
        }
    }
    for (int d = 0; d < DIM; ++d) out[d] = v[d];
    return 0;
}

/* --------------------------------------------------------------- batches */

typedef struct {
    const oracle_book* b;
    const float* x;
    int64_t n;
    int mode;
    int64_t* idx;
    int32_t* golay;
    int32_t* cls;
    double* score;
    int64_t next;
    pthread_mutex_t lock;
} batch_job;

static void* batch_worker(void* arg) {
    batch_job* j = (batch_job*)arg;
    for (;;) {
        pthread_mutex_lock(&j->lock);
        int64_t r = j->next++;
        pthread_mutex_unlock(&j->lock);
        if (r >= j->n) break;
        double x[DIM];
        for (int d = 0; d < DIM; ++d) x[d] = (double)j->x[r * DIM + d];
        int32_t g, k;
        double s;
        int64_t idx = oracle_quantize(j->b, x, j->mode, &g, &k, &s, NULL);
        j->idx[r] = idx;
        if (j->golay) j->golay[r] = g;
        if (j->cls) j->cls[r] = k;
        if (j->score) j->score[r] = s;
    }
    return NULL;
}

/* Quantize n fp32 rows with `threads` POSIX threads (rows handed out one at a
 * time).  golay/cls/score may be NULL. */
int oracle_quantize_batch(const oracle_book* b, const float* x, int64_t n, int mode, int threads, int64_t* idx,
                          int32_t* golay, int32_t* cls, double* score) {
    batch_job j;
    j.b = b; j.x = x; j.n = n; j.mode = mode; j.idx = idx; j.golay = golay; j.cls = cls; j.score = score;
    j.next = 0;
    pthread_mutex_init(&j.lock, NULL);
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    pthread_t th[256];
    for (int t = 0; t < threads; ++t) pthread_create(&th[t], NULL, batch_worker, &j);
    for (int t = 0; t < threads; ++t) pthread_join(th[t], NULL);
    pthread_mutex_destroy(&j.lock);
    return 0;
}

/* Batch codeword(): out is n*24 int32; returns the number of failed rows
 * (zero-filled).  oracle_codeword_batch_mt splits the rows into `threads`
 * contiguous ranges, one POSIX thread each. */
int64_t oracle_codeword_batch(const oracle_book* b, const int64_t* idx, int64_t n, int32_t* out) {
    int64_t bad = 0;
    for (int64_t r = 0; r < n; ++r) {
        if (oracle_codeword(b, idx[r], out + r * DIM)) {
            memset(out + r * DIM, 0, DIM * sizeof(int32_t));
            bad++;
        }
    }
    return bad;
}

typedef struct {
    const oracle_book* b;
    const int64_t* idx;
    int64_t n;
    int32_t* out;
    int64_t bad;
} codeword_job;

static void* codeword_worker(void* arg) {
    codeword_job* j = (codeword_job*)arg;
    j->bad = oracle_codeword_batch(j->b, j->idx, j->n, j->out);
    return NULL;
}

int64_t oracle_codeword_batch_mt(const oracle_book* b, const int64_t* idx, int64_t n, int32_t* out, int threads) {
    if (threads < 1) threads = 1;
    if (threads > 256) threads = 256;
    if ((int64_t)threads > n) threads = n > 0 ? (int)n : 1;
    pthread_t th[256];
    codeword_job jobs[256];
    const int64_t per = (n + threads - 1) / threads;
    for (int t = 0; t < threads; ++t) {
        const int64_t lo = per * t < n ? per * t : n, hi = per * (t + 1) < n ? per * (t + 1) : n;
        jobs[t].b = b; jobs[t].idx = idx + lo; jobs[t].n = hi - lo; jobs[t].out = out + lo * DIM; jobs[t].bad = 0;
        pthread_create(&th[t], NULL, codeword_worker, &jobs[t]);
    }
    int64_t bad = 0;
    for (int t = 0; t < threads; ++t) {
        pthread_join(th[t], NULL);
        bad += jobs[t].bad;
    }
    return bad;
}

/* Score of one given (Golay word, class) pair with the reference arithmetic;
 * used by tests that plant near-ties. */
double oracle_pair_score(const oracle_book* b, const double* x, int g, int k, int32_t* yout) {
    word_orders o;
    int y[DIM];
    const ocls* c = &b->cls[k];
    uint32_t word = b->golay[g];
    if (c->parity == 0) {
        if (b->golay_weight[g] != c->even_weight) return -INFINITY;
        compute_orders(x, word, &o, 1, 0);
        solve_even(x, c, &o, y);
    } else {
        compute_orders(x, word, &o, 0, 1);
        solve_odd(c, word, &o, y);
    }
    if (yout) for (int d = 0; d < DIM; ++d) yout[d] = y[d];
    return LATTICE_SCALE * ref_projection(x, y) - (double)c->shell;
}

double oracle_ref_projection(const double* x, const int32_t* y) {
    int yy[DIM];
    for (int d = 0; d < DIM; ++d) yy[d] = y[d];
    return ref_projection(x, yy);
}
