"""Emit straight-line CUDA scoring code for one Λ24 codebook (a class list).

For a fixed Golay word the best codeword of a class is fixed by sorting (the
reference's solve_even_subclass / solve_odd_subclass,
impl/leech_lattice_vector_quantizer.py:619-666), so its projection is a short
linear form in suffix sums of the sorted coordinates:

  odd class, signed values u1 > ... > uG (counts n_j, cum_j = n_1+...+n_j):
      proj = sum_{j<G} (u_j - u_{j+1}) * R[cum_j] + u_G * R[24]
      R[t] = sum of the t largest x'_i,  x' = x with signs flipped on the word
  even class of word weight w, f0 values a_1 > ... > a_H >= 0 (|v| = 0 mod 4),
  f1 values b_1 > ... > b_J (|v| = 2 mod 4):
      proj = sum_j (a_j - a_{j+1}) R0[cum0_j] + sum_j (b_j - b_{j+1}) R1[cum1_j]
             - 2 b_J * P[required]        (a_{H+1} = b_{J+1} = 0)
      R0/R1 = suffix sums of |x| outside / inside the word, P = sign-parity
      penalty (smallest |x| inside the word, or 0).

Each class costs one FFMA per distinct value; classes that share leading
terms share their FFMAs (the chains are emitted as a prefix trie, terms
ordered by how many classes use them), and class scores are folded with a
3-input max.  Every suffix-sum index is a compile-time constant so the sums
stay in registers.  The script also emits the window constants the kernel
needs for its error bound and a signature the host matches against a runtime
class list.

Angular specs (NAME:MIN:MAX:a) score the multi-shell shape of shape-gain
quantization instead: the correlation per unit norm, proj / sqrt(shell)
(no shell offset), so every coefficient of a shell is divided by
sqrt(shell) (rounded to fp32) and the chains start at zero.  All classes of
one shell share the factor, so the per-shell tries stay as they are.

Usage:  python gen_search.py OUT.cuh NAME:MIN_SHELL:MAX_SHELL[:a] [...]
"""
from __future__ import annotations

import math
import sys
from collections import Counter
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
sys.path.insert(0, str(HERE.parent.parent))

from llvq_paper_reproduction_b200.tables import codebook_classes  # noqa: E402

DIM = 24
WEIGHTS = (0, 8, 12, 16, 24)


def distinct_desc(values):
    out = []
    for v in sorted(values, reverse=True):
        if out and out[-1][0] == v:
            out[-1][1] += 1
        else:
            out.append([v, 1])
    return out


def odd_terms(leader):
    signed = [m if m % 4 == 1 else -m for m in leader]
    groups = distinct_desc(signed)
    terms, cum = [], 0
    for j, (u, n) in enumerate(groups):
        cum += n
        coef = u - groups[j + 1][0] if j + 1 < len(groups) else u
        terms.append((coef, cum))
    return terms


def even_terms(leader):
    f0 = [m for m in leader if m % 4 == 0]
    f1 = [m for m in leader if m % 4 == 2]
    t0, t1 = [], []
    g0 = distinct_desc(f0)
    cum = 0
    for j, (a, n) in enumerate(g0):
        cum += n
        nxt = g0[j + 1][0] if j + 1 < len(g0) else 0
        if a - nxt:
            t0.append((a - nxt, cum))
    g1 = distinct_desc(f1)
    cum = 0
    for j, (b, n) in enumerate(g1):
        cum += n
        nxt = g1[j + 1][0] if j + 1 < len(g1) else 0
        t1.append((b - nxt, cum))
    bmin = g1[-1][0] if g1 else 0
    return t0, t1, bmin, len(f1)


def class_chain(c):
    """The FFMA terms of one class as (array, coefficient, index) triples;
    array is R (odd), R0/R1 (even) or P0/P1 (even sign-parity penalty)."""
    if c.parity == 1:
        return [("R", coef, cum) for coef, cum in odd_terms(c.leader)]
    t0, t1, bmin, w = even_terms(c.leader)
    req = (sum(c.leader) % 8) // 4
    chain = [("R0", coef, cum) for coef, cum in t0] + [("R1", coef, cum) for coef, cum in t1]
    if w:
        chain.append((f"P{req}", -2 * bmin, 0))
    return chain


def ordered_chains(classes):
    """Order every class's terms by global frequency (most shared first) so
    classes of one shell share the longest possible FFMA prefix."""
    freq = Counter(t for c in classes for t in class_chain(c))
    return [sorted(class_chain(c), key=lambda t: (-freq[t], t)) for c in classes]


def term_bound(term):
    """Upper bound of |array value| in units of 2^Q (one coordinate <= 2^Q)."""
    arr, _, idx = term
    return 1 if arr.startswith("P") else idx


def shell_scale(shell, angular):
    """The factor an angular spec multiplies a shell's coefficients by
    (1/sqrt(shell), rounded to fp32), or 1."""
    return float(np.float32(1.0 / math.sqrt(shell))) if angular else 1.0


def scaled(coef, shell, angular):
    return float(np.float32(coef * shell_scale(shell, angular))) if angular else float(coef)


def window_constants(classes, chains, angular=False):
    """L1max, MG = max m*(G+2), AM = max sum_j sum_{i<=j} |c_i|*bound_i over
    the FFMA chain each class issues (in emitted order).  Angular specs have
    no shell offset (MG = 0) and round every coefficient once more, so AM
    also takes sum_i |c_i|*bound_i (bounds in units of 2^Q; the kernel
    multiplies AM by 2^-24 * 2^Q)."""
    l1max = mg = am = 0
    for c, chain in zip(classes, chains):
        l1max = max(l1max, sum(c.leader))
        acc = total = 0
        for t in chain:
            acc += abs(scaled(t[1], c.shell, angular)) * term_bound(t)
            total += acc
        if angular:
            total += acc  # coefficient rounding: sum_i |c_i| bound_i
        else:
            mg = max(mg, c.shell * (len(chain) + 2))
        am = max(am, total)
    return l1max, mg, int(math.ceil(am))


class _Emitter:
    """DFS over the prefix trie of FFMA chains, with 3-input max folding."""

    def __init__(self, min_shell, cands, angular=False):
        self.min_shell = min_shell
        self.cands = cands
        self.angular = angular
        self.lines = []
        self.tmp = 0
        self.pending = False

    def leaf(self, k, name, indent):
        if self.cands:
            self.lines.append(f"{indent}if ({name} >= thr) f({k}, {name});")
        elif not self.pending:
            self.pending = True
            self.lines.append(f"{indent}pend = {name};")
        else:
            self.lines.append(f"{indent}b = llvq_max3(b, pend, {name});")
            self.pending = False

    def run(self, items):
        """items: list of (class index, shell, ordered chain)."""
        trie = {}
        for k, shell, chain in items:
            node = trie.setdefault(shell, {"kids": {}, "ends": []})
            for t in chain:
                node = node["kids"].setdefault(t, {"kids": {}, "ends": []})
            node["ends"].append(k)

        def visit(node, parent, indent, shell):
            for term, child in node["kids"].items():
                arr, coef, idx = term
                self.tmp += 1
                name = f"t{self.tmp}"
                operand = arr if arr.startswith("P") else f"{arr}[{idx}]"
                c = scaled(coef, shell, self.angular)
                self.lines.append(f"{indent}{{ const float {name} = fmaf({c!r}f, {operand}, {parent});")
                for k in child["ends"]:
                    self.leaf(k, name, indent + "  ")
                visit(child, name, indent + "  ", shell)
                self.lines.append(f"{indent}}}")

        for shell, root in trie.items():
            assert not root["ends"]
            visit(root, "0.0f" if self.angular else f"nmk[{shell - self.min_shell}]", "    ", shell)
        if not self.cands and self.pending:
            self.lines.append("    b = fmaxf(b, pend);")
            self.pending = False
        return self.lines


class _PackedEmitter:
    """The same tries for a word pair (c, ~c) held in the two lanes of float2
    operands: FFMA2 below the roots (one instruction for both words, each lane
    rounded exactly like the scalar FFMA), two scalar FFMAs at a root (its
    addend, the shell offset, is a scalar), and per-lane 3-input maxima."""

    def __init__(self, min_shell, angular=False):
        self.min_shell = min_shell
        self.angular = angular
        self.lines = []
        self.tmp = 0
        self.pending = False

    def leaf(self, name, indent):
        if not self.pending:
            self.pending = True
            self.lines.append(f"{indent}pend = {name};")
        else:
            self.lines.append(f"{indent}b.x = llvq_max3(b.x, pend.x, {name}.x); "
                              f"b.y = llvq_max3(b.y, pend.y, {name}.y);")
            self.pending = False

    def run(self, items):
        trie = {}
        for k, shell, chain in items:
            node = trie.setdefault(shell, {"kids": {}, "ends": []})
            for t in chain:
                node = node["kids"].setdefault(t, {"kids": {}, "ends": []})
            node["ends"].append(k)

        def visit(node, parent, indent, shell, root):
            for term, child in node["kids"].items():
                arr, coef, idx = term
                operand = f"{arr}p" if arr.startswith("P") else f"{arr}p[{idx}]"
                self.tmp += 1
                name = f"t{self.tmp}"
                c = scaled(coef, shell, self.angular)
                if root:
                    self.lines.append(f"{indent}{{ const float2 {name} = make_float2(fmaf({c!r}f, {operand}.x, {parent}), "
                                      f"fmaf({c!r}f, {operand}.y, {parent}));")
                else:
                    self.lines.append(f"{indent}{{ const float2 {name} = __ffma2_rn(make_float2({c!r}f, {c!r}f), "
                                      f"{operand}, {parent});")
                for _ in child["ends"]:
                    self.leaf(name, indent + "  ")
                visit(child, name, indent + "  ", shell, False)
                self.lines.append(f"{indent}}}")

        for shell, root in trie.items():
            assert not root["ends"]
            visit(root, "0.0f" if self.angular else f"nmk[{shell - self.min_shell}]", "    ", shell, True)
        if self.pending:
            self.lines.append("    b.x = fmaxf(b.x, pend.x); b.y = fmaxf(b.y, pend.y);")
            self.pending = False
        return self.lines


# Golay words per weight; the scoring code a word runs is the odd classes'
# plus the even classes' of its weight.
WORDS_BY_WEIGHT = {0: 1, 8: 759, 12: 2576, 16: 759, 24: 1}
# CTA shape by the FFMAs per word of the scoring code (shell 32: 2112; shell
# 23: 667; shells 2..13: 495; shell 13: 111; shell 11: 77).  Up to
# SMALL_CODE the code fits the instruction cache as it is: 6 CTAs of 128
# threads, no realignment.  Up to LARGE_CODE: 3 CTAs of 256 threads whose
# warps realign at every pair (a barrier) so they share the cache.  Beyond:
# one 512-thread CTA per SM, 16 warps realigned (+44% at shell 32 over 256).
SMALL_CODE_FFMA_PER_WORD = 200
LARGE_CODE_FFMA_PER_WORD = 1000


def trie_size(items):
    """FFMAs of the per-shell prefix tries of (shell, chain) items."""
    roots, n = {}, 0
    for shell, chain in items:
        node = roots.setdefault(shell, {})
        for t in chain:
            if t not in node:
                node[t] = {}
                n += 1
            node = node[t]
    return n


def ffma_per_word(classes, chains):
    odd = trie_size([(c.shell, ch) for c, ch in zip(classes, chains) if c.parity == 1])
    total = 0
    for w, count in WORDS_BY_WEIGHT.items():
        even = trie_size([(c.shell, ch) for c, ch in zip(classes, chains)
                          if c.parity == 0 and even_terms(c.leader)[3] == w])
        total += count * (odd + even)
    return total / sum(WORDS_BY_WEIGHT.values())


def emit_spec(name, classes, angular=False):
    min_shell = min(c.shell for c in classes)
    max_shell = max(c.shell for c in classes)
    chains = ordered_chains(classes)
    fpw = ffma_per_word(classes, chains)
    threads, min_blocks = (128, 6) if fpw <= SMALL_CODE_FFMA_PER_WORD else \
        (256, 3) if fpw <= LARGE_CODE_FFMA_PER_WORD else (512, 1)
    lines = []
    L = lines.append
    l1max, mg, am = window_constants(classes, chains, angular)
    r0max = {w: 0 for w in WEIGHTS}
    has_w = {w: False for w in WEIGHTS}
    for c in classes:
        if c.parity == 0:
            t0, _, _, w = even_terms(c.leader)
            has_w[w] = True
            r0max[w] = max(r0max[w], max((cum for _, cum in t0), default=0))
    has_odd = any(c.parity == 1 for c in classes)
    L(f"struct Spec_{name} {{")
    L(f"  static constexpr int kNumClasses = {len(classes)};")
    L(f"  static constexpr int kMinShell = {min_shell};")
    L(f"  static constexpr int kNumShells = {max_shell - min_shell + 1};")
    L(f"  static constexpr int kL1Max = {l1max};")
    L(f"  static constexpr int kWinMG = {mg};")
    L(f"  static constexpr int kWinAM = {am};")
    L(f"  static constexpr bool kHasOdd = {'true' if has_odd else 'false'};")
    L(f"  static constexpr bool kAngular = {'true' if angular else 'false'};")
    L(f"  static constexpr int kCtaThreads = {threads};")
    L(f"  static constexpr int kCtaMinBlocks = {min_blocks};")
    L(f"  static constexpr bool kCtaRealign = {'true' if threads > 128 else 'false'};")
    for w in WEIGHTS:
        L(f"  static constexpr int kR0Max_w{w} = {r0max[w]};")
        L(f"  static constexpr bool kHasEven_w{w} = {'true' if has_w[w] else 'false'};")

    def items(parity, w=None):
        out = []
        for k, (c, ch) in enumerate(zip(classes, chains)):
            if c.parity != parity:
                continue
            if parity == 0 and even_terms(c.leader)[3] != w:
                continue
            out.append((k, c.shell, ch))
        return out

    L("  __device__ __forceinline__ static float odd_max(const float (&R)[25], const float* nmk) {")
    body = _Emitter(min_shell, False, angular).run(items(1))
    L("    float b = -INFINITY;" + (" float pend;" if body else ""))
    lines.extend(body)
    L("    (void)R; (void)nmk;")
    L("    return b;")
    L("  }")
    L("  __device__ __forceinline__ static float2 odd_max2(const float2 (&Rp)[25], const float* nmk) {")
    body = _PackedEmitter(min_shell, angular).run(items(1))
    L("    float2 b = make_float2(-INFINITY, -INFINITY);" + (" float2 pend;" if body else ""))
    lines.extend(body)
    L("    (void)Rp; (void)nmk;")
    L("    return b;")
    L("  }")
    # both words of a weight-12 pair run the weight-12 classes
    L("  __device__ __forceinline__ static float2 even_max2_w12(const float2 (&R0p)[25], const float2 (&R1p)[25], "
      "float2 P0p, float2 P1p, const float* nmk) {")
    body = _PackedEmitter(min_shell, angular).run(items(0, 12))
    L("    float2 b = make_float2(-INFINITY, -INFINITY);" + (" float2 pend;" if body else ""))
    lines.extend(body)
    L("    (void)R0p; (void)R1p; (void)P0p; (void)P1p; (void)nmk;")
    L("    return b;")
    L("  }")
    L("  template <class F>")
    L("  __device__ __forceinline__ static void odd_cands(const float (&R)[25], const float* nmk, float thr, F&& f) {")
    lines.extend(_Emitter(min_shell, True, angular).run(items(1)))
    L("    (void)R; (void)nmk; (void)thr; (void)f;")
    L("  }")
    for w in WEIGHTS:
        L(f"  __device__ __forceinline__ static float even_max_w{w}(const float (&R0)[25], const float (&R1)[25], "
          f"float P0, float P1, const float* nmk) {{")
        body = _Emitter(min_shell, False, angular).run(items(0, w))
        L("    float b = -INFINITY;" + (" float pend;" if body else ""))
        lines.extend(body)
        L("    (void)R0; (void)R1; (void)P0; (void)P1; (void)nmk;")
        L("    return b;")
        L("  }")
        L("  template <class F>")
        L(f"  __device__ __forceinline__ static void even_cands_w{w}(const float (&R0)[25], const float (&R1)[25], "
          f"float P0, float P1, const float* nmk, float thr, F&& f) {{")
        lines.extend(_Emitter(min_shell, True, angular).run(items(0, w)))
        L("    (void)R0; (void)R1; (void)P0; (void)P1; (void)nmk; (void)thr; (void)f;")
        L("  }")
    L("};")
    sig = [len(classes)]
    for c in classes:
        sig += [c.shell, c.parity] + list(c.leader)
    L(f"static const int kSig_{name}[] = {{{', '.join(map(str, sig))}}};")
    return lines


def main(argv):
    out = Path(argv[1])
    specs = []
    for arg in argv[2:]:
        parts = arg.split(":")
        specs.append((parts[0], int(parts[1]), int(parts[2]), len(parts) > 3 and parts[3] == "a"))
    lines = ["// Generated by gen_search.py from the codebook class lists -- do not edit.",
             "#pragma once", "#include <cmath>", "namespace llvq {", "namespace gen {"]
    for name, lo, hi, angular in specs:
        lines += emit_spec(name, codebook_classes(hi, min_shell=lo), angular)
    lines += ["}  // namespace gen", "}  // namespace llvq", ""]
    lines.append("#define LLVQ_FOR_EACH_SPEC(X) " + " ".join(f"X({name})" for name, _, _, _ in specs))
    text = "\n".join(lines) + "\n"
    if not out.exists() or out.read_text() != text:
        out.parent.mkdir(parents=True, exist_ok=True)
        out.write_text(text)


if __name__ == "__main__":
    main(sys.argv)
