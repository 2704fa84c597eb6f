"""Host-side codebook tables for the Leech lattice Λ24 quantizer.

This is the table builder that sits under the GPU quantizer API: the extended
Golay code G24 in the reference's lexicographic order, the class leaders of
every shell generated from the shell equation, the per-class local structure
(compatible Golay words, sign count, permutation count), shell/class offsets and
the theta-series check.  Names, fields and orderings follow the reference
module impl/leech_lattice_vector_quantizer_gpu.py (dmnunez1993/llvq-paper-
reproduction) so code written against it keeps working:

    ClassLeader / RankedCodeword / LocalDecomposition /
    ClassLocalStructure ........................... _gpu.py:37-119
    build_local_structure ......................... _gpu.py:570-601
    generate_class_leaders (+ cache) .............. _gpu.py:604-682
    generate_shell_class_leaders .................. _gpu.py:685-690
    extended_golay_codewords ...................... _gpu.py:1048-1067
    leech_shell_counts ............................ _gpu.py:1070-1077

Everything here is host-only integer work done once per codebook; the
per-vector hot path lives in the CUDA library.
"""
from __future__ import annotations

import math
import pickle
from dataclasses import dataclass
from functools import lru_cache
from pathlib import Path
from time import perf_counter
from typing import Iterator, Sequence

DIM = 24
LATTICE_SCALE = 1.0 / math.sqrt(8.0)
CLASS_LEADER_CACHE_VERSION = 1
_GOLAY_WEIGHTS = (0, 8, 12, 16, 24)


@dataclass(frozen=True)
class ClassLeader:
    """Absolute-value leader of one class: multiplicity of each magnitude.

    Field order matches the reference (shell, parity, count, then the
    multiplicities of |8|,|6|,|5|,|4|,|3|,|2|,|1|,|0|, then any other
    magnitudes as (magnitude, count) pairs, descending)."""

    shell: int
    parity: str
    count: int
    mult_abs8: int
    mult_abs6: int
    mult_abs5: int
    mult_abs4: int
    mult_abs3: int
    mult_abs2: int
    mult_abs1: int
    mult_abs0: int
    extra_multiplicities: tuple[tuple[int, int], ...] = ()

    @property
    def multiplicities(self) -> dict[int, int]:
        named = ((8, self.mult_abs8), (6, self.mult_abs6), (5, self.mult_abs5), (4, self.mult_abs4),
                 (3, self.mult_abs3), (2, self.mult_abs2), (1, self.mult_abs1), (0, self.mult_abs0))
        out = dict(named)
        out.update(dict(self.extra_multiplicities))
        return {mag: cnt for mag, cnt in out.items() if cnt}

    @property
    def leader(self) -> tuple[int, ...]:
        values = [mag for mag, cnt in sorted(self.multiplicities.items(), reverse=True) for _ in range(cnt)]
        if len(values) != DIM:
            raise ValueError(f"leader has {len(values)} coordinates, expected {DIM}")
        return tuple(values)

    @property
    def even_weight(self) -> int:
        """Number of coordinates with |v| = 2 (mod 4)."""
        return sum(cnt for mag, cnt in self.multiplicities.items() if mag % 4 == 2)

    @property
    def nonzero_count(self) -> int:
        return DIM - self.mult_abs0


@dataclass(frozen=True)
class RankedCodeword:
    global_index: int
    shell: int
    shell_local_index: int
    class_index: int
    class_local_index: int
    class_offset: int
    leader: ClassLeader


@dataclass(frozen=True)
class LocalDecomposition:
    golay_choice: int
    golay_codeword: tuple[int, ...]
    sign_choice: int
    permutation_choice: int


@dataclass(frozen=True)
class ClassLocalStructure:
    shell: int
    class_index: int
    leader: ClassLeader
    golay_codeword_indices: tuple[int, ...]
    sign_count: int
    permutation_count: int

    @property
    def count(self) -> int:
        return len(self.golay_codeword_indices) * self.sign_count * self.permutation_count


# The Adoul-Barth small-shell table (m = 2..4) the reference compares its
# generated leaders against (_gpu.py:126-142).  Columns: |8| |6| |5| |4| |3| |2| |1| |0|.
TABLE_CLASS_LEADERS_REFERENCE: tuple[ClassLeader, ...] = tuple(
    ClassLeader(shell, parity, count, *mults)
    for shell, parity, count, mults in (
        (2, "even", 1104, (0, 0, 0, 2, 0, 0, 0, 22)),
        (2, "even", 97152, (0, 0, 0, 0, 0, 8, 0, 16)),
        (2, "odd", 98304, (0, 0, 0, 0, 1, 0, 23, 0)),
        (3, "even", 3108864, (0, 0, 0, 1, 0, 8, 0, 15)),
        (3, "even", 5275648, (0, 0, 0, 0, 0, 12, 0, 12)),
        (3, "odd", 98304, (0, 0, 1, 0, 0, 0, 23, 0)),
        (3, "odd", 8290304, (0, 0, 0, 0, 3, 0, 21, 0)),
        (4, "even", 170016, (0, 0, 0, 4, 0, 0, 0, 20)),
        (4, "even", 48, (1, 0, 0, 0, 0, 0, 0, 23)),
        (4, "even", 46632960, (0, 0, 0, 2, 0, 8, 0, 14)),
        (4, "even", 777216, (0, 1, 0, 0, 0, 7, 0, 16)),
        (4, "even", 126615552, (0, 0, 0, 1, 0, 12, 0, 11)),
        (4, "even", 24870912, (0, 0, 0, 0, 0, 16, 0, 8)),
        (4, "odd", 24870912, (0, 0, 1, 0, 2, 0, 21, 0)),
        (4, "odd", 174096384, (0, 0, 0, 0, 5, 0, 19, 0)),
    )
)


# ---------------------------------------------------------------- Golay code

@lru_cache(maxsize=1)
def extended_golay_codewords() -> tuple[tuple[int, ...], ...]:
    """All 4096 words of the extended binary Golay code G24, as 0/1 tuples in
    lexicographic order (coordinate 0 compared first).

    The code is the cyclic [23,12,7] Golay code with generator polynomial
    g(x) = x^11 + x^9 + x^7 + x^6 + x^5 + x + 1 plus an overall parity bit;
    the sorted order is what the codebook index of odd classes counts in."""
    g = 0b101011100011  # bits 11,9,7,6,5,1,0
    words = []
    for msg in range(4096):
        c = 0
        m = msg
        shift = 0
        while m:
            if m & 1:
                c ^= g << shift
            m >>= 1
            shift += 1
        bits = [(c >> i) & 1 for i in range(23)]
        bits.append(sum(bits) & 1)
        words.append(tuple(bits))
    words.sort()
    return tuple(words)


@lru_cache(maxsize=1)
def golay_masks() -> tuple[int, ...]:
    """Golay words as 24-bit masks (bit d = coordinate d), lexicographic order."""
    return tuple(sum(b << d for d, b in enumerate(w)) for w in extended_golay_codewords())


@lru_cache(maxsize=1)
def _golay_weight_counts() -> dict[int, int]:
    out: dict[int, int] = {}
    for w in extended_golay_codewords():
        out[sum(w)] = out.get(sum(w), 0) + 1
    return out


# ------------------------------------------------------------- combinatorics

def multiset_permutation_count(multiplicities: dict[int, int]) -> int:
    """Number of distinct orderings of a multiset: n! / prod(c!)."""
    n = sum(multiplicities.values())
    out = math.factorial(n)
    for c in multiplicities.values():
        out //= math.factorial(c)
    return out


def _residue_counts(leader: ClassLeader, modulus: int, residues: tuple[int, ...]) -> dict[int, int]:
    """Magnitude counts of the leader restricted to magnitudes whose residue
    modulo `modulus` is one of `residues` (an even class splits into its
    |v| = 0 and |v| = 2 (mod 4) parts; an odd class keeps every magnitude)."""
    return {m: c for m, c in leader.multiplicities.items() if m % modulus in residues}


# ------------------------------------------------------------- class leaders

# Word positions by weight (and all positions) of a Golay word list, shared by
# every class built from the same list: one pass over the 4096 words instead
# of one per class, and one tuple per weight instead of one per class.
_WORDS_BY_WEIGHT: dict[int, tuple[Sequence[tuple[int, ...]], dict[int, tuple[int, ...]]]] = {}


def _words_by_weight(golay_codewords: Sequence[tuple[int, ...]]) -> dict[int, tuple[int, ...]]:
    hit = _WORDS_BY_WEIGHT.get(id(golay_codewords))
    if hit is not None and hit[0] is golay_codewords:
        return hit[1]
    groups: dict[int, list[int]] = {}
    for i, c in enumerate(golay_codewords):
        groups.setdefault(sum(c), []).append(i)
    table = {w: tuple(ix) for w, ix in groups.items()}
    table[-1] = tuple(range(len(golay_codewords)))
    _WORDS_BY_WEIGHT[id(golay_codewords)] = (golay_codewords, table)  # keeps the list alive: ids stay unique
    return table


def build_local_structure(shell: int, class_index: int, leader: ClassLeader,
                          golay_codewords: Sequence[tuple[int, ...]]) -> ClassLocalStructure:
    """Compatible Golay words, sign count and permutation count of one class.

    Even class: the words whose weight equals the number of |v| = 2 (mod 4)
    coordinates; 2^(nonzero-1) sign patterns (2^nonzero when that weight is 0,
    none when it is 0 and the leader sum is not 0 mod 8); magnitudes permuted
    independently inside and outside the word.  Odd class: every word, one sign
    pattern, all magnitude orderings."""
    words = _words_by_weight(golay_codewords)
    if leader.parity == "even":
        w = leader.even_weight
        golay = words.get(w, ())
        if w == 0 and sum(leader.leader) % 8:
            signs = 0
        else:
            signs = 1 << (leader.nonzero_count - (0 if w == 0 else 1))
        perms = multiset_permutation_count(_residue_counts(leader, 4, (0,))) * \
            multiset_permutation_count(_residue_counts(leader, 4, (2,)))
    elif leader.parity == "odd":
        golay = words[-1]
        signs = 1
        perms = multiset_permutation_count(_residue_counts(leader, 2, (1,)))
    else:
        raise ValueError(f"unknown parity {leader.parity!r}")
    return ClassLocalStructure(shell, class_index, leader, golay, signs, perms)


def _class_cardinality(shell: int, parity: str, mults: dict[int, int]) -> int:
    counts = _golay_weight_counts()
    if parity == "odd":
        return 4096 * multiset_permutation_count(mults)
    w = sum(c for m, c in mults.items() if m % 4 == 2)
    words = counts.get(w, 0)
    if not words:
        return 0
    total = sum(m * c for m, c in mults.items())
    nonzero = sum(c for m, c in mults.items() if m)
    if w == 0 and total % 8:
        return 0
    signs = 1 << (nonzero - (0 if w == 0 else 1))
    f0 = {m: c for m, c in mults.items() if m % 4 == 0}
    f1 = {m: c for m, c in mults.items() if m % 4 == 2}
    return words * signs * multiset_permutation_count(f0) * multiset_permutation_count(f1)


def _make_leader(shell: int, parity: str, mults: dict[int, int], count: int) -> ClassLeader:
    named = (8, 6, 5, 4, 3, 2, 1, 0)
    extra = tuple(sorted(((m, c) for m, c in mults.items() if m not in named and c), reverse=True))
    return ClassLeader(shell, parity, count, *(mults.get(m, 0) for m in named), extra)


def _magnitude_profiles(mags: Sequence[int], slots: int, square_sum: int) -> Iterator[dict[int, int]]:
    """Every way to fill `slots` coordinates with magnitudes from `mags`
    (ascending) so that the squares add up to `square_sum`."""
    stack = [(len(mags) - 1, slots, square_sum, {})]
    while stack:
        i, left, sq, chosen = stack.pop()
        if i < 0:
            if left == 0 and sq == 0:
                yield chosen
            continue
        m = mags[i]
        top = left if m == 0 else min(left, sq // (m * m))
        for c in range(top + 1):
            nxt = dict(chosen)
            if c:
                nxt[m] = c
            stack.append((i - 1, left - c, sq - c * m * m, nxt))


def _leader_sort_key(row: ClassLeader):
    return (row.leader, 0 if row.parity == "even" else 1, row.count)


def generate_shell_class_leaders(shell: int) -> tuple[ClassLeader, ...]:
    """All non-empty classes of shell m: vectors with squared norm 16m whose
    coordinates are all even or all odd, grouped by sorted absolute values,
    in the reference's class order (leader tuple, even before odd, count)."""
    target = 16 * shell
    top = math.isqrt(target)
    rows = []
    for parity, first in (("even", 0), ("odd", 1)):
        mags = tuple(range(first, top + 1, 2))
        for mults in _magnitude_profiles(mags, DIM, target):
            count = _class_cardinality(shell, parity, mults)
            if count:
                rows.append(_make_leader(shell, parity, mults, count))
    return tuple(sorted(rows, key=_leader_sort_key))


def _cache_path(cache_dir: str | Path | None, shell: int) -> Path | None:
    if cache_dir is None:
        return None
    return Path(cache_dir) / f"class_leaders_v{CLASS_LEADER_CACHE_VERSION}_shell{shell}.pkl"


def generate_shell_class_leaders_cached(shell: int, cache_dir: str | Path | None = ".llvq_cache"
                                        ) -> tuple[tuple[ClassLeader, ...], str]:
    """Leaders of one shell through a versioned pickle cache (atomic write;
    unreadable or stale files are regenerated)."""
    path = _cache_path(cache_dir, shell)
    if path is not None and path.exists():
        try:
            with path.open("rb") as fh:
                payload = pickle.load(fh)
            if (payload.get("version") == CLASS_LEADER_CACHE_VERSION and payload.get("shell") == shell
                    and isinstance(payload.get("leaders"), tuple)):
                return tuple(ClassLeader(*row) if not isinstance(row, ClassLeader) else row
                             for row in payload["leaders"]), "loaded cached"
        except (OSError, pickle.PickleError, AttributeError, EOFError, TypeError, ValueError):
            pass
    leaders = generate_shell_class_leaders(shell)
    if path is not None:
        try:
            path.parent.mkdir(parents=True, exist_ok=True)
            tmp = path.with_suffix(path.suffix + ".tmp")
            with tmp.open("wb") as fh:
                pickle.dump({"version": CLASS_LEADER_CACHE_VERSION, "shell": shell,
                             "leaders": tuple(tuple(getattr(r, f) for f in r.__dataclass_fields__) for r in leaders)},
                            fh, protocol=pickle.HIGHEST_PROTOCOL)
            tmp.replace(path)
        except OSError:
            pass  # a read-only cache directory only costs regeneration time
    return leaders, "generated"


def generate_class_leaders(max_shell: int, cache_dir: str | Path | None = ".llvq_cache", use_cache: bool = True,
                           verbose: bool = False, min_shell: int = 2) -> tuple[ClassLeader, ...]:
    """Class leaders of shells min_shell..max_shell (the reference uses 2..max_shell)."""
    out: list[ClassLeader] = []
    for shell in range(min_shell, max_shell + 1):
        t0 = perf_counter()
        if use_cache:
            rows, status = generate_shell_class_leaders_cached(shell, cache_dir)
        else:
            rows, status = generate_shell_class_leaders(shell), "generated"
        if verbose:
            print(f"{status} class leaders for shell m={shell}: {len(rows)} classes in "
                  f"{perf_counter() - t0:.3f}s", flush=True)
        out.extend(rows)
    return tuple(out)


def compare_with_reference(max_shell: int = 4) -> bool:
    """Generated leaders equal the Adoul-Barth table for shells <= min(max_shell, 4)."""
    key = lambda r: (r.shell,) + _leader_sort_key(r)  # noqa: E731
    gen = sorted((r for r in generate_class_leaders(max_shell, use_cache=False) if r.shell <= max_shell), key=key)
    ref = sorted((r for r in TABLE_CLASS_LEADERS_REFERENCE if r.shell <= max_shell), key=key)
    return gen == ref


# ------------------------------------------------------------- theta series

def _sigma3(n: int) -> int:
    return sum(d ** 3 for d in range(1, n + 1) if n % d == 0)


def _poly_mul(a: Sequence[int], b: Sequence[int], deg: int) -> list[int]:
    out = [0] * (deg + 1)
    for i, ai in enumerate(a[:deg + 1]):
        if ai:
            for j, bj in enumerate(b[:deg + 1 - i]):
                out[i + j] += ai * bj
    return out


def leech_shell_counts(max_shell: int) -> dict[int, int]:
    """Number of Λ24 vectors of squared norm 2m (shell m): the coefficients of
    the theta series E4^3 - 720 Δ."""
    deg = max_shell
    e4 = [1] + [240 * _sigma3(n) for n in range(1, deg + 1)]
    e4_3 = _poly_mul(_poly_mul(e4, e4, deg), e4, deg)
    prod = [1] + [0] * deg  # prod_{n>=1} (1 - q^n)^24
    for n in range(1, deg + 1):
        factor = [0] * (deg + 1)
        for k in range(0, deg // n + 1):
            if k > 24:
                break
            factor[n * k] = (-1) ** k * math.comb(24, k)
        prod = _poly_mul(prod, factor, deg)
    delta = [0] + prod[:deg]
    return {m: e4_3[m] - 720 * delta[m] for m in range(2, max_shell + 1)}


# ------------------------------------------------------------ flat codebook

@dataclass(frozen=True)
class FlatClass:
    """One class in global order with everything the device tables need."""
    shell: int
    parity: int              # 0 even, 1 odd
    leader: tuple[int, ...]  # magnitudes, descending
    start: int               # global index of its first codeword
    count: int
    golay_count: int
    sign_count: int
    permutation_count: int


def flatten(classes_by_shell: dict[int, Sequence[ClassLeader]], shell_offsets: dict[int, int],
            class_offsets: dict[int, Sequence[int]], local_structures) -> list[FlatClass]:
    out = []
    for shell in sorted(classes_by_shell):
        for i, st in enumerate(local_structures[shell]):
            out.append(FlatClass(shell, 0 if st.leader.parity == "even" else 1, st.leader.leader,
                                 shell_offsets[shell] + class_offsets[shell][i], st.count,
                                 len(st.golay_codeword_indices), st.sign_count, st.permutation_count))
    return out


def codebook_classes(max_shell: int, min_shell: int = 2) -> list[FlatClass]:
    """Flat class list of shells min_shell..max_shell in index order (no cache)."""
    words = extended_golay_codewords()
    out = []
    cursor = 0
    for shell in range(min_shell, max_shell + 1):
        for i, row in enumerate(generate_shell_class_leaders(shell)):
            st = build_local_structure(shell, i, row, words)
            out.append(FlatClass(shell, 0 if row.parity == "even" else 1, row.leader, cursor, st.count,
                                 len(st.golay_codeword_indices), st.sign_count, st.permutation_count))
            cursor += st.count
    return out
