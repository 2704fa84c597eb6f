"""The oracle (C restatement of the reference quantizer) against every pin
the reference has: its own outputs (fixtures made by running the Python
reference), the notebook golden indices, the Adoul-Barth leader table and the
theta series."""
from __future__ import annotations

import math

import numpy as np
import pytest

from conftest import f32, oracle_book
from oracle.oracle import golay_words, rank_even_signs, ref_projection

# notebooks/play_around_leech_lattice.ipynb cell 3: default_rng(0).normal((8,24))[0]
NOTEBOOK_ROW0 = {2: 126660, 3: 14156728, 4: 264775541, 5: 1846424557, 6: 26392167930, 8: 1003031253988,
                 10: 3696071938165, 13: 3696071938165}


def test_golay_order_and_weights():
    from llvq_paper_reproduction_b200.tables import golay_masks

    g = golay_words()
    assert tuple(int(v) for v in g) == golay_masks()
    w = np.array([bin(int(v)).count("1") for v in g])
    assert {k: int((w == k).sum()) for k in (0, 8, 12, 16, 24)} == {0: 1, 8: 759, 12: 2576, 16: 759, 24: 1}


@pytest.mark.parametrize("m", [2, 3, 4, 5, 8, 13])
def test_class_tables_match_reference(reference_tables, m):
    ref = reference_tables["tables"][str(m)]
    ob = oracle_book(m)
    assert ob.total_count == ref["total_count"]
    assert ob.n_classes == len(ref["classes"])
    for k, row in enumerate(ref["classes"]):
        ci = ob.class_info(k)
        assert (ci["shell"], ci["parity"], list(ci["leader"])) == (row["shell"], row["parity"], row["leader"])
        assert (ci["count"], ci["sign_count"], ci["permutation_count"], ci["golay_count"], ci["start"]) == \
            (row["count"], row["sign_count"], row["permutation_count"], row["golay_count"], row["start"])


def test_quantize_matches_reference_outputs(reference_cases):
    """Every quantize call recorded from the reference (225 calls: Gaussian,
    zeros, signed zeros, integer rows, exact ties, lattice points, midpoints,
    tiny, subnormal and huge rows)."""
    n = 0
    for case in reference_cases:
        x = f32(case["x"]).astype(np.float64)
        for m, res in case["results"].items():
            got = oracle_book(int(m)).quantize(x)
            assert got["index"] == res["index"], (case["name"], m)
            assert list(got["codeword"]) == res["codeword"], (case["name"], m)
            n += 1
    assert n == 225


def test_faithful_and_hoisted_modes_agree(reference_cases):
    ob = oracle_book(4)
    for case in reference_cases[:12]:
        x = f32(case["x"]).astype(np.float64)
        assert ob.quantize(x, mode=0)["index"] == ob.quantize(x, mode=1)["index"]


def test_codewords_match_reference(reference_tables):
    ob = oracle_book(13)
    for cw in reference_tables["codewords"]:
        assert list(ob.codeword(cw["index"])) == cw["codeword"]
        assert ob.encode(cw["codeword"]) == cw["index"]


@pytest.mark.parametrize("m,expected", sorted(NOTEBOOK_ROW0.items()))
def test_notebook_golden_indices(m, expected):
    x = np.random.default_rng(0).normal(size=(8, 24))[0]
    assert oracle_book(m).quantize(x)["index"] == expected
    assert oracle_book(m).quantize(x.astype(np.float32).astype(np.float64))["index"] == expected


def test_integer_input_notebook():
    # notebooks/test.ipynb: max_shell=12
    x = np.array([4, 7, 2, 8, 6, 1, 6, 5, 7, 2, 4, 6, 5, 9, 2, 6, 3, 8, 5, 7, 4, 11, 2, 8], dtype=np.float64)
    r = oracle_book(12).quantize(x)
    assert r["index"] == 42882272439546
    assert abs(r["score"] - 123.764502) < 1e-6


def test_figure1_golden_indices_m31():
    # notebooks/recreate_figure1_gaussian_sqnr.ipynb cell 11 (max_shell=31)
    ob = oracle_book(31)
    counts = {}
    for k in range(ob.n_classes):
        ci = ob.class_info(k)
        counts[ci["shell"]] = counts.get(ci["shell"], 0) + ci["count"]
    beta = math.sqrt(24.0 / (sum(2.0 * s * c for s, c in counts.items()) / ob.total_count))
    w = np.random.default_rng(0).normal(0.0, 1.0, size=(20, 24)).astype(np.float32)[0]
    assert ob.quantize((w / beta).astype(np.float64))["index"] == 121958412121151779
    shell_beta = float(np.linalg.norm(w) / math.sqrt(2.0 * 31))
    assert ob.quantize((w / shell_beta).astype(np.float64))["index"] == 5013492481700883026


def test_sign_rank_counting_equals_enumeration():
    rng = np.random.default_rng(3)
    ob = oracle_book(5)
    for _ in range(200):
        y = np.array(ob.codeword(int(rng.integers(ob.total_count))), dtype=np.int32)
        if y.sum() % 2 == 0 and np.count_nonzero(y) <= 16:
            assert rank_even_signs(y) == rank_even_signs(y, enumerate_masks=True)


def test_reference_projection_is_compensated():
    # CPython 3.12 sum() keeps the 1.0 that a naive left-to-right sum loses
    x = np.zeros(24)
    x[:3] = [1e100, 1.0, -1e100]
    assert ref_projection(x, np.ones(24, dtype=np.int32)) == 1.0
