"""The table-driven decoder (the tables and the decode code the GPU kernels
use, run on the host through llvq_codeword_batch_host) against the oracle's
restatement of the reference codeword(): every class's first, last and
middle index plus random ones, on the codebooks whose tables are built."""
from __future__ import annotations

import numpy as np
import pytest

from conftest import oracle_book


def _book(lo: int, hi: int):
    from llvq_paper_reproduction_b200 import LeechLatticeVectorQuantizerGpu

    return LeechLatticeVectorQuantizerGpu(max_shell=hi, min_shell=lo, use_cache=False, device="cpu")


@pytest.mark.parametrize("lo,hi", [(2, 4), (2, 13), (11, 11), (2, 2), (5, 5), (13, 13)])
def test_table_decoder_matches_oracle(lo, hi):
    q = _book(lo, hi)
    hb = q._host()
    info = hb.tables()
    assert info["tabulated"] and info["max_lookups"] <= 4  # two searches, then a tail per part
    rng = np.random.default_rng(lo * 100 + hi)
    starts = [q.shell_offsets[s] + o for s in q.classes_by_shell for o in q.class_offsets[s]]
    counts = [st.count for s in q.classes_by_shell for st in q.local_structures[s]]
    picks = [rng.integers(0, q.total_count, 20000)]
    for st, c in zip(starts, counts):
        picks.append(np.array([st, st + c - 1, st + c // 2], dtype=np.int64))
        picks.append(st + rng.integers(0, c, 8))
    idx = np.concatenate(picks)
    got, bad = hb.codeword_batch(idx)
    assert bad == 0
    np.testing.assert_array_equal(got, oracle_book(hi, lo).codeword_batch(idx, threads=0))
    # out of range: zero rows, counted
    got, bad = hb.codeword_batch(np.array([-1, q.total_count], dtype=np.int64))
    assert bad == 2 and not got.any()


def test_large_codebooks_fall_back_to_arithmetic_unranking():
    """Shell 23 alone has parts too large to tabulate; its decoder stays the
    arithmetic one (checked on the GPU against the oracle elsewhere)."""
    assert not _book(23, 23)._host().tables()["tabulated"]
