"""The C-ABI library without a GPU: it loads, exports every symbol the public
header declares, and its host-side paths (codebook build, codeword, encode,
error mapping) behave like the reference."""
from __future__ import annotations

import re

import numpy as np
import pytest

from conftest import ROOT
from llvq_paper_reproduction_b200 import _native
from llvq_paper_reproduction_b200.tables import codebook_classes


def _book(m, lo=2, device=-1):
    cls = codebook_classes(m, min_shell=lo)
    return _native.NativeCodebook([c.shell for c in cls], [c.parity for c in cls], [c.leader for c in cls], device)


def test_exports_every_header_symbol():
    header = (ROOT / "include" / "llvq_b200.h").read_text()
    declared = set(re.findall(r"\b(llvq_[a-z0-9_]+)\s*\(", header))
    lib = _native.load()
    for name in declared:
        assert hasattr(lib, name), name
    assert declared == set(_native.EXPORTS)
    assert lib.llvq_version() >= 1


def test_host_codebook_matches_tables(reference_tables):
    for m in ("4", "13"):
        b = _book(int(m))
        assert b.total_count == reference_tables["tables"][m]["total_count"]
    assert _book(13).specialized and _book(4).specialized and not _book(3).specialized
    assert _book(13, 13).specialized


def test_host_codeword_and_encode(reference_tables):
    b = _book(13)
    for cw in reference_tables["codewords"]:
        assert list(b.codeword(cw["index"])) == cw["codeword"]
        assert b.encode(cw["codeword"]) == cw["index"]
    rng = np.random.default_rng(11)
    for i in rng.integers(0, b.total_count, size=3000):
        assert b.encode(b.codeword(int(i))) == int(i)


def test_error_mapping():
    b = _book(4)
    with pytest.raises(IndexError):
        b.codeword(b.total_count)
    with pytest.raises(IndexError):
        b.codeword(-1)
    with pytest.raises(ValueError):
        b.encode([1] * 24)  # norm 24 is not a shell norm
    with pytest.raises(ValueError):
        b.encode([2, 2] + [0] * 22)  # norm 8: no shell
    with pytest.raises(ValueError):  # host-only book has no device tables
        b.quantize(0, 1, 0, 0, 0, 0)
    with pytest.raises(ValueError):  # leader norm is not 16 * shell
        _native.NativeCodebook([2], [0], [[4, 4, 2] + [0] * 21])
    with pytest.raises(ValueError):  # classes out of shell order
        cls = codebook_classes(3)
        _native.NativeCodebook([c.shell for c in cls][::-1], [c.parity for c in cls][::-1],
                               [c.leader for c in cls][::-1])


def test_unsigned_indices_shells_2_32():
    """Shells 2..32 have 1.09e19 codewords: more than int64 holds (the
    reference's torch.long overflows) but fewer than 2^64 - 1, so indices are
    unsigned 64-bit (int64 arguments carry their two's-complement image, -1
    stays invalid).  Host decode and encode against the oracle, across 2^63."""
    from conftest import oracle_book

    assert _book(31).total_count == 7501022209994367600
    hb = _book(32)
    assert hb.total_count == 10918909325316807360
    ob = oracle_book(32)
    rng = np.random.default_rng(32)
    idx = [int(v) for v in rng.integers(0, 2**63, 10, dtype=np.uint64)]
    idx += [int(v) + 2**63 for v in rng.integers(0, hb.total_count - 2**63, 30, dtype=np.uint64)]
    idx += [2**63 - 1, 2**63, hb.total_count - 1]
    for i in idx:
        y = hb.codeword(i)
        assert y == ob.codeword(i)
        assert hb.encode(y) == i
    with pytest.raises(IndexError):
        hb.codeword(hb.total_count)


def test_api_class_host_paths():
    from llvq_paper_reproduction_b200 import LeechLatticeVectorQuantizerGpu

    q = LeechLatticeVectorQuantizerGpu(max_shell=4, use_cache=False, device="cpu")
    r = q.unrank(264775541)
    assert (r.shell, r.class_index, r.class_local_index) == (4, 2, 48838565)
    assert q.codeword(264775541) == (0, -2, 2, 0, 0, 0, 2, 2, -2, -2, -2, 0, -4, 0, -2, 0, -2, 0, 0, 2, 0, 2, -2, 0)
    assert q.encode_codeword(q.codeword(12345)) == 12345
    loc = q.decompose_local_index(q.unrank(126660))
    assert (loc.golay_choice, loc.sign_choice) == (loc.golay_choice, 0)
    with pytest.raises(ValueError):
        q.quantize([0.0] * 24)  # tensor paths need CUDA, as in the reference
