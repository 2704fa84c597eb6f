"""Host-side table builder of the package against the reference's tables."""
from __future__ import annotations

import dataclasses

import numpy as np
import pytest

from conftest import golden
from llvq_paper_reproduction_b200 import tables as T


@pytest.mark.parametrize("m", [2, 3, 4, 5, 8, 13])
def test_codebook_classes_match_reference(reference_tables, m):
    ref = reference_tables["tables"][str(m)]
    cls = T.codebook_classes(m)
    assert len(cls) == len(ref["classes"])
    for c, r in zip(cls, ref["classes"]):
        assert c.shell == r["shell"] and ("odd" if c.parity else "even") == r["parity"]
        assert list(c.leader) == r["leader"]
        assert (c.count, c.golay_count, c.sign_count, c.permutation_count, c.start) == \
            (r["count"], r["golay_count"], r["sign_count"], r["permutation_count"], r["start"])
    assert sum(c.count for c in cls) == ref["total_count"]


def test_adoul_barth_table_and_theta():
    assert T.compare_with_reference(4)
    counts = T.leech_shell_counts(13)
    assert counts[2] == 196560 and counts[3] == 16773120 and counts[13] == 169931095326720


def test_leader_cache_roundtrip(tmp_path):
    a = T.generate_class_leaders(6, cache_dir=tmp_path)
    b = T.generate_class_leaders(6, cache_dir=tmp_path)  # loaded from the cache
    assert [dataclasses.astuple(r) for r in a] == [dataclasses.astuple(r) for r in b]
    (tmp_path / "class_leaders_v1_shell3.pkl").write_bytes(b"corrupt")
    c = T.generate_class_leaders(6, cache_dir=tmp_path)  # corrupt file is regenerated
    assert [dataclasses.astuple(r) for r in a] == [dataclasses.astuple(r) for r in c]


def _meta_tensors(d):
    import torch

    out = {}
    for k, v in d.items():
        out[k] = torch.tensor(v["data"], dtype=getattr(torch, v["dtype"])) if isinstance(v, dict) else v
    return out


@pytest.mark.parametrize("m", ["4", "13"])
def test_shim_metadata_parsing(m):
    """The shims rebuild the exact class list from the reference's own
    metadata dicts (recorded from LeechLatticeVectorQuantizerGpu)."""
    from llvq_paper_reproduction_b200.llvq_cuda_dequantize import classes_from_codeword_meta
    from llvq_paper_reproduction_b200.llvq_cuda_quantize import classes_from_quantize_meta

    meta = golden("reference_metadata.json")["shells"][m]
    want = T.codebook_classes(int(m))
    for shell, parity, leaders in (classes_from_quantize_meta(_meta_tensors(meta["quantize_meta"])),
                                   classes_from_codeword_meta(_meta_tensors(meta["codeword_meta"]))):
        assert list(shell) == [c.shell for c in want]
        assert list(parity) == [c.parity for c in want]
        assert np.array_equal(leaders, np.array([c.leader for c in want]))


def test_generated_window_constants():
    import sys
    sys.path.insert(0, str(T.Path(T.__file__).parent / "csrc"))
    import gen_search

    cls = T.codebook_classes(13)
    l1, mg, am = gen_search.window_constants(cls, gen_search.ordered_chains(cls))
    assert l1 == 70 and mg > 0 and am > 0
    # every exact suffix sum fits fp32's 24-bit significand: 24 * 2^19 < 2^24
    assert 24 * 2 ** 19 < 2 ** 24
