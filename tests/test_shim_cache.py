"""The launcher shims cache a codebook per metadata dict without reading the
device tensors back (which would synchronise every launch).  An entry may only
be reused while the very tensors it was built from are alive and unmodified:
a different dict whose tensors sit at the same addresses must get its own
class list."""
from __future__ import annotations

import torch

from llvq_paper_reproduction_b200 import _native


def _books(monkeypatch):
    calls = []

    def classes(meta):
        calls.append(int(meta["a"][0]))
        return [int(meta["a"][0])], [0], [[0] * 24]

    monkeypatch.setattr(_native, "codebook_for", lambda s, p, l, d: ("book", tuple(s), d))
    return _native.MetadataBooks(("a", "b"), classes), calls


def test_same_dict_is_cached(monkeypatch):
    books, calls = _books(monkeypatch)
    meta = {"a": torch.tensor([3, 4]), "b": torch.tensor([1])}
    assert books.get(meta, 0) == ("book", (3,), 0)
    assert books.get(meta, 0) == ("book", (3,), 0)
    assert calls == [3]
    assert books.get(meta, 1) == ("book", (3,), 1)  # per device
    assert calls == [3, 3]


def test_new_tensors_at_the_same_address_rebuild(monkeypatch):
    books, calls = _books(monkeypatch)
    a = torch.tensor([3, 4])
    meta = {"a": a, "b": torch.tensor([1])}
    books.get(meta, 0)
    # another dict whose tensor objects share the first dict's memory
    # (same data_ptr, as after a free and reallocation), other contents
    other = {"a": a.view_as(a), "b": meta["b"].view_as(meta["b"])}
    assert other["a"].data_ptr() == a.data_ptr()
    other["a"][0] = 7
    assert books.get(other, 0) == ("book", (7,), 0)
    assert calls == [3, 7]


def test_in_place_update_rebuilds(monkeypatch):
    books, calls = _books(monkeypatch)
    meta = {"a": torch.tensor([3, 4]), "b": torch.tensor([1])}
    books.get(meta, 0)
    meta["a"].fill_(5)  # same object, same address, new contents
    assert books.get(meta, 0) == ("book", (5,), 0)
    assert calls == [3, 5]
