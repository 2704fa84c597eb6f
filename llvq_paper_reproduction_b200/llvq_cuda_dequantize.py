"""Drop-in for impl/llvq_cuda_dequantize.py (dmnunez1993/llvq-paper-reproduction).

``dequantize_lattice_cuda(indices, out, meta, comb)`` keeps the reference
launcher's signature (impl/llvq_cuda_dequantize.py:221-261): int64 indices
[N] in, int64 integer codewords [N, 24] written into the caller's ``out``,
``meta`` the dict of LeechLatticeVectorQuantizerGpu._codeword_cuda_metadata
(impl/leech_lattice_vector_quantizer_gpu.py:424-518).  It calls the C ABI of
the in-tree sm_100a library (llvq_dequantize_lattice) on torch's current
stream.  As in the reference, range checking is the caller's job; an index
outside the codebook decodes to a zero row.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _native



def classes_from_codeword_meta(meta: dict) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """(shell, parity, leader[n,24] descending) from _codeword_cuda_metadata."""
    parity = meta["parity"].detach().cpu().numpy().astype(np.int32)
    cols = {k: meta[k].detach().cpu().numpy() for k in
            ("f0_counts", "f0_values", "f1_counts", "f1_values", "odd_counts", "odd_values")}
    n = parity.shape[0]
    leaders = np.zeros((n, 24), dtype=np.int32)
    shells = np.zeros(n, dtype=np.int32)
    for k in range(n):
        parts = ("odd",) if parity[k] else ("f0", "f1")
        vals = []
        for p in parts:
            for v, c in zip(cols[f"{p}_values"][k], cols[f"{p}_counts"][k]):
                vals += [int(v)] * int(c)
        if len(vals) != 24:
            raise ValueError(f"class {k}: metadata does not describe 24 coordinates")
        leaders[k] = sorted(vals, reverse=True)
        sq = sum(v * v for v in vals)
        if sq % 16:
            raise ValueError(f"class {k}: leader norm is not a shell norm")
        shells[k] = sq // 16
    return shells, parity, leaders


# Every metadata tensor the class list is read from (see classes_from_codeword_meta).
_BOOKS = _native.MetadataBooks(("parity", "f0_counts", "f0_values", "f1_counts", "f1_values", "odd_counts",
                                "odd_values"), classes_from_codeword_meta)


def _book_for(meta: dict, device: torch.device) -> _native.NativeCodebook:
    return _BOOKS.get(meta, device.index)


def dequantize_lattice_cuda(indices: torch.Tensor, out: torch.Tensor, meta: dict, comb: torch.Tensor) -> torch.Tensor:
    """Integer codewords of ``indices`` into ``out`` ([N, 24] int64)."""
    if indices.device.type != "cuda":
        raise ValueError("indices must be a CUDA tensor")
    n = indices.numel()
    if indices.dtype != torch.long or not indices.is_contiguous():
        raise ValueError("indices must be a contiguous int64 tensor")
    if out.device != indices.device or out.dtype != torch.long or out.shape != (n, 24) or not out.is_contiguous():
        raise ValueError("out must be a contiguous int64 [N, 24] tensor on the indices' device")
    device = indices.device if indices.device.index is not None else \
        torch.device("cuda", torch.cuda.current_device())
    book = _book_for(meta, device)
    with torch.cuda.device(device):
        book.dequantize_lattice(indices.data_ptr(), n, out.data_ptr(), None, torch.cuda.current_stream().cuda_stream)
    return out
