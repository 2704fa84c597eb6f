"""Drop-in for impl/llvq_cuda_quantize.py (dmnunez1993/llvq-paper-reproduction).

``quantize_lattice_cuda`` keeps the reference launcher's signature and
argument meaning (impl/llvq_cuda_quantize.py:544-602): it takes the caller's
preallocated outputs and the metadata dicts of
LeechLatticeVectorQuantizerGpu._quantize_cuda_metadata / _codeword_cuda_metadata,
and raises ValueError for a non-CUDA or non-fp32 ``x``.  Instead of JIT-
compiling an NVRTC kernel it calls the C ABI of the in-tree sm_100a library
(llvq_quantize) on torch's current stream.  Results are the reference CPU
quantizer's indices, bit-exact.
"""
from __future__ import annotations

import numpy as np
import torch

from . import _native



def classes_from_quantize_meta(meta: dict) -> tuple[np.ndarray, np.ndarray, np.ndarray]:
    """(shell, parity, leader[n,24] descending) from _quantize_cuda_metadata
    (impl/leech_lattice_vector_quantizer_gpu.py:345-411)."""
    parity = meta["class_parity"].detach().cpu().numpy().astype(np.int32)
    shell = meta["class_shell"].detach().cpu().numpy().astype(np.int64).astype(np.int32)
    f0 = meta["class_f0_mags"].detach().cpu().numpy()
    f1 = meta["class_f1_mags"].detach().cpu().numpy()
    n0 = meta["class_f0_len"].detach().cpu().numpy()
    n1 = meta["class_f1_len"].detach().cpu().numpy()
    odd = meta["class_odd_leaders"].detach().cpu().numpy()
    leaders = np.zeros((parity.shape[0], 24), dtype=np.int32)
    for k in range(parity.shape[0]):
        if parity[k]:
            vals = np.abs(odd[k])
        else:
            vals = np.concatenate([f0[k, :n0[k]], f1[k, :n1[k]]])
        if vals.shape[0] != 24:
            raise ValueError(f"class {k}: metadata does not describe 24 coordinates")
        leaders[k] = np.sort(vals)[::-1]
    return shell, parity, leaders


# Every metadata tensor the class list is read from (see classes_from_quantize_meta).
_BOOKS = _native.MetadataBooks(("class_parity", "class_shell", "class_f0_mags", "class_f1_mags", "class_f0_len",
                                "class_f1_len", "class_odd_leaders"), classes_from_quantize_meta)


def _book_for(meta: dict, device: torch.device) -> _native.NativeCodebook:
    return _BOOKS.get(meta, device.index)


def quantize_lattice_cuda(x: torch.Tensor, indices: torch.Tensor, best_pair: torch.Tensor, best_score: torch.Tensor,
                          meta: dict, rank_meta: dict, comb: torch.Tensor):
    """Nearest Λ24 codeword index of every 24-D row of ``x`` into ``indices``;
    ``best_pair`` = class_id * n_golay + golay_index, ``best_score`` = fp32 of
    the reference score.  ``rank_meta`` and ``comb`` are accepted for
    signature compatibility; the library derives its rank tables itself."""
    if x.device.type != "cuda":
        raise ValueError("x must be a CUDA tensor")
    if x.dtype != torch.float32:
        raise ValueError("x must be float32")
    if x.dim() != 2 or x.shape[1] != 24 or not x.is_contiguous():
        raise ValueError("x must be a contiguous [N, 24] tensor")
    n = x.shape[0]
    for name, t, dt in (("indices", indices, torch.long), ("best_pair", best_pair, torch.long),
                        ("best_score", best_score, torch.float32)):
        if t.device != x.device or t.dtype != dt or t.numel() != n or not t.is_contiguous():
            raise ValueError(f"{name} must be a contiguous {dt} tensor of {n} elements on {x.device}")
    device = x.device if x.device.index is not None else torch.device("cuda", torch.cuda.current_device())
    book = _book_for(meta, device)
    with torch.cuda.device(device):
        book.quantize(x.data_ptr(), n, indices.data_ptr(), best_pair.data_ptr(), best_score.data_ptr(),
                      torch.cuda.current_stream().cuda_stream)
    return indices, best_pair, best_score
