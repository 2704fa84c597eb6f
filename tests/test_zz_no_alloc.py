"""llvq_gemm_noalloc (static staging array, no device allocation) against
llvq_gemm (stream-ordered staging allocation) on the same inputs.

Both run the same kernels with the same k order per output element (the K
split, when there is one, is decided from the whole matrix, not from the
staging chunk, and two halves added into zero commute), so the outputs are
compared bit for bit.  Two calls in a row with different weights check that
nothing of the first call's staging survives into the second.
The file name sorts last so the suite also runs it after every other test
has used the device.
"""
from __future__ import annotations

import pytest
import torch

pytestmark = pytest.mark.gpu

MAX_BPR = 2730  # LLVQ_GEMM_NOALLOC_MAX_BLOCKS_PER_ROW


def _quantizer():
    from llvq_paper_reproduction_b200 import LeechLatticeVectorQuantizerGpu

    return LeechLatticeVectorQuantizerGpu(max_shell=13, use_cache=False, device="cuda")


def _case(q, m, n, bpr, k, seed):
    g = torch.Generator(device="cuda").manual_seed(seed)
    idx = torch.randint(0, q.total_count, (n, bpr), generator=g, device="cuda")
    a = torch.randn((m, k), generator=g, device="cuda").to(torch.bfloat16)
    scale = (torch.rand(n, generator=g, device="cuda") * 0.04 + 0.005).to(torch.float16)
    return idx, a, scale


def _run(q, fn_name, idx, a, scale):
    m, k = a.shape
    n, bpr = idx.shape
    y = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    err = torch.zeros((1,), dtype=torch.int32, device="cuda")
    stream = torch.cuda.current_stream().cuda_stream
    getattr(q._book(), fn_name)(idx.data_ptr(), n, bpr, scale.data_ptr(), a.data_ptr(), m, k, y.data_ptr(),
                                err.data_ptr(), stream)
    torch.cuda.synchronize()
    assert int(err.item()) == 0
    return y


# (m, n, bpr, k): one with weights wider than the 16 MiB array holds at once
# (K = 14336: 512 rows per chunk, 3 chunks), one with enough output tiles to
# run without the K split, one whose single launch (llvq_gemm) splits the
# tiles of its partial last wave into half-width tiles while the chunked
# launches (no partial wave) do not, and small batches.
CASES = [(300, 1300, 598, 14336), (513, 384, 171, 4096), (1100, 131, 3, 56), (1024, 4736, 8, 192),
         (4096, 1280, 598, 14336), (64, 256, 171, 4096), (1, 700, 40, 960)]


@pytest.mark.parametrize("m,n,bpr,k", CASES)
def test_noalloc_matches_gemm_two_calls(m, n, bpr, k):
    q = _quantizer()
    first = _case(q, m, n, bpr, k, seed=11)
    second = _case(q, m, n, bpr, k, seed=12)
    ref1 = _run(q, "gemm", *first)
    ref2 = _run(q, "gemm", *second)
    out1 = _run(q, "gemm_noalloc", *first)
    out2 = _run(q, "gemm_noalloc", *second)
    assert torch.equal(out1, ref1)
    assert torch.equal(out2, ref2)
    assert not torch.equal(out1, out2)


def test_noalloc_widest_rows_accepted_and_wider_rejected():
    q = _quantizer()
    idx, a, scale = _case(q, 260, 130, MAX_BPR, 24 * MAX_BPR, seed=13)
    assert torch.equal(_run(q, "gemm_noalloc", idx, a, scale), _run(q, "gemm", idx, a, scale))
    wide = torch.zeros((4, MAX_BPR + 1), dtype=torch.long, device="cuda")
    a = torch.zeros((300, 64), dtype=torch.bfloat16, device="cuda")
    with pytest.raises(ValueError, match="2730"):
        _run(q, "gemm_noalloc", wide, a, torch.ones(4, dtype=torch.float16, device="cuda"))


def test_noalloc_empty_call_then_small_batch_wide_rows():
    """An empty call prepares the device (loads the array's module); batches
    of m <= 4 decode in registers, so rows wider than the array's limit are
    accepted there and match llvq_gemm."""
    q = _quantizer()
    idx, a, scale = _case(q, 3, 40, MAX_BPR + 7, 24 * (MAX_BPR + 7), seed=14)
    _run(q, "gemm_noalloc", idx, a[:0], scale)  # m = 0: setup only
    assert torch.equal(_run(q, "gemm_noalloc", idx, a, scale), _run(q, "gemm", idx, a, scale))
