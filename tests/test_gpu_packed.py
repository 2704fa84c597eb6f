"""Packed index storage: int64 <-> index_bytes little-endian bytes (6 for
shells 2..13), and the dequantizer / dequant-GEMM reading packed indices,
bit-exact against the same calls on int64 indices."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu

_Q = {}


def api(m: int = 13):
    from llvq_paper_reproduction_b200 import LeechLatticeVectorQuantizerGpu

    if m not in _Q:
        _Q[m] = LeechLatticeVectorQuantizerGpu(max_shell=m, use_cache=False, device="cuda")
    return _Q[m]


def random_indices(q, shape, seed):
    return torch.from_numpy(np.random.default_rng(seed).integers(0, q.total_count, shape)).cuda()


@pytest.mark.parametrize("m,bytes_", [(13, 6), (4, 4), (2, 3)])
def test_pack_roundtrip(m, bytes_):
    q = api(m)
    assert q.index_bytes == bytes_
    idx = random_indices(q, (1000,), m)
    idx[:3] = torch.tensor([0, q.total_count - 1, -1])
    pk = q.pack_indices(idx)
    assert pk.shape == (1000, bytes_) and pk.dtype == torch.uint8
    # little-endian bytes of the value; -1 is all-ones
    want = idx.cpu().numpy().astype("<i8").view(np.uint8).reshape(-1, 8)[:, :bytes_]
    np.testing.assert_array_equal(pk.cpu().numpy(), want)
    assert torch.equal(q.unpack_indices(pk), idx)


def test_pack_rejects_what_does_not_fit():
    q = api(2)
    with pytest.raises(IndexError):
        q.pack_indices(torch.tensor([0, 1 << 24], device="cuda"), check=True)
    with pytest.raises(IndexError):
        q.pack_indices(torch.tensor([-2], device="cuda"), check=True)
    # without check the call stays asynchronous; the count waits in the flags
    q.pack_indices(torch.tensor([-2], device="cuda"))
    assert q.pending_errors()["index_range"] == 1
    with pytest.raises(IndexError):
        q.raise_pending_errors()
    assert q.pending_errors() == {"index_range": 0, "gemm_timeout": 0}


def test_dequantize_packed_every_kind():
    from llvq_paper_reproduction_b200 import _native

    q = api()
    idx = random_indices(q, (5000,), 1)
    pk = q.pack_indices(idx)
    stream = torch.cuda.current_stream().cuda_stream
    for kind, dtype in ((_native.OUT_INT64, torch.long), (_native.OUT_F32, torch.float32),
                        (_native.OUT_F32_DOUBLE, torch.float32)):
        got = torch.empty((5000, 24), dtype=dtype, device="cuda")
        q._book().dequantize_packed(pk.data_ptr(), q.index_bytes, 5000, got.data_ptr(), kind, None, 1, None, stream)
        want = torch.empty_like(got)
        if kind == _native.OUT_INT64:
            q._book().dequantize_lattice(idx.data_ptr(), 5000, want.data_ptr(), None, stream)
        else:
            q._book().dequantize(idx.data_ptr(), 5000, want.data_ptr(), kind, None, stream)
        assert torch.equal(got, want)


def test_dequantize_bf16_packed_matches_int64():
    q = api()
    idx = random_indices(q, (96, 171), 2)
    scale = (torch.rand(96, device="cuda") * 0.05 + 0.001).to(torch.float16)
    assert torch.equal(q.dequantize_bf16(q.pack_indices(idx), scale), q.dequantize_bf16(idx, scale))


def test_packed_invalid_index_raises():
    q = api()
    pk = q.pack_indices(torch.tensor([[5, -1]], device="cuda"))
    with pytest.raises(IndexError):
        q.dequantize_bf16(pk, torch.ones(1, dtype=torch.float16, device="cuda"), check=True)


@pytest.mark.parametrize("m_act,n,bpr,k", [(8, 300, 20, 472), (513, 384, 171, 4096)])
def test_gemm_packed_matches_int64(m_act, n, bpr, k):
    q = api()
    g = torch.Generator(device="cuda").manual_seed(5)
    idx = random_indices(q, (n, bpr), 3)
    a = torch.randn((m_act, k), generator=g, device="cuda").to(torch.bfloat16)
    scale = (torch.rand(n, generator=g, device="cuda") * 0.04 + 0.005).to(torch.float16)
    assert torch.equal(q.gemm(a, q.pack_indices(idx), scale), q.gemm(a, idx, scale))
