"""Dequant-GEMM (decode to bf16 staging, tcgen05 GEMM) against dequantize-
then-matmul in fp32 (relative Frobenius error <= 1e-3; the path only rounds
the bf16 activations, so the observed error is far smaller)."""
from __future__ import annotations

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu
TOL = 1e-3

_Q = {}


def api(m: int = 13):
    from llvq_paper_reproduction_b200 import LeechLatticeVectorQuantizerGpu

    if m not in _Q:
        _Q[m] = LeechLatticeVectorQuantizerGpu(max_shell=m, use_cache=False, device="cuda")
    return _Q[m]


def reference(q, a, idx, scale, k):
    w = q.dequantize(idx.reshape(-1)).reshape(idx.shape[0], -1)[:, :k]
    if scale is not None:
        w = w * scale.float()[:, None]
    return a.float() @ w.T


def rel_err(y, ref):
    return float(torch.linalg.norm(y - ref) / torch.linalg.norm(ref))


# the K range is split in two while the output has fewer 128 x 256 tiles
# than SMs; (1024, 4736, 8, 192) has 148 tiles (no split); (1100, 4736, 8,
# 192) has 185 (148 + 37: the last wave's tiles are split into half-width
# tiles, some of them wholly beyond the 1100 activation rows); (300, 2500,
# 598, 14336) is one staging chunk here and three in the no-allocation variant
@pytest.mark.parametrize("m_act,n,bpr,k", [(1, 128, 8, 192), (8, 300, 20, 472), (64, 256, 171, 4096),
                                           (200, 130, 25, 600), (256, 200, 12, 288), (300, 257, 9, 216),
                                           (16, 1024, 598, 14336), (513, 384, 171, 4096), (300, 2500, 598, 14336),
                                           (1100, 131, 3, 56), (1024, 4736, 8, 192), (1100, 4736, 8, 192)])
def test_gemm_matches_dequantize_matmul(m_act, n, bpr, k):
    q = api()
    g = torch.Generator(device="cuda").manual_seed(4)
    idx = torch.randint(0, q.total_count, (n, bpr), generator=g, device="cuda")
    a = torch.randn((m_act, k), generator=g, device="cuda").to(torch.bfloat16)
    scale = (torch.rand(n, generator=g, device="cuda") * 0.04 + 0.005).to(torch.float16)
    y = q.gemm(a, idx, scale)
    ref = reference(q, a, idx, scale, k)
    assert y.shape == (m_act, n)
    assert rel_err(y, ref) <= TOL
    y2 = q.gemm(a, idx)  # no row scales
    assert rel_err(y2, reference(q, a, idx, None, k)) <= TOL


# m <= 4 takes the fused decode-in-registers kernel (no staging): partial
# last blocks (k not a multiple of 24), each batch-size template, wide rows,
# and the first staged size (5)
@pytest.mark.parametrize("m_act,n,bpr,k", [(1, 77, 33, 784), (2, 40, 3, 64), (3, 129, 20, 472), (4, 64, 171, 4104),
                                           (1, 1000, 598, 14336), (4, 9, 171, 4096), (5, 300, 20, 472)])
def test_small_batch_gemm(m_act, n, bpr, k):
    q = api()
    g = torch.Generator(device="cuda").manual_seed(6)
    idx = torch.randint(0, q.total_count, (n, bpr), generator=g, device="cuda")
    a = torch.randn((m_act, k), generator=g, device="cuda").to(torch.bfloat16)
    scale = (torch.rand(n, generator=g, device="cuda") * 0.04 + 0.005).to(torch.float16)
    y = q.gemm(a, idx, scale)
    assert y.shape == (m_act, n)
    assert rel_err(y, reference(q, a, idx, scale, k)) <= TOL
    assert torch.equal(y, q.gemm(a, idx, scale))  # one summation order: the same result every call
    packed = q.pack_indices(idx)
    assert torch.equal(y, q.gemm(a, packed, scale))


def test_gemm_argument_checks():
    q = api(4)
    idx = torch.zeros((4, 2), dtype=torch.long, device="cuda")
    with pytest.raises(ValueError):
        q.gemm(torch.zeros((2, 60), device="cuda"), idx)  # k > 24 * blocks
    with pytest.raises(ValueError):
        q.gemm(torch.zeros((2, 20), device="cuda"), idx)  # k % 8 != 0
    assert q.gemm(torch.zeros((0, 48), device="cuda"), idx).shape == (0, 4)


def test_bf16_hadamard_matches_fp32_rotation():
    from llvq_paper_reproduction_b200 import _native
    from llvq_paper_reproduction_b200.model_quant import hadamard_signs, rotate

    a = torch.randn((37, 1024), generator=torch.Generator(device="cuda").manual_seed(8), device="cuda")
    a16 = a.to(torch.bfloat16)
    signs = hadamard_signs(1024, 5, "cuda")
    out = torch.empty_like(a16)
    _native.hadamard_ex(a16.data_ptr(), _native.DT_BF16, out.data_ptr(), _native.DT_BF16, 37, 1024, 256,
                        signs.data_ptr(), False, torch.cuda.current_stream().cuda_stream)
    # same fp32 butterflies as the fp32 kernel on the widened input, one bf16 rounding
    assert torch.equal(out, rotate(a16.float(), signs, 256).to(torch.bfloat16))


def test_gemm_with_activation_rotation():
    """A weight quantized after a Hadamard rotation, multiplied with the
    rotation applied to the activations, approximates x W^T up to the
    quantization error; without the rotation the result is unrelated."""
    from llvq_paper_reproduction_b200.model_quant import hadamard_signs, rotate

    q = api()
    g = torch.Generator(device="cuda").manual_seed(9)
    n, k, block = 192, 1536, 512
    w = torch.randn((n, k), generator=g, device="cuda") * 0.02
    signs = hadamard_signs(k, 3, "cuda")
    wr = rotate(w, signs, block)
    scale = wr.pow(2).mean(1).sqrt().to(torch.float16)
    idx = q.quantize((wr / scale.float()[:, None]).reshape(-1, 24)).reshape(n, k // 24)
    x = torch.randn((64, k), generator=g, device="cuda").to(torch.bfloat16)
    want = x.float() @ w.T
    y = q.gemm(x, idx, scale, rotation=(block, signs))
    assert rel_err(y, want) < 0.4
    assert rel_err(q.gemm(x, idx, scale), want) > 0.9
    # the rotation is exactly a bf16 Hadamard of the activations, then the plain GEMM
    xr = rotate(x.float(), signs, block).to(torch.bfloat16)
    assert torch.equal(y, q.gemm(xr, idx, scale))


@pytest.mark.parametrize("m_act", [1, 64])
def test_gemm_does_not_synchronise_the_host(m_act):
    """The dequant-GEMM returns while the GPU is still busy: behind a long
    device-side sleep on the same stream the call comes back before the
    stream drains; errors wait in the pending flags."""
    q = api()
    g = torch.Generator(device="cuda").manual_seed(5)
    idx = torch.randint(0, q.total_count, (512, 171), generator=g, device="cuda")
    a = torch.randn((m_act, 4096), generator=g, device="cuda").to(torch.bfloat16)
    want = q.gemm(a, idx, check=True)
    torch.cuda.synchronize()
    stream = torch.cuda.current_stream()
    torch.cuda._sleep(2_000_000_000)  # about a second of device time
    y = q.gemm(a, idx)
    assert not stream.query()
    torch.cuda.synchronize()
    assert torch.equal(y, want)
    q.raise_pending_errors()



@pytest.fixture(scope="module")
def llama3_mlp():
    """The Llama-3-8B MLP weights at their real shapes, random valid indices
    (seed 4), fp16 row scales, and each W decoded by the oracle (the
    reference's codeword() restated) in fp32: W = fp32(1/sqrt 8) * k * s."""
    from conftest import oracle_book

    q = api()
    g = torch.Generator(device="cuda").manual_seed(4)
    mats = []
    for n_out, k in ((14336, 4096), (4096, 14336)):
        bpr = (k + 23) // 24
        idx = torch.randint(0, q.total_count, (n_out, bpr), generator=g, device="cuda")
        scale = (torch.rand(n_out, generator=g, device="cuda") * 0.04 + 0.005).to(torch.float16)
        cw = oracle_book(13).codeword_batch(idx.cpu().numpy().reshape(-1), threads=0)
        w = torch.from_numpy(cw).cuda().view(n_out, bpr * 24)[:, :k].float() * np.float32(1 / np.sqrt(8.0))
        mats.append((idx, scale, w * scale.float()[:, None], k))
    return mats


@pytest.mark.parametrize("m_act", [1, 8, 64, 512, 4096])
def test_gemm_llama3_mlp_shapes(llama3_mlp, m_act):
    """W 14336 x 4096 and 4096 x 14336 at every batch size of the benchmark
    against an fp32 matmul with the oracle's decoded weights (relative
    Frobenius error <= 1e-3)."""
    q = api()
    g = torch.Generator(device="cuda").manual_seed(100 + m_act)
    for idx, scale, w, k in llama3_mlp:
        a = torch.randn((m_act, k), generator=g, device="cuda").to(torch.bfloat16)
        y = q.gemm(a, idx, scale, check=True)
        ref = a.float() @ w.T
        assert rel_err(y, ref) <= TOL
