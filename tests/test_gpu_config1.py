"""The 65,536-block Gaussian workload at full size: every index against the
oracle's fixture (the reference CPU quantizer restated and run over all
blocks by tests/golden/make_config1.py), plus SQNR.

Workload: 65,536 x 24 i.i.d. N(0, 1) fp32 values from torch's CPU generator
with seed 0.  Two codes: the reference's own quantize over shells 2..13 (the
48-bit codebook) and the shape-gain code at 2 bits/dim (shell-11 shape, 45
bits, + 3-bit chi(24) gain code)."""
from __future__ import annotations

import hashlib
import math

import numpy as np
import pytest
import torch

from conftest import GOLDEN, oracle_book

pytestmark = pytest.mark.gpu
N = 65536


def _unpack6(b: np.ndarray) -> np.ndarray:
    out = np.zeros((b.shape[0], 8), dtype=np.uint8)
    out[:, :6] = b
    return out.view("<u8").reshape(-1).astype(np.int64)


@pytest.fixture(scope="module")
def workload():
    x = torch.randn((N, 24), generator=torch.Generator().manual_seed(0), dtype=torch.float32)
    fx = np.load(GOLDEN / "config1_indices.npz")
    assert hashlib.sha256(x.numpy().tobytes()).hexdigest() == str(fx["sha256"]), "torch generator output changed"
    return x, _unpack6(fx["ball"]), _unpack6(fx["shape"])


def _sqnr_db(x: torch.Tensor, rec: torch.Tensor) -> float:
    xd = x.double()
    return 10.0 * math.log10(xd.pow(2).sum().item() / (xd - rec.double().cpu()).pow(2).sum().item())


def test_every_index_shells_2_13(workload):
    from llvq_paper_reproduction_b200 import LeechLatticeVectorQuantizerGpu

    x, ball, _ = workload
    q = LeechLatticeVectorQuantizerGpu(max_shell=13, use_cache=False, device="cuda")
    idx = q.quantize(x.cuda()).cpu().numpy()
    assert int((idx != ball).sum()) == 0
    lat = q.dequantize_lattice(torch.from_numpy(ball).cuda()).cpu().numpy()
    np.testing.assert_array_equal(lat, oracle_book(13).codeword_batch(ball, threads=0))
    # the ball at unit scale clips the Gaussian tails: a sanity bound only
    assert _sqnr_db(x, q.dequantize(torch.from_numpy(ball).cuda())) > 5.0


def test_every_shape_index_and_gain_code_2_bits(workload):
    from llvq_paper_reproduction_b200.shaping import ShapeGainQuantizer

    x, _, shape = workload
    sg = ShapeGainQuantizer.for_rate(2.0, device="cuda")
    assert (sg.shell, sg.bits) == (11, 48)
    sidx, gidx = sg.quantize_parts(x.cuda())
    assert int((sidx.cpu().numpy() != shape).sum()) == 0
    # gain code: the reference's compensated fp64 projection <x, y> over
    # |y| = sqrt(16 * 11), against the fp64 thresholds: exactly the kernel's
    from oracle.oracle import ref_projection

    y = oracle_book(11, 11).codeword_batch(shape, threads=0)
    xd = x.numpy().astype(np.float64)
    g = np.array([ref_projection(xd[i], y[i]) for i in range(N)]) / np.sqrt(16.0 * 11)
    want = np.searchsorted(sg.thresholds.cpu().numpy(), g, side="left")
    np.testing.assert_array_equal(gidx.cpu().numpy(), want)
    sqnr = _sqnr_db(x, sg.dequantize_parts(sidx, gidx))
    assert 10.5 < sqnr < 11.5  # measured 10.9 dB at this rate
