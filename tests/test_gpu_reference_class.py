"""The reference's own API class driven through this library's launchers.

LeechLatticeVectorQuantizerGpu of the reference imports its two NVRTC
launchers optionally (impl/leech_lattice_vector_quantizer_gpu.py:19-27).
Seeding sys.modules with this library's shims under those module names makes
the unmodified reference class run on the sm_100a kernels; its quantize and
dequantize must then equal the oracle.

Needs a GPU and the reference: its copy installed in baseline/_ref (pip
install --target of a checkout copy whose pyproject.toml declares packages =
["impl"]), or a checkout whose root directory is given in the environment
variable LLVQ_REFERENCE_ROOT (skipped when neither exists)."""
from __future__ import annotations

import os
import sys

import numpy as np
import pytest
import torch

from conftest import oracle_book

pytestmark = pytest.mark.gpu
_INSTALLED = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "baseline", "_ref")
ROOT = os.environ.get("LLVQ_REFERENCE_ROOT") or (_INSTALLED if os.path.isdir(_INSTALLED) else "")


@pytest.fixture(scope="module")
def reference_gpu_module():
    if not ROOT or not os.path.isdir(os.path.join(ROOT, "impl")):
        pytest.skip("no reference: neither baseline/_ref nor LLVQ_REFERENCE_ROOT")
    from llvq_paper_reproduction_b200 import llvq_cuda_dequantize, llvq_cuda_quantize

    sys.modules["impl.llvq_cuda_quantize"] = llvq_cuda_quantize
    sys.modules["impl.llvq_cuda_dequantize"] = llvq_cuda_dequantize
    sys.path.insert(0, ROOT)
    try:
        from impl import leech_lattice_vector_quantizer_gpu as ref
    finally:
        sys.path.remove(ROOT)
    assert ref.quantize_lattice_cuda is llvq_cuda_quantize.quantize_lattice_cuda
    assert ref.dequantize_lattice_cuda is llvq_cuda_dequantize.dequantize_lattice_cuda
    return ref


@pytest.mark.parametrize("m", [4, 13])
def test_reference_class_on_the_shims(reference_gpu_module, m, tmp_path):
    q = reference_gpu_module.LeechLatticeVectorQuantizerGpu(max_shell=m, use_cache=False, device="cuda")
    x = torch.randn((512, 24), generator=torch.Generator().manual_seed(m), dtype=torch.float32)
    idx = q.quantize(x.cuda())
    want = oracle_book(m).quantize_batch(x.numpy())[0]
    np.testing.assert_array_equal(idx.cpu().numpy(), want)
    lat = q.dequantize_lattice(idx)
    np.testing.assert_array_equal(lat.cpu().numpy(), oracle_book(m).codeword_batch(want))
