"""GPU dequantizer: integer codewords bit-exact against the oracle's
codeword(); fp32 outputs bit-exact against the reference API's formulas; bf16
with per-row fp16 scales bit-exact against the same product done by torch."""
from __future__ import annotations

import numpy as np
import pytest
import torch

from conftest import golden, oracle_book

pytestmark = pytest.mark.gpu


def api(m: int):
    from llvq_paper_reproduction_b200 import LeechLatticeVectorQuantizerGpu

    return LeechLatticeVectorQuantizerGpu(max_shell=m, use_cache=False, device="cuda")


def random_indices(total: int, n: int, seed: int) -> np.ndarray:
    rng = np.random.default_rng(seed)
    return rng.integers(0, total, size=n, dtype=np.int64)


@pytest.mark.parametrize("m", [2, 4, 13])
def test_lattice_vs_oracle(m):
    q = api(m)
    idx = random_indices(q.total_count, 4000, seed=m)
    idx[:4] = [0, q.total_count - 1, 1103 % q.total_count, 196560 % q.total_count]
    got = q.dequantize_lattice(torch.from_numpy(idx).cuda()).cpu().numpy()
    np.testing.assert_array_equal(got, oracle_book(m).codeword_batch(idx))


def test_reference_codeword_fixtures(reference_tables):
    q = api(13)
    rows = reference_tables["codewords"]
    idx = torch.tensor([r["index"] for r in rows], device="cuda")
    np.testing.assert_array_equal(q.dequantize_lattice(idx).cpu().numpy(), np.array([r["codeword"] for r in rows]))


def test_fp32_kinds_bit_exact():
    from llvq_paper_reproduction_b200 import _native

    q = api(13)
    idx = torch.from_numpy(random_indices(q.total_count, 20000, seed=1)).cuda()
    lat = q.dequantize_lattice(idx)
    # GPU API semantics (_gpu.py:298): python-float scale times an fp32 tensor
    want = (0.35355339059327373 * lat.to(torch.float32))
    got = q.dequantize(idx)
    assert torch.equal(got, want)
    # CPU API semantics: the double product rounded to fp32
    out = torch.empty_like(got)
    q._book().dequantize(idx.data_ptr(), idx.numel(), out.data_ptr(), _native.OUT_F32_DOUBLE, None,
                         torch.cuda.current_stream().cuda_stream)
    want_d = (0.35355339059327373 * lat.cpu().numpy().astype(np.float64)).astype(np.float32)
    np.testing.assert_array_equal(out.cpu().numpy(), want_d)


def test_bf16_rowscale_bit_exact():
    q = api(13)
    rows, blocks = 64, 171
    idx = torch.from_numpy(random_indices(q.total_count, rows * blocks, seed=2).reshape(rows, blocks)).cuda()
    scale = (torch.rand(rows, device="cuda") * 0.05 + 0.001).to(torch.float16)
    got = q.dequantize_bf16(idx, scale)
    ref32 = q.dequantize(idx.reshape(-1)).reshape(rows, blocks * 24) * scale.float()[:, None]
    assert torch.equal(got, ref32.to(torch.bfloat16))


def test_out_of_range_raises():
    q = api(4)
    with pytest.raises(IndexError):
        q.dequantize(torch.tensor([0, q.total_count], device="cuda"))
    with pytest.raises(IndexError):
        q.dequantize_lattice(torch.tensor([-1], device="cuda"))
    assert q.dequantize(torch.empty(0, dtype=torch.long, device="cuda")).shape == (0, 24)


@pytest.mark.parametrize("lo,hi", [(2, 13), (23, 23), (32, 32)])
def test_every_class_vs_oracle(lo, hi):
    """First, last and seeded interior indices of every class, including
    classes with more than four distinct magnitudes and permutation counts
    of 2^32 and more (the single shells 23 and 32), against the oracle."""
    from llvq_paper_reproduction_b200 import LeechLatticeVectorQuantizerGpu
    from oracle.oracle import OracleBook

    q = LeechLatticeVectorQuantizerGpu(max_shell=hi, min_shell=lo, use_cache=False, device="cuda")
    ob = OracleBook(hi, min_shell=lo)
    rng = np.random.default_rng(lo * 100 + hi)
    idx = []
    for k in range(ob.n_classes):
        info = ob.class_info(k)
        start, count = info["start"], info["count"]
        idx += [start, start + count - 1]
        idx += [start + int(rng.integers(count)) for _ in range(4)]
        # the first and last permutation of a random (golay, sign) choice
        perm = info["permutation_count"]
        base = start + int(rng.integers(count // perm)) * perm
        idx += [base, base + perm - 1]
    idx = np.array(idx, dtype=np.int64)
    got = q.dequantize_lattice(torch.from_numpy(idx).cuda()).cpu().numpy()
    np.testing.assert_array_equal(got, ob.codeword_batch(idx))
    assert q.total_count == ob.total_count


def _class_uniform_indices(q, n: int, seed: int) -> np.ndarray:
    """Random valid indices drawn like the dequant benchmark's workload:
    uniform shell, uniform class within the shell, uniform local index."""
    rng = np.random.default_rng(seed)
    shells = sorted(q.classes_by_shell)
    starts = [[q.shell_offsets[s] + o for o in q.class_offsets[s]] for s in shells]
    counts = [[st.count for st in q.local_structures[s]] for s in shells]
    sh = rng.integers(0, len(shells), n)
    out = np.empty(n, dtype=np.int64)
    for i, s in enumerate(shells):
        sel = np.nonzero(sh == i)[0]
        cls = rng.integers(0, len(starts[i]), sel.shape[0])
        st = np.asarray(starts[i], dtype=np.int64)[cls]
        cnt = np.asarray(counts[i], dtype=np.float64)[cls]
        out[sel] = st + np.minimum((rng.random(sel.shape[0]) * cnt).astype(np.int64), cnt.astype(np.int64) - 1)
    return out


def test_llama3_layer_bf16_vs_oracle():
    """One whole Llama-3-8B layer (q, k, v, o, gate, up, down: 9,103,360
    indices, bf16 out, fp16 row scales), int64 and packed indices, bit for
    bit against the oracle's codewords scaled as the kernel defines it:
    bf16(fp32(fp32(1/sqrt 8) * k) * s)."""
    q = api(13)
    shapes = [(4096, 4096), (1024, 4096), (1024, 4096), (4096, 4096), (14336, 4096), (14336, 4096), (4096, 14336)]
    g = torch.Generator().manual_seed(3)
    for j, (rows, cols) in enumerate(shapes):
        bpr = (cols + 23) // 24
        idx = _class_uniform_indices(q, rows * bpr, seed=30 + j)
        scale = (torch.rand(rows, generator=g) * 0.04 + 0.005).to(torch.float16)
        k = torch.from_numpy(oracle_book(13).codeword_batch(idx, threads=0)).view(rows, bpr * 24)
        want = ((k.float() * np.float32(0.35355339059327373)) * scale.float()[:, None]).to(torch.bfloat16)
        it = torch.from_numpy(idx).cuda().view(rows, bpr)
        sc = scale.cuda()
        assert torch.equal(q.dequantize_bf16(it, sc, check=True).cpu(), want)
        assert torch.equal(q.dequantize_bf16(q.pack_indices(it, check=True), sc, check=True).cpu(), want)
