"""Whole-model sharding: host logic on CPU with gloo ranks (plan, per-matrix
checkpoints, resume, gather, a failing rank), and the GPU pipeline pieces
(Hadamard rotation, one quantized matrix)."""
from __future__ import annotations

import os
import socket
from pathlib import Path

import numpy as np
import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from llvq_paper_reproduction_b200.model_quant import (gather_to_rank0, hadamard_block, llama2_7b_matrices,
                                                      plan_shards, run_shard)


def test_plan_balance_and_determinism():
    specs = llama2_7b_matrices()
    assert len(specs) == 224 and sum(s.blocks for s in specs) == 270_286_848
    for world in (1, 2, 4, 8):
        plan = plan_shards(specs, world)
        assert sorted(i for p in plan for i in p) == list(range(224))
        loads = [sum(specs[i].blocks for i in p) for p in plan]
        assert max(loads) - min(loads) <= max(s.blocks for s in specs)
        assert plan == plan_shards(specs, world)


def test_hadamard_block_sizes():
    assert hadamard_block(4096) == 4096 and hadamard_block(11008) == 256 and hadamard_block(14336) == 2048


def fake_quantize(spec):
    """Deterministic CPU stand-in for the GPU quantizer (host-logic tests)."""
    g = torch.Generator().manual_seed(spec.ordinal)
    return {"indices": torch.randint(0, 1 << 40, (spec.out_features, spec.blocks_per_row), generator=g),
            "row_scale": torch.rand(spec.out_features, generator=g).to(torch.float16)}


def _free_port() -> int:
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_host_pack_roundtrip():
    from llvq_paper_reproduction_b200.model_quant import pack_le_bytes, unpack_le_bytes

    idx = torch.tensor([0, 1, (1 << 40) - 1, 123456789012], dtype=torch.int64)
    pk = pack_le_bytes(idx, 5)
    assert pk.shape == (4, 5) and pk.dtype == torch.uint8
    assert torch.equal(unpack_le_bytes(pk, 5), idx)


def _worker(rank, world, port, out_dir, fail_rank, result_path):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    from datetime import timedelta

    dist.init_process_group("gloo", rank=rank, world_size=world, timeout=timedelta(seconds=20))
    specs = llama2_7b_matrices(layers=2, scale_down=64)
    if rank == fail_rank:
        raise RuntimeError("injected failure on this rank")
    local = run_shard(specs, rank, world, Path(out_dir), fake_quantize)
    res = gather_to_rank0(specs, local, rank, world, "cpu", index_bytes=5)  # fake indices < 2^40
    if rank == 0:
        torch.save(res, result_path)
    dist.destroy_process_group()


def _spawn(world, tmp_path, fail_rank=-1):
    port = _free_port()
    ctx = mp.get_context("spawn")
    procs = [ctx.Process(target=_worker, args=(r, world, port, str(tmp_path / "ckpt"), fail_rank,
                                                str(tmp_path / "result.pt"))) for r in range(world)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(60)
    codes = []
    for p in procs:
        if p.is_alive():
            p.kill()
            p.join()
        codes.append(p.exitcode)
    return codes


def test_gloo_two_ranks_gather_and_resume(tmp_path):
    codes = _spawn(2, tmp_path)
    assert codes == [0, 0]
    res = torch.load(tmp_path / "result.pt")
    specs = llama2_7b_matrices(layers=2, scale_down=64)
    assert set(res) == {s.key for s in specs}
    for s in specs:
        want = fake_quantize(s)
        assert torch.equal(res[s.key][0], want["indices"])
        assert torch.equal(res[s.key][1], want["row_scale"])
    # resume: every checkpoint exists; corrupt one, it is recomputed, the rest are loaded
    ck = tmp_path / "ckpt"
    assert len(list(ck.glob("*.pt"))) == len(specs)
    (ck / f"{specs[3].key}.pt").write_bytes(b"broken")
    (tmp_path / "result.pt").unlink()
    assert _spawn(2, tmp_path) == [0, 0]
    res2 = torch.load(tmp_path / "result.pt")
    assert all(torch.equal(res2[k][0], res[k][0]) for k in res)


def test_stale_checkpoints_are_quantized_again(tmp_path):
    """A checkpoint from another configuration (other fingerprint, other
    shape) is not reused; a matching one is."""
    specs = llama2_7b_matrices(layers=1, scale_down=64)
    calls = []

    def q(spec):
        calls.append(spec.key)
        return fake_quantize(spec)

    run_shard(specs, 0, 1, tmp_path, q, fingerprint={"rate": 2.0, "seed": 2})
    assert len(calls) == len(specs)
    run_shard(specs, 0, 1, tmp_path, q, fingerprint={"rate": 2.0, "seed": 2})
    assert len(calls) == len(specs)  # all resumed
    run_shard(specs, 0, 1, tmp_path, q, fingerprint={"rate": 2.5, "seed": 2})
    assert len(calls) == 2 * len(specs)  # other rate: every matrix again
    wider = llama2_7b_matrices(layers=1, scale_down=32)  # same keys, more rows
    run_shard(wider, 0, 1, tmp_path, q, fingerprint={"rate": 2.5, "seed": 2})
    assert len(calls) == 3 * len(specs)
    assert not list(tmp_path.glob("*.tmp*"))


def test_gloo_failing_rank_is_reported(tmp_path):
    codes = _spawn(2, tmp_path, fail_rank=1)
    assert codes[1] != 0  # the failing rank exits with an error
    assert codes[0] != 0  # its peer's collective times out instead of hanging


@pytest.mark.gpu
def test_gpu_hadamard_matches_dense_reference():
    from llvq_paper_reproduction_b200.model_quant import hadamard_signs, rotate

    for cols in (4096, 11008, 256):
        block = hadamard_block(cols)
        w = torch.randn((8, cols), device="cuda").to(torch.float16)
        signs = hadamard_signs(cols, 11, "cuda")
        out = rotate(w, signs, block)
        h = torch.tensor([[1.0]], dtype=torch.float64)
        while h.shape[0] < block:
            h = torch.cat([torch.cat([h, h], 1), torch.cat([h, -h], 1)], 0)
        x = (w.double() * signs.double()).view(8, cols // block, block)
        ref = (x @ h.cuda().T / np.sqrt(block)).view(8, cols)
        assert torch.allclose(out.double(), ref, atol=1e-4, rtol=1e-5)
        back = rotate(out, signs, block, inverse=True)
        assert torch.allclose(back, w.float(), atol=1e-5)


@pytest.mark.gpu
def test_gpu_matrix_quantization():
    from llvq_paper_reproduction_b200.model_quant import MatrixQuantizer

    mq = MatrixQuantizer(rate=2.0, device="cuda")
    for spec in llama2_7b_matrices(layers=1, scale_down=32)[3:6]:
        r = mq.quantize(spec, with_error=True)
        assert r["indices"].shape == (spec.out_features, spec.blocks_per_row)
        assert int(r["indices"].min()) >= 0 and int(r["indices"].max()) < (1 << mq.sg.bits)
        assert r["rel_mse"] < 0.15  # ~2 bits/dim on a Gaussian source


@pytest.mark.gpu
def test_gpu_rotate_scale_matches_separate_passes():
    """The fused rotation + RMS scale + pad kernel against the rotation kernel
    followed by the same steps in torch: the rotated rows are identical; the
    fp16 scale may differ by one fp16 step (the RMS reduction order differs)."""
    from llvq_paper_reproduction_b200 import _native
    from llvq_paper_reproduction_b200.model_quant import hadamard_signs, rotate

    for rows, cols in ((64, 4096), (33, 11008)):
        block = hadamard_block(cols)
        ld = (cols + 23) // 24 * 24
        w = (torch.randn((rows, cols), device="cuda") * 0.02).to(torch.float16)
        signs = hadamard_signs(cols, 5, "cuda")
        xp = torch.full((rows, ld), float("nan"), device="cuda")
        sc = torch.empty(rows, dtype=torch.float16, device="cuda")
        _native.rotate_scale(w.data_ptr(), rows, cols, ld, block, signs.data_ptr(), xp.data_ptr(), sc.data_ptr(),
                             torch.cuda.current_stream().cuda_stream)
        wr = rotate(w, signs, block)
        want_sc = wr.pow(2).mean(1).sqrt().clamp_min(1e-8).to(torch.float16)
        assert (sc.float() - want_sc.float()).abs().max() <= want_sc.float().max() * 2 ** -10
        assert torch.equal(xp[:, :cols], wr / sc.float()[:, None])
        assert not xp[:, cols:].any()
