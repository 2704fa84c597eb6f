"""Whole-model weight quantization, sharded by matrix across GPUs.

Workload (no reference implementation: the reference's LLM pipeline is a
README stub): every linear of a Llama-2-7B-shaped model -- 32 layers of
q/k/v/o 4096x4096, gate/up 11008x4096, down 4096x11008 -- with fp16 entries
N(0, sigma_row^2), sigma_row ~ LogNormal(log 0.02, 0.5) per row (seeded).
Per matrix:
  1. seeded random Hadamard rotation along the input dimension (+-1 signs
     times the normalised Walsh-Hadamard transform, in segments of the
     largest power of two dividing the row length: 4096 for 4096, 256 for
     11008);
  2. per-row scale = RMS of the rotated row, stored as fp16;
  3. rows divided by their scale, padded with zeros to a multiple of 24
     (4104, 11016) and split into 24-D blocks -- steps 1-3 are one library
     kernel (llvq_rotate_scale);
  4. shape-gain quantization of every block (shaping.ShapeGainQuantizer,
     2 bits/dim by default: index = shape * 2^b + gain).
Sharding: matrices are independent, so ranks own whole matrices (greedy
balance of block counts), quantize them with no inter-GPU traffic,
checkpoint each finished matrix (atomic write; a restart skips finished
ones), and finally gather every index tensor (packed to 6 bytes per block)
and row scale to rank 0 over the process group (NCCL on GPUs, gloo in CPU
tests).
"""
from __future__ import annotations

import argparse
import math
import os
import time
from dataclasses import dataclass
from pathlib import Path
from typing import Callable, Sequence

import torch

DIM = 24
LLAMA2_7B_LINEARS = (("q_proj", 4096, 4096), ("k_proj", 4096, 4096), ("v_proj", 4096, 4096),
                     ("o_proj", 4096, 4096), ("gate_proj", 11008, 4096), ("up_proj", 11008, 4096),
                     ("down_proj", 4096, 11008))


@dataclass(frozen=True)
class MatrixSpec:
    layer: int
    name: str
    out_features: int
    in_features: int

    @property
    def key(self) -> str:
        return f"layer{self.layer:02d}.{self.name}"

    @property
    def blocks_per_row(self) -> int:
        return (self.in_features + DIM - 1) // DIM

    @property
    def blocks(self) -> int:
        return self.out_features * self.blocks_per_row

    @property
    def ordinal(self) -> int:
        return self.layer * len(LLAMA2_7B_LINEARS) + [n for n, _, _ in LLAMA2_7B_LINEARS].index(self.name)


def llama2_7b_matrices(layers: int = 32, scale_down: int = 1) -> list[MatrixSpec]:
    """The model's linears; scale_down > 1 divides the output features (for
    small test runs) while keeping the input dimensions."""
    return [MatrixSpec(l, n, max(1, o // scale_down), i) for l in range(layers) for n, o, i in LLAMA2_7B_LINEARS]


def plan_shards(specs: Sequence[MatrixSpec], world: int) -> list[list[int]]:
    """Greedy balance: largest matrices first, each to the least-loaded rank
    (ties to the lowest rank).  Deterministic for a given list."""
    order = sorted(range(len(specs)), key=lambda i: (-specs[i].blocks, i))
    load = [0] * world
    out: list[list[int]] = [[] for _ in range(world)]
    for i in order:
        r = min(range(world), key=lambda k: (load[k], k))
        out[r].append(i)
        load[r] += specs[i].blocks
    return [sorted(v) for v in out]


def hadamard_block(cols: int) -> int:
    b = 1
    while cols % (b * 2) == 0 and b * 2 <= 4096:
        b *= 2
    return b


def hadamard_signs(cols: int, seed: int, device) -> torch.Tensor:
    g = torch.Generator(device="cpu").manual_seed(seed)
    return (torch.randint(0, 2, (cols,), generator=g, dtype=torch.int8) * 2 - 1).to(device)


def rotate(w: torch.Tensor, signs: torch.Tensor, block: int, inverse: bool = False) -> torch.Tensor:
    """Seeded Hadamard rotation of each row (fp16/fp32 in, fp32 out) on the GPU."""
    from . import _native

    if w.dtype not in (torch.float16, torch.float32):
        raise ValueError("rotate expects fp16 or fp32")
    w = w.contiguous()
    out = torch.empty(w.shape, dtype=torch.float32, device=w.device)
    with torch.cuda.device(w.device):
        _native.hadamard(w.data_ptr(), w.dtype == torch.float16, out.data_ptr(), w.shape[0], w.shape[1], block,
                         signs.data_ptr(), inverse, torch.cuda.current_stream().cuda_stream)
    return out


def synth_weight(spec: MatrixSpec, seed: int, device) -> torch.Tensor:
    """fp16 [out, in]: N(0, sigma_row^2) with sigma_row ~ LogNormal(log 0.02, 0.5)."""
    g = torch.Generator(device=device).manual_seed(seed * 1_000_003 + spec.ordinal)
    sigma = torch.exp(math.log(0.02) + 0.5 * torch.randn(spec.out_features, generator=g, device=device))
    w = torch.randn((spec.out_features, spec.in_features), generator=g, device=device) * sigma[:, None]
    return w.to(torch.float16)


class MatrixQuantizer:
    """Rotation + row scaling + shape-gain quantization of one matrix."""

    def __init__(self, rate: float = 2.0, seed: int = 2, device="cuda"):
        from .shaping import ShapeGainQuantizer

        self.sg = ShapeGainQuantizer.for_rate(rate, device=device)
        self.seed = seed
        self.device = torch.device(device)

    def quantize(self, spec: MatrixSpec, with_error: bool = False) -> dict:
        from . import _native

        w = synth_weight(spec, self.seed, self.device)
        block = hadamard_block(spec.in_features)
        signs = hadamard_signs(spec.in_features, self.seed * 7919 + spec.in_features, self.device)
        bpr = spec.blocks_per_row
        # rotation, fp16 RMS row scale, division and zero padding in one kernel
        xp = torch.empty((spec.out_features, bpr * DIM), dtype=torch.float32, device=self.device)
        scale = torch.empty(spec.out_features, dtype=torch.float16, device=self.device)
        with torch.cuda.device(self.device):
            _native.rotate_scale(w.data_ptr(), spec.out_features, spec.in_features, bpr * DIM, block,
                                 signs.data_ptr(), xp.data_ptr(), scale.data_ptr(),
                                 torch.cuda.current_stream().cuda_stream)
        idx = self.sg.quantize(xp.view(-1, DIM)).view(spec.out_features, bpr)
        out = {"indices": idx, "row_scale": scale}
        if with_error:
            recon = self.sg.dequantize(idx.view(-1)).view(spec.out_features, -1)[:, : spec.in_features]
            wq = rotate(recon * scale.float()[:, None], signs, block, inverse=True)
            ref = w.float()
            out["rel_mse"] = float((wq - ref).pow(2).sum() / ref.pow(2).sum())
        return out


def _save_atomic(path: Path, obj) -> None:
    """Write to a temporary file, flush it to disk, then rename over `path`,
    so a crash leaves either the old file or the complete new one."""
    tmp = path.with_suffix(path.suffix + f".tmp{os.getpid()}")
    with open(tmp, "wb") as fh:
        torch.save(obj, fh)
        fh.flush()
        os.fsync(fh.fileno())
    tmp.replace(path)


def _checkpoint_meta(spec: MatrixSpec, fingerprint: dict | None) -> dict:
    return {"key": spec.key, "out_features": spec.out_features, "in_features": spec.in_features,
            "blocks_per_row": spec.blocks_per_row, **(fingerprint or {})}


def run_shard(specs: Sequence[MatrixSpec], rank: int, world: int, out_dir: Path,
              quantize_fn: Callable[[MatrixSpec], dict], log: Callable[[str], None] = lambda s: None,
              fingerprint: dict | None = None) -> dict:
    """Quantize this rank's matrices (skipping finished checkpoints) and
    return {key: (indices, row_scale)} on CPU.  A checkpoint is reused only
    when it loads, carries the same matrix shape and the same `fingerprint`
    (the settings that determine its contents, e.g. rate and seed), and holds
    tensors of the expected shapes; anything else is quantized again."""
    out_dir.mkdir(parents=True, exist_ok=True)
    mine = plan_shards(specs, world)[rank]
    done = {}
    for i in mine:
        spec = specs[i]
        path = out_dir / f"{spec.key}.pt"
        meta = _checkpoint_meta(spec, fingerprint)
        res = None
        if path.exists():
            try:
                res = torch.load(path, map_location="cpu")
                ok = (res.get("meta") == meta
                      and tuple(res["indices"].shape) == (spec.out_features, spec.blocks_per_row)
                      and tuple(res["row_scale"].shape) == (spec.out_features,))
                if ok:
                    log(f"rank {rank}: resumed {spec.key}")
                else:
                    log(f"rank {rank}: stale checkpoint {spec.key}, quantizing again")
                    res = None
            except Exception:
                res = None
        if res is None:
            r = quantize_fn(spec)
            res = {"indices": r["indices"].cpu(), "row_scale": r["row_scale"].cpu(), "meta": meta}
            _save_atomic(path, res)
        done[spec.key] = (res["indices"], res["row_scale"])
    return done


def pack_le_bytes(indices: torch.Tensor, index_bytes: int) -> torch.Tensor:
    """Non-negative int64 indices (any device) -> uint8 [n, index_bytes],
    little-endian (the low bytes of each index)."""
    flat = indices.reshape(-1).contiguous()
    return flat.view(torch.uint8).view(-1, 8)[:, :index_bytes].contiguous()


def unpack_le_bytes(packed: torch.Tensor, index_bytes: int) -> torch.Tensor:
    """uint8 [n, index_bytes] -> int64 [n] on the same device."""
    out = torch.zeros((packed.shape[0], 8), dtype=torch.uint8, device=packed.device)
    out[:, :index_bytes] = packed
    return out.view(torch.int64).reshape(-1)


def gather_to_rank0(specs: Sequence[MatrixSpec], local: dict, rank: int, world: int, device,
                    index_bytes: int = 8) -> dict | None:
    """Gather every rank's indices (as index_bytes little-endian bytes each:
    6 for the 48-bit shape-gain index, a quarter less than int64) and row
    scales to rank 0, flattened and padded to the largest shard, entirely on
    `device` (indices that are already there never visit the host).  Two
    gathers to rank 0 (not all-gathers: only rank 0 keeps the result, so each
    other rank sends its shard once and receives nothing); rank 0 unpacks
    them per matrix into int64 tensors on `device`."""
    import torch.distributed as dist

    plan = plan_shards(specs, world)
    sizes = [sum(specs[i].blocks for i in p) for p in plan]
    rows = [sum(specs[i].out_features for i in p) for p in plan]
    mine_idx = [local[specs[i].key][0].to(device).reshape(-1) for i in plan[rank]]
    mine_sc = [local[specs[i].key][1].to(device).reshape(-1).view(torch.int16).to(torch.int32) for i in plan[rank]]
    flat_idx = torch.zeros((max(sizes), index_bytes), dtype=torch.uint8, device=device)
    flat_sc = torch.zeros(max(rows), dtype=torch.int32, device=device)
    if mine_idx:
        cat = torch.cat(mine_idx)
        if int(cat.min()) < 0 or (index_bytes < 8 and int(cat.max()) >> (8 * index_bytes)):
            raise ValueError(f"indices do not fit {index_bytes} bytes")
        flat_idx[: cat.numel()] = pack_le_bytes(cat, index_bytes)
        cs = torch.cat(mine_sc)
        flat_sc[: cs.numel()] = cs
    all_idx = [torch.empty_like(flat_idx) for _ in range(world)] if rank == 0 else None
    all_sc = [torch.empty_like(flat_sc) for _ in range(world)] if rank == 0 else None
    dist.gather(flat_idx, all_idx, dst=0)
    dist.gather(flat_sc, all_sc, dst=0)
    if rank != 0:
        return None
    result = {}
    for r in range(world):
        oi, os_ = 0, 0
        gi, gs = unpack_le_bytes(all_idx[r], index_bytes), all_sc[r]
        for i in plan[r]:
            s = specs[i]
            result[s.key] = (gi[oi: oi + s.blocks].view(s.out_features, s.blocks_per_row),
                             gs[os_: os_ + s.out_features].to(torch.int16).view(torch.float16))
            oi += s.blocks
            os_ += s.out_features
    return result


def main():
    import torch.distributed as dist
    from datetime import timedelta

    ap = argparse.ArgumentParser(description="Shard whole-model Λ24 quantization over the GPUs of one node")
    ap.add_argument("--out", type=Path, required=True)
    ap.add_argument("--layers", type=int, default=32)
    ap.add_argument("--rate", type=float, default=2.0)
    ap.add_argument("--seed", type=int, default=2)
    ap.add_argument("--scale-down", type=int, default=1)
    args = ap.parse_args()
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=timedelta(seconds=600), device_id=device)
    specs = llama2_7b_matrices(args.layers, args.scale_down)
    mq = MatrixQuantizer(args.rate, args.seed, device)
    torch.cuda.synchronize()
    dist.barrier()
    t0 = time.perf_counter()
    local_res = run_shard(specs, rank, world, args.out, mq.quantize,
                          fingerprint={"rate": args.rate, "seed": args.seed, "scale_down": args.scale_down})
    torch.cuda.synchronize()
    t_local = torch.tensor([time.perf_counter() - t0], dtype=torch.float64, device=device)
    dist.all_reduce(t_local, op=dist.ReduceOp.MAX)
    result = gather_to_rank0(specs, local_res, rank, world, device, index_bytes=(mq.sg.bits + 7) // 8)
    if rank == 0:
        total = sum(s.blocks for s in specs)
        print(f"{len(result)} matrices, {total} blocks in {t_local.item():.2f} s "
              f"({total / t_local.item() / 1e6:.2f} M blocks/s on {world} GPUs)")
    dist.barrier()
    dist.destroy_process_group()


if __name__ == "__main__":
    main()
