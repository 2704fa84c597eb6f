"""Benchmark of the B200 Λ24 quantizer (one JSON line on rank 0).

Primary metric: Λ24 blocks quantized per second on the Gaussian rate-sweep
workload at 2 bits/dim -- N(0,1) fp32 blocks [16,777,216, 24], seed 1 (+rank),
codebook shells 2..13 (48-bit index, the reference's quantize semantics,
bit-exact).  One step = one quantize pass over the whole batch.  Inputs
(1.6 GB) are larger than L2 (126 MB), so no flush is needed between steps.
  value  -- device-resident inputs and outputs, timed with CUDA events on the
            launching stream, barrier + synchronize on both sides, max over ranks.
  e2e    -- the public API (LeechLatticeVectorQuantizerGpu.quantize) fed from
            pinned host memory, host->device copy of the blocks and
            device->host copy of the int64 indices inside the timed region.
Secondary (rank 0, N=1): dequantizer GB/s on all Llama-3-8B linear shapes
(291,307,520 random valid indices, seed 3, bf16 weights with fp16 per-row
scales); dequant-GEMM TFLOP/s on the Llama-3-8B MLP shapes at
M = 1 ... 4096; shape-gain quantization at 1.0 ... 3.0 bits/dim and the
spherical-shaping variant (blocks/s, SQNR).
At every N: whole-model quantization of the Llama-2-7B-shaped linears,
sharded by matrix over the ranks (blocks/s, plus the gather to rank 0).

--impl reference times the reference algorithm on the host cores instead:
the oracle's restatement of LeechLatticeVectorQuantizer.quantize (per-pair
sorting exactly as the reference), all threads, a bounded sample per step.
Multi-GPU: `torchrun --nproc-per-node N bench.py --gpus N`; every rank
quantizes its own batch (weak scaling, no data-path collective).
"""
from __future__ import annotations

import argparse
import json
import os
import subprocess
import sys
import tempfile
import time
from datetime import timedelta
from pathlib import Path

import numpy as np

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

METRIC = "Λ₂₄ blocks/sec quantized, dequant GB/s, fused-GEMM TFLOP/s at 1/2/4/8 B200 vs host CPU"
SMS = 148
FP32_LANES = 128
# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) measured with ncu
# on smaller launches of the same kernels, per unit, for the roofline
# `traffic` entry: the search kernel on 65,536 blocks (6,630,144 + 2,780,160 B)
# and the table-driven bf16 dequant kernel on 9,797,632 indices
# (131,759,104 + 414,060,544 B).
SEARCH_DRAM_BYTES_PER_BLOCK = (6_630_144 + 2_780_160) / 65_536
DEQUANT_DRAM_BYTES_PER_INDEX = (131_759_104 + 414_060_544) / 9_797_632


def log(*a):
    print(*a, file=sys.stderr, flush=True)


def algorithmic_ops_per_block(min_shell: int, max_shell: int) -> float:
    """2 ops per distinct nonzero leader magnitude per evaluated (Golay word,
    class) pair, plus a 24-add prefix sum for each of the 4096 odd and 4096
    even orderings.  Sorting is not counted."""
    from llvq_paper_reproduction_b200.tables import codebook_classes

    weights = {0: 1, 8: 759, 12: 2576, 16: 759, 24: 1}
    ops = 2 * 4096 * 24
    for c in codebook_classes(max_shell, min_shell=min_shell):
        distinct = len({v for v in c.leader if v})
        pairs = 4096 if c.parity else weights[sum(1 for v in c.leader if v % 4 == 2)]
        ops += 2 * distinct * pairs
    return float(ops)


class ClockSampler:
    """nvidia-smi clocks/throttle sampling during the timed region."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.file = None

    def __enter__(self):
        try:
            self.file = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
            self.proc = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                                          "-lms", "200", "-i", str(self.gpu)], stdout=self.file,
                                         stderr=subprocess.DEVNULL)
        except (OSError, FileNotFoundError):
            self.proc = None
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.file is None:
            return {}
        self.file.flush()
        rows = []
        for line in Path(self.file.name).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.file.name)
        if not rows:
            return {}
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({names[i] for _, _, r in rows for i, v in enumerate(r) if v.lower() == "active"})
        return {"sm_mhz": float(np.median([r[0] for r in rows])), "sm_max_mhz": rows[0][1], "reasons": reasons,
                "samples": len(rows)}


def measured_peaks() -> dict:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.exists():
        return json.loads(p.read_text())
    return {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "fallback": True}


# ----------------------------------------------------------------- CPU side

def cpu_reference_rate(x: np.ndarray, max_shell: int, mode: int = 0) -> tuple[float, int]:
    """Blocks/s of the oracle restatement of the reference CPU quantizer on
    the rows of x, all host threads."""
    from oracle.oracle import OracleBook

    threads = os.cpu_count() or 1
    ob = OracleBook(max_shell)
    t0 = time.perf_counter()
    ob.quantize_batch(x, mode=mode, threads=threads)
    return x.shape[0] / (time.perf_counter() - t0), threads


def reference_gpu_bench(blocks: int = 2048, n_dequant: int = 1 << 20) -> dict:
    """The reference's own GPU path (its NVRTC kernels, through its unmodified
    LeechLatticeVectorQuantizerGpu installed in baseline/_ref) timed on this
    GPU beside this library on the same inputs: quantize (shells 2..13) of
    N(0,1) blocks and dequantize_lattice of random valid indices (int64
    codewords, the reference's output kind).  Index agreement is counted:
    this library returns the reference CPU quantizer's indices; the NVRTC
    kernel scores in fp32 and may differ on near-ties."""
    import torch

    ref_root = ROOT / "baseline" / "_ref"
    if not (ref_root / "impl" / "leech_lattice_vector_quantizer_gpu.py").exists():
        return {"unavailable": "reference not installed in baseline/_ref"}
    if str(ref_root) not in sys.path:
        sys.path.insert(0, str(ref_root))
    try:
        from impl.leech_lattice_vector_quantizer_gpu import LeechLatticeVectorQuantizerGpu as RefGpu
    except Exception as exc:  # the reference's optional CUDA imports failed
        return {"unavailable": f"reference import failed: {exc!r}"[:200]}
    from llvq_paper_reproduction_b200 import LeechLatticeVectorQuantizerGpu

    dev = torch.device("cuda", 0)
    stream = torch.cuda.current_stream()
    with tempfile.TemporaryDirectory() as cache:
        ref = RefGpu(max_shell=13, cache_dir=cache, use_cache=False, device=dev)
    ours = LeechLatticeVectorQuantizerGpu(max_shell=13, use_cache=False, device=dev)

    def timed(fn, reps: int) -> float:
        fn()  # first call: NVRTC compile / codebook upload
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(reps):
            fn()
        e1.record(stream)
        torch.cuda.synchronize()
        return e0.elapsed_time(e1) / 1000.0 / reps

    x = torch.randn((blocks, 24), generator=torch.Generator().manual_seed(1), dtype=torch.float32).to(dev)
    t_ref = timed(lambda: ref.quantize_cuda(x), 3)
    t_ours = timed(lambda: ours.quantize(x), 3)
    equal = int((ref.quantize_cuda(x) == ours.quantize(x)).sum().item())
    g = torch.Generator(device=dev).manual_seed(3)
    idx = torch.randint(0, ours.total_count, (n_dequant,), generator=g, device=dev)
    td_ref = timed(lambda: ref.dequantize_lattice_cuda(idx), 5)
    td_ours = timed(lambda: ours.dequantize_lattice(idx), 5)
    ref_cw, our_cw = ref.dequantize_lattice_cuda(idx), ours.dequantize_lattice(idx)
    differ = (ref_cw != our_cw.view_as(ref_cw)).any(dim=1)
    n_differ = int(differ.sum().item())
    # where the two disagree, ask the reference's own CPU codeword() (pure Python)
    sample = idx[differ][:16].tolist()
    ref_cpu_agrees = {"b200": 0, "reference_gpu": 0, "checked": len(sample)}
    for i, v in zip(sample, torch.nonzero(differ).view(-1)[:16].tolist()):
        truth = tuple(ref.codeword(int(i)))
        ref_cpu_agrees["b200"] += tuple(our_cw.view_as(ref_cw)[v].tolist()) == truth
        ref_cpu_agrees["reference_gpu"] += tuple(ref_cw[v].tolist()) == truth
    nbytes = n_dequant * (8 + 24 * 8)
    return {
        "workload": f"quantize: {blocks} N(0,1) blocks (torch CPU generator seed 1), shells 2..13; "
                    f"dequantize_lattice: {n_dequant} indices uniform over [0, total) (seed 3), int64 codewords",
        "kernels": "reference NVRTC kernels (compute_100 PTX, JIT) through its LeechLatticeVectorQuantizerGpu, "
                   "against this library's sm_100a kernels, same GPU, same inputs",
        "quantize": {"reference_blocks_per_s": blocks / t_ref, "b200_blocks_per_s": blocks / t_ours,
                     "speedup": t_ref / t_ours, "index_equal": equal, "blocks": blocks},
        "dequantize_lattice": {"reference_gbs": nbytes / td_ref / 1e9, "b200_gbs": nbytes / td_ours / 1e9,
                               "speedup": td_ref / td_ours, "rows_differing": n_differ,
                               "reference_cpu_codeword_agrees_on_differing_sample": ref_cpu_agrees,
                               "indices": n_dequant},
    }


def run_reference_arm(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch

    sample = args.cpu_sample
    g = torch.Generator().manual_seed(1)
    x = torch.randn((sample * (args.steps + args.warmup), 24), generator=g, dtype=torch.float32).numpy()
    rates = []
    threads = 1
    for s in range(args.warmup + args.steps):
        r, threads = cpu_reference_rate(x[s * sample:(s + 1) * sample], args.max_shell)
        if s >= args.warmup:
            rates.append(r)
    value = float(np.mean(rates))
    desc = (f"{sample} N(0,1) blocks per step from the [16777216, 24] seed-1 workload, shells 2..{args.max_shell}; "
            "oracle restatement of LeechLatticeVectorQuantizer.quantize with per-pair sorts (mode 0)")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "blocks/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": 1000.0 * sample / value,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64", "data": "synthetic",
        "config": {"workload": f"gaussian N(0,1) fp32 [16777216, 24] seed 1, shells 2..{args.max_shell} "
                               "(48-bit index), CPU sample", "sample_blocks_per_step": sample},
        "cpu_baseline": {"value": value, "unit": "blocks/s", "cores": threads, "kind": "port", "sample": desc},
        "e2e": {"value": value, "unit": "blocks/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    if not args.skip_reference_gpu:
        try:
            import torch

            line["reference_gpu"] = (reference_gpu_bench() if torch.cuda.is_available()
                                     else {"unavailable": "no CUDA device"})
        except Exception as exc:  # keep the CPU baseline line whatever the GPU comparison does
            line["reference_gpu"] = {"unavailable": f"{exc!r}"[:200]}
    print(json.dumps(line), flush=True)


# ----------------------------------------------------------------- GPU side

def llama3_dequant_workload(q, device, seed: int = 3, layers: int = 32):
    """Random valid indices of every Llama-3-8B linear (uniform shell, class
    within shell, local index) and fp16 per-row scales, grouped by blocks per
    row: in-dim 4096 -> 171 blocks (4104), in-dim 14336 -> 598 blocks (14352)."""
    import torch

    groups = {171: layers * (4096 + 1024 + 1024 + 4096 + 14336 + 14336), 598: layers * 4096}
    g = torch.Generator(device=device).manual_seed(seed)
    flat = [st for s in q.classes_by_shell for st in q.local_structures[s]]
    starts, counts = [], []
    for s in q.classes_by_shell:
        for i, st in enumerate(q.local_structures[s]):
            starts.append(q.shell_offsets[s] + q.class_offsets[s][i])
            counts.append(st.count)
    shells = sorted(q.classes_by_shell)
    first = []
    k = 0
    for s in shells:
        first.append(k)
        k += len(q.classes_by_shell[s])
    ncls = torch.tensor([len(q.classes_by_shell[s]) for s in shells], device=device)
    first = torch.tensor(first, device=device)
    starts = torch.tensor(starts, dtype=torch.long, device=device)
    counts = torch.tensor(counts, dtype=torch.float64, device=device)
    out = {}
    for bpr, rows in groups.items():
        n = rows * bpr
        sh = torch.randint(0, len(shells), (n,), generator=g, device=device)
        cls = first[sh] + (torch.rand(n, generator=g, device=device, dtype=torch.float64) * ncls[sh]).long()
        del sh
        local = (torch.rand(n, generator=g, device=device, dtype=torch.float64) * counts[cls]).long()
        idx = (starts[cls] + local).reshape(rows, bpr)
        del cls, local
        scale = (torch.rand(rows, generator=g, device=device) * 0.04 + 0.005).to(torch.float16)
        out[bpr] = (idx, scale)
    assert len(flat) == len(starts)
    return out


def run_gpu_arm(args) -> None:
    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    device = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=300), device_id=device)

    from llvq_paper_reproduction_b200 import LeechLatticeVectorQuantizerGpu

    q = LeechLatticeVectorQuantizerGpu(max_shell=args.max_shell, use_cache=False, device=device)
    book = q._book()
    n = args.rows
    g = torch.Generator(device=device).manual_seed(1 + rank)
    x = torch.randn((n, 24), generator=g, device=device, dtype=torch.float32)
    idx = torch.empty(n, dtype=torch.long, device=device)
    pair = torch.empty(n, dtype=torch.long, device=device)
    score = torch.empty(n, dtype=torch.float32, device=device)
    stream = torch.cuda.current_stream()

    def step():
        book.quantize(x.data_ptr(), n, idx.data_ptr(), pair.data_ptr(), score.data_ptr(), stream.cuda_stream)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], dtype=torch.float64, device=device)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
    barrier()
    torch.cuda.synchronize()
    ms = max_over_ranks(e0.elapsed_time(e1)) / args.steps
    value = world * n / (ms / 1000.0)

    # end to end through the public API, pinned host input and output
    x_host = x.cpu().pin_memory()
    host_out = torch.empty(n, dtype=torch.long).pin_memory()
    for _ in range(1):
        host_out.copy_(q.quantize(x_host))
    torch.cuda.synchronize()
    barrier()
    e2 = torch.cuda.Event(enable_timing=True)
    e3 = torch.cuda.Event(enable_timing=True)
    e2e_steps = max(1, min(args.steps, 3))
    e2.record(stream)
    for _ in range(e2e_steps):
        r = q.quantize(x_host)
        host_out.copy_(r, non_blocking=True)
    e3.record(stream)
    torch.cuda.synchronize()
    barrier()
    e2e_ms = max_over_ranks(e2.elapsed_time(e3)) / e2e_steps
    if not torch.equal(host_out, idx.cpu()):
        raise RuntimeError("end-to-end indices differ from the device-resident run")

    extra = {}
    mq = None
    if args.model_layers > 0:  # every rank takes part (sharded by matrix)
        mq = model_quant_bench(rank, world, device, stream, args, barrier, max_over_ranks)
    if rank == 0 and world == 1 and args.sweep_rows > 0:
        extra["rate_sweep"] = rate_sweep_bench(q, x, device, stream, args)
    if rank == 0 and world == 1 and not args.skip_gemm:
        extra["gemm"] = gemm_bench(q, device, stream, args)
    if rank == 0 and world == 1 and not args.skip_dequant:
        extra["dequant"] = dequant_bench(q, device, stream, args)
    if rank == 0 and world == 1 and not args.skip_config1:
        extra["config1"] = config1_bench(q, device, stream)
    if rank == 0 and mq is not None:
        extra["model_quant"] = mq  # last: the end of the line is what a truncated log keeps
    cpu = None
    if rank == 0 and world == 1 and args.cpu_sample > 0:
        sample = x_host[: args.cpu_sample].numpy()
        rate, threads = cpu_reference_rate(sample, args.max_shell)
        cpu = {"value": rate, "unit": "blocks/s", "cores": threads, "kind": "port",
               "sample": f"first {args.cpu_sample} blocks of the same workload; oracle restatement of "
                         "LeechLatticeVectorQuantizer.quantize with per-pair sorts (mode 0), all host threads"}
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return
    ops = algorithmic_ops_per_block(2, args.max_shell)
    clk = clocks.summary()
    peak_tflops = SMS * FP32_LANES * 2 * (clk.get("sm_max_mhz") or 1965.0) * 1e6 / 1e12
    achieved = ops * n / (ms / 1000.0) / 1e12
    line = {
        "metric": METRIC, "value": value, "unit": "blocks/s", "n_gpus": world, "steps": args.steps,
        "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": f"gaussian N(0,1) fp32 [{n}, 24] per GPU, seed 1+rank, shells 2..{args.max_shell} "
                               "(48-bit index), bit-exact reference quantize", "blocks_per_gpu": n,
                   "l2": "inputs (1.6 GB) larger than L2, no flush", "parallelism": f"weak x{world}"},
        "e2e": {"value": world * n / (e2e_ms / 1000.0), "unit": "blocks/s", "h2d_bytes_per_step": world * n * 96,
                "d2h_bytes_per_step": world * n * 8},
        "gpu_launches": 2 * args.steps,
        "roofline": {"bound": "alu", "achieved": achieved, "peak": peak_tflops, "unit": "TFLOP/s",
                     "frac": achieved / peak_tflops, "traffic": SEARCH_DRAM_BYTES_PER_BLOCK * n,
                     "traffic_unit": "bytes per launch (ncu on 65,536 blocks, scaled by blocks)",
                     "note": f"{ops / 1e6:.3f} M algorithmic ops/block (2 per distinct nonzero leader value per "
                             "evaluated pair + 2x4096x24 prefix adds); peak = 148 SMs x 128 FP32 lanes x 2 x "
                             "max SM clock (FFMA); achieved over the whole quantize step (search + finalize "
                             "kernels; the search kernel is 97% of its device time in the launch list)"},
        "clocks": clk,
    }
    if cpu:
        line["cpu_baseline"] = cpu
    line.update(extra)
    print(json.dumps(line), flush=True)


def model_quant_bench(rank, world, device, stream, args, barrier, max_over_ranks) -> dict:
    """Whole-model quantization of the Llama-2-7B-shaped linears (the first
    --model-layers layers; seed 2): each rank quantizes its greedy share of
    whole matrices (synthetic fp16 weights, Hadamard rotation, row scales,
    shape-gain at 2 bits/dim) with no inter-GPU traffic, timed with CUDA
    events on the launching stream (max over ranks); then one gather brings
    every index tensor and row scale to rank 0, timed separately the same way."""
    import torch

    from llvq_paper_reproduction_b200.model_quant import (MatrixQuantizer, MatrixSpec, gather_to_rank0,
                                                          llama2_7b_matrices, plan_shards)

    specs = llama2_7b_matrices(args.model_layers)
    mine = plan_shards(specs, world)[rank]
    mq = MatrixQuantizer(2.0, seed=2, device=device)
    mq.quantize(MatrixSpec(0, "q_proj", 256, 4096))  # codebook upload and first launches
    torch.cuda.synchronize()
    barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    results = {specs[i].key: mq.quantize(specs[i]) for i in mine}
    e1.record(stream)
    torch.cuda.synchronize()
    barrier()
    own_s = e0.elapsed_time(e1) / 1000.0
    secs = max_over_ranks(own_s)
    # strong-scaling efficiency: the job rate against N times the mean of
    # the ranks' own rates on their shards (each rank runs the one-GPU code
    # path on its matrices, so that mean stands for the one-GPU rate)
    own_blocks = sum(specs[i].blocks for i in mine)
    mean_rate = own_blocks / own_s
    if world > 1:
        import torch.distributed as dist

        t = torch.tensor([mean_rate], dtype=torch.float64, device=device)
        dist.all_reduce(t)
        mean_rate = float(t.item()) / world
    if world > 1:  # set up the point-to-point connections of the gather outside the timed region
        import torch.distributed as dist

        probe = torch.zeros(1, dtype=torch.int32, device=device)
        dist.gather(probe, [torch.empty_like(probe) for _ in range(world)] if rank == 0 else None, dst=0)
        torch.cuda.synchronize()
        barrier()
    # the gather timed on the device (CUDA events on the stream its packing,
    # NCCL gather and unpacking are ordered on), max over ranks, twice: the
    # first includes NCCL's one-time setup of its large point-to-point
    # transfers (about 50 ms at 2 GPUs), the second is the steady state
    local = {k: (r["indices"], r["row_scale"]) for k, r in results.items()}  # stay on the device
    index_bytes = (mq.sg.bits + 7) // 8  # 48-bit shape-gain index -> 6 bytes per block on the wire
    times = []
    for _ in range(2):
        g0, g1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        g0.record(stream)
        gathered = gather_to_rank0(specs, local, rank, world, device, index_bytes) if world > 1 else local
        g1.record(stream)
        torch.cuda.synchronize()
        barrier()
        times.append(max_over_ranks(g0.elapsed_time(g1) / 1000.0))
    gather_first_s, gather_s = times
    total = sum(s.blocks for s in specs)
    if rank == 0 and len(gathered) != len(specs):
        raise RuntimeError("gather lost matrices")
    return {"workload": f"Llama-2-7B linears x{args.model_layers} layers, {total} blocks, shape-gain 2 b/dim, "
                        "sharded by matrix (strong scaling)", "n_gpus": world, "seconds": secs,
            "blocks_per_s": total / secs, "mean_gpu_blocks_per_s": mean_rate,
            "strong_efficiency": (total / secs) / (world * mean_rate),
            "gather_seconds": gather_s, "gather_first_seconds": gather_first_s,
            "gather_bytes": total * index_bytes + sum(s.out_features for s in specs) * 4}


def rate_sweep_bench(q, x, device, stream, args) -> dict:
    """Shape-gain quantization of the same N(0,1) blocks at 1.0 ... 3.0
    bits/dim (single shell + chi(24)-matched gain code, shaping.rate_split),
    the multi-shell shape-gain variant at 1.5 and 2.0 bits/dim (shells 2..5 and
    2..10 by correlation per unit norm) and the spherical-shaping variant at 2 bits/dim (shells 2..13 ball, global
    beta): blocks/s of the full quantize call (shape search, gain, index
    packing) on a sample of the batch, and SQNR in dB of the reconstruction.
    The sample is the first --sweep-rows blocks, cut so that one rate takes
    about 10 s when its search is slow (the 2.5 and 3.0 bits/dim shells 23
    and 32 have the largest scoring codes)."""
    import math

    import torch

    from llvq_paper_reproduction_b200.shaping import ShapeGainQuantizer, SphericalShaping

    def timed(fn, rows):
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        out = fn(rows)
        e1.record(stream)
        torch.cuda.synchronize()
        return out, e0.elapsed_time(e1) / 1000.0

    def sqnr_db(xs, rec):
        err = (xs.double() - rec.double()).pow(2).sum().item()
        return 10.0 * math.log10(xs.double().pow(2).sum().item() / err)

    out = {}
    probe = x[:65536]

    def run(name, quant, dequant, bits):
        quant(probe[:4096])  # codebook upload and first-launch setup
        _, t_probe = timed(lambda r: quant(r), probe)
        rows = int(min(args.sweep_rows, x.shape[0], max(65536, 10.0 / max(t_probe / probe.shape[0], 1e-12))))
        xs = x[:rows]
        idx, t = timed(lambda r: quant(r), xs)
        out[name] = {"bits_per_dim": bits, "blocks": rows, "blocks_per_s": rows / t,
                     "sqnr_db": sqnr_db(xs, dequant(idx).reshape(xs.shape))}

    design = torch.randn((65536, 24), generator=torch.Generator().manual_seed(7)).to(device)

    def post_shape(name, sg):
        # the same code refitted after the shape quantizer on a separate
        # seeded sample (optimal post-shape scales); SQNR of both codes on
        # the first 65,536 blocks
        chi = sqnr_db(probe, sg.dequantize_parts(*sg.quantize_parts(probe)))
        sg.fit_gain_code(design)
        fitted = sqnr_db(probe, sg.dequantize_parts(*sg.quantize_parts(probe)))
        out[name]["post_shape_gain_code"] = {"sqnr_db": fitted, "chi_code_sqnr_db": chi, "blocks": probe.shape[0],
                                             "design": "65,536 N(0,1) blocks, seed 7"}

    for rate in (1.0, 1.5, 2.0, 2.5, 3.0):
        sg = ShapeGainQuantizer.for_rate(rate, device=device)
        # (shape, gain) index pairs: 3.0 bits/dim needs 72 bits
        run(f"shape_gain_{rate}", sg.quantize_parts, lambda p, sg=sg: sg.dequantize_parts(*p), sg.bits / 24)
        out[f"shape_gain_{rate}"].update({"shell": sg.shell, "gain_bits": sg.gain_bits})
        post_shape(f"shape_gain_{rate}", sg)
        del sg
    for rate in (1.5, 2.0):  # multi-shell shape (shells 2..m by correlation per unit norm) + gain
        sg = ShapeGainQuantizer.for_rate(rate, device=device, multi_shell=True)
        run(f"multi_shell_{rate}", sg.quantize_parts, lambda p, sg=sg: sg.dequantize_parts(*p), sg.bits / 24)
        out[f"multi_shell_{rate}"].update({"shells": [sg.min_shell, sg.shell], "gain_bits": sg.gain_bits})
        post_shape(f"multi_shell_{rate}", sg)
        del sg
    sph = SphericalShaping(q)
    run("spherical_2.0", sph.quantize, sph.dequantize, q.shape_bits / 24)
    out["spherical_2.0"]["beta"] = sph.beta
    return {"workload": "the first blocks of the same N(0,1) batch (seed 1); blocks/s of the whole quantize call "
                        "(search + gain code + packing), SQNR = 10 log10(|x|^2 / |x - x_hat|^2); "
                        "post_shape_gain_code: the gain code refitted after the shape quantizer", "by_rate": out}


def config1_bench(q, device, stream) -> dict:
    """The 65,536-block Gaussian workload (N(0,1) fp32, torch CPU generator
    seed 0): shape-gain at 2 bits/dim (shell-11 shape, 45 bits, + 3-bit
    chi(24) gain code = 48 bits per block) and the reference's own quantize
    over shells 2..13.  Indices are compared one by one with the committed
    fixture of the oracle (the reference CPU quantizer restated, run over
    every block: tests/golden/make_config1.py); SQNR of each reconstruction."""
    import hashlib
    import math

    import torch

    from llvq_paper_reproduction_b200.shaping import ShapeGainQuantizer

    x = torch.randn((65536, 24), generator=torch.Generator().manual_seed(0), dtype=torch.float32)
    fx_path = ROOT / "tests" / "golden" / "config1_indices.npz"
    fx = np.load(fx_path) if fx_path.exists() else None
    digest_ok = fx is not None and hashlib.sha256(x.numpy().tobytes()).hexdigest() == str(fx["sha256"])

    def unpack6(b):
        out = np.zeros((b.shape[0], 8), dtype=np.uint8)
        out[:, :6] = b
        return out.view("<u8").reshape(-1).astype(np.int64)

    def sqnr_db(rec):
        xd = x.double()
        return 10.0 * math.log10(xd.pow(2).sum().item() / (xd - rec.double().cpu()).pow(2).sum().item())

    xd = x.to(device)
    sg = ShapeGainQuantizer.for_rate(2.0, device=device)
    sg.quantize_parts(xd[:1024])
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    sidx, gidx = sg.quantize_parts(xd)
    e1.record(stream)
    torch.cuda.synchronize()
    t_sg = e0.elapsed_time(e1) / 1000.0
    ball = q.quantize(xd)
    out = {"blocks": 65536, "input_sha256_matches_fixture": digest_ok,
           "shape_gain_2.0": {"shell": sg.shell, "bits": sg.bits, "blocks_per_s": 65536 / t_sg,
                              "sqnr_db": sqnr_db(sg.dequantize_parts(sidx, gidx))},
           "ball_2..13": {"bits": q.shape_bits, "sqnr_db_at_unit_scale": sqnr_db(q.dequantize(ball))}}
    if fx is not None:
        out["shape_gain_2.0"]["shape_index_equal"] = int((sidx.cpu().numpy() == unpack6(fx["shape"])).sum())
        out["ball_2..13"]["index_equal"] = int((ball.cpu().numpy() == unpack6(fx["ball"])).sum())
    return out


def dequant_bench(q, device, stream, args) -> dict:
    import torch

    work = llama3_dequant_workload(q, device, layers=args.dequant_layers)
    book = q._book()
    outs = {bpr: torch.empty((idx.shape[0], bpr * 24), dtype=torch.bfloat16, device=device)
            for bpr, (idx, _) in work.items()}
    n_idx = sum(idx.numel() for idx, _ in work.values())
    n_rows = sum(idx.shape[0] for idx, _ in work.values())

    def step():
        for bpr, (idx, scale) in work.items():
            book.dequantize_bf16(idx.data_ptr(), idx.numel(), scale.data_ptr(), bpr, outs[bpr].data_ptr(), None,
                                 stream.cuda_stream)

    for _ in range(3):
        step()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(args.steps):
        step()
    e1.record(stream)
    torch.cuda.synchronize()
    ms = e0.elapsed_time(e1) / args.steps
    algo_bytes = n_idx * (8 + 48) + n_rows * 2
    gbs = algo_bytes / (ms / 1000.0) / 1e9
    peaks = measured_peaks()
    # host reference: the oracle's restatement of the reference codeword()
    # per index (one thread) on a sample of the same indices
    from oracle.oracle import OracleBook

    sample = next(iter(work.values()))[0].reshape(-1)[: args.cpu_dequant_sample].cpu().numpy()
    ob = OracleBook(args.max_shell)
    t0 = time.perf_counter()
    ob.codeword_batch(sample)
    cpu_rate = sample.shape[0] / (time.perf_counter() - t0)
    del outs, work
    torch.cuda.empty_cache()
    return {"value": gbs, "unit": "GB/s", "ms_per_step": ms, "indices": n_idx, "rows": n_rows,
            "cpu_baseline": {"value": cpu_rate * 56 / 1e9, "unit": "GB/s", "indices_per_s": cpu_rate, "cores": 1,
                             "kind": "port", "sample": f"first {sample.shape[0]} indices of the workload; oracle "
                                                       "restatement of the reference codeword() (int32 codewords)"},
            "workload": f"Llama-3-8B linears ({args.dequant_layers} layers), random valid int64 indices seed 3, "
                        "bf16 out, fp16 row scales",
            "gpu_launches": 2 * args.steps,
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": peaks["hbm_gbs"], "unit": "GB/s",
                         "frac": gbs / peaks["hbm_gbs"],
                         "traffic": DEQUANT_DRAM_BYTES_PER_INDEX * n_idx,
                         "traffic_unit": "bytes per step (ncu on 9,797,632 indices, scaled by indices)",
                         "note": "56 B per index (8 B int64 index + 48 B bf16) + 2 B per row; the kernel is "
                                 "SM-bound (about 790 thread instructions per index under ncu, ALU pipe 65%, "
                                 "L1/shared data pipe 61%), not HBM-bound; peak of "
                                 + ("fallback" if peaks.get("fallback") else "measured") + " copy bandwidth"}}


def gemm_bench(q, device, stream, args) -> dict:
    """Dequant-GEMM on the Llama-3-8B MLP shapes: W 14336 x 4096 (171
    blocks per row) and 4096 x 14336 (598 blocks per row), random valid
    indices (seed 4) with fp16 row scales, bf16 activations N(0,1) [M, K]."""
    import torch

    g = torch.Generator(device=device).manual_seed(4)
    mats = []
    for n_out, k in ((14336, 4096), (4096, 14336)):
        bpr = (k + 23) // 24
        idx = torch.randint(0, q.total_count, (n_out, bpr), generator=g, device=device)
        scale = (torch.rand(n_out, generator=g, device=device) * 0.04 + 0.005).to(torch.float16)
        mats.append((n_out, k, bpr, idx, scale))
    book = q._book()
    peaks = measured_peaks()
    out = {}
    for m in args.gemm_m:
        acts = [torch.randn((m, k), generator=g, device=device).to(torch.bfloat16) for _, k, _, _, _ in mats]
        ys = [torch.empty((m, n), dtype=torch.float32, device=device) for n, _, _, _, _ in mats]

        def step():
            for (n_out, k, bpr, idx, scale), a, y in zip(mats, acts, ys):
                book.gemm(idx.data_ptr(), n_out, bpr, scale.data_ptr(), a.data_ptr(), m, k, y.data_ptr(), None,
                          stream.cuda_stream)

        for _ in range(3):
            step()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(args.steps):
            step()
        e1.record(stream)
        torch.cuda.synchronize()
        ms = e0.elapsed_time(e1) / args.steps
        flops = sum(2.0 * m * n * k for n, k, _, _, _ in mats)
        tflops = flops / (ms / 1000.0) / 1e12
        nbytes = sum(n * bpr * 8 + n * 2 + m * k * 2 + m * n * 4 for n, k, bpr, _, _ in mats)
        t_tensor = flops / (peaks["bf16_tflops"] * 1e12)
        t_hbm = nbytes / (peaks["hbm_gbs"] * 1e9)
        bound = "tensor" if t_tensor >= t_hbm else "hbm"
        out[str(m)] = {"tflops": tflops, "ms": ms,
                       "roofline": {"bound": bound, "time_frac": max(t_tensor, t_hbm) / (ms / 1000.0),
                                    "achieved": tflops if bound == "tensor" else nbytes / (ms / 1000.0) / 1e9,
                                    "peak": peaks["bf16_tflops"] if bound == "tensor" else peaks["hbm_gbs"],
                                    "unit": "TFLOP/s" if bound == "tensor" else "GB/s"}}
        del acts, ys
    return {"workload": "Llama-3-8B MLP weights 14336x4096 + 4096x14336, random valid indices seed 4, fp16 row "
                        "scales, bf16 activations N(0,1), fp32 out", "by_m": out,
            "gpu_launches": args.steps * len(args.gemm_m) * sum(2 * gemm_chunks(n, bpr) for n, _, bpr, _, _ in mats)}


def gemm_chunks(n_out: int, bpr: int, budget: int = 256 << 20) -> int:
    """Staging chunks of one dequant-GEMM call (one decode and one GEMM
    launch each): rows of 24 * bpr bf16 columns padded to 64, at most
    `budget` bytes (the library's stream-ordered staging limit)."""
    row_bytes = (24 * bpr + 63) // 64 * 64 * 2
    rows = min(n_out, max(128, budget // row_bytes // 128 * 128))
    return -(-n_out // rows)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=5)
    ap.add_argument("--warmup", type=int, default=3)
    ap.add_argument("--impl", choices=("b200", "reference"), default="b200")
    ap.add_argument("--rows", type=int, default=16_777_216)
    ap.add_argument("--max-shell", type=int, default=13)
    ap.add_argument("--cpu-sample", type=int, default=96)
    ap.add_argument("--skip-dequant", action="store_true")
    ap.add_argument("--dequant-layers", type=int, default=32)
    ap.add_argument("--cpu-dequant-sample", type=int, default=200_000)
    ap.add_argument("--skip-gemm", action="store_true")
    ap.add_argument("--skip-config1", action="store_true")
    ap.add_argument("--skip-reference-gpu", action="store_true",
                    help="--impl reference: skip timing the reference's NVRTC kernels on the GPU")
    ap.add_argument("--model-layers", type=int, default=32,
                    help="Llama-2-7B layers of the whole-model quantization section (0 skips it)")
    ap.add_argument("--sweep-rows", type=int, default=4_194_304,
                    help="blocks of the rate sweep sample (0 skips the sweep)")
    ap.add_argument("--gemm-m", type=int, nargs="+", default=[1, 8, 64, 512, 4096])
    args = ap.parse_args()
    if args.impl == "reference":
        run_reference_arm(args)
    else:
        run_gpu_arm(args)


if __name__ == "__main__":
    main()
