"""Generate golden fixtures by running the reference's own pure-Python CPU
quantizer (impl/leech_lattice_vector_quantizer.py of
dmnunez1993/llvq-paper-reproduction).

Run once in a container where the reference checkout is readable:

    python tests/golden/make_golden.py --reference /path/to/llvq-paper-reproduction

It writes ``tests/golden/reference_quantize.json`` and
``tests/golden/reference_tables.json``.  The fixtures are committed; the test
suite only reads them (the reference does not exist where the GPU tests run).

fp32 inputs are stored as their IEEE bit patterns so the fixtures are exact.
"""
from __future__ import annotations

import argparse
import contextlib
import io
import json
import multiprocessing as mp
import os
import random
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
DIM = 24


def _reference_module(root: str):
    sys.path.insert(0, root)
    from impl import leech_lattice_vector_quantizer as ref  # noqa: E402

    return ref


_Q = {}


def _worker_init(root: str):
    global _REF
    _REF = _reference_module(root)


def _quantize_job(args):
    max_shell, bits = args
    ref = _REF
    q = _Q.get(max_shell)
    if q is None:
        q = ref.LeechLatticeVectorQuantizer(max_shell=max_shell, use_cache=False)
        _Q[max_shell] = q
    x = np.array(bits, dtype=np.uint32).view(np.float32).astype(np.float64)
    buf = io.StringIO()
    with contextlib.redirect_stdout(buf):  # the reference prints on every call
        index = q.quantize(tuple(float(v) for v in x))
    return index, list(q.codeword(index))


def _f32_bits(x: np.ndarray) -> list[int]:
    return [int(b) for b in np.ascontiguousarray(x, dtype=np.float32).view(np.uint32)]


def build_inputs() -> list[dict]:
    """Seeded inputs: Gaussian rows plus the degenerate shapes the domain has
    (zeros, signed zeros, exact ties in |x|, integer-valued rows, rows that are
    scaled lattice points or midpoints of two lattice points, tiny and large
    magnitudes)."""
    cases: list[dict] = []
    rng = np.random.default_rng(20240601)

    def add(name, x, shells):
        cases.append({"name": name, "x": _f32_bits(np.asarray(x, dtype=np.float32)), "shells": shells})

    gauss = rng.standard_normal((64, DIM)).astype(np.float32)
    for i in range(64):
        add(f"gauss_{i}", gauss[i], [2] + ([3] if i < 32 else []) + ([4] if i < 16 else []) + ([5] if i < 8 else []))
    nb = np.random.default_rng(0).normal(size=(8, DIM))[0].astype(np.float32)
    add("notebook_row0", nb, [2, 3, 4, 5, 6])
    for i in range(12):
        add(f"gauss13_{i}", gauss[i], [13])
    add("zeros", np.zeros(DIM), [2, 3, 4, 13])
    add("neg_zeros", -np.zeros(DIM), [2, 3])
    add("ones", np.ones(DIM), [2, 3, 4, 13])
    add("minus_ones", -np.ones(DIM), [2, 3, 4])
    add("test_ipynb_int", [4, 7, 2, 8, 6, 1, 6, 5, 7, 2, 4, 6, 5, 9, 2, 6, 3, 8, 5, 7, 4, 11, 2, 8], [2, 3, 4, 12])
    ints = rng.integers(-3, 4, size=(6, DIM)).astype(np.float32)
    for i in range(6):
        add(f"small_int_{i}", ints[i], [2, 3, 4] + ([13] if i < 2 else []))
    halves = (rng.integers(-6, 7, size=(4, DIM)) / 2.0).astype(np.float32)
    for i in range(4):
        add(f"halves_{i}", halves[i], [2, 3, 4])
    ties = np.abs(rng.standard_normal(DIM)).astype(np.float32)
    ties[::2] = ties[1::2]  # pairs of equal |x|
    ties *= np.where(rng.random(DIM) < 0.5, -1, 1).astype(np.float32)
    add("abs_ties", ties, [2, 3, 4, 13])
    zmix = rng.standard_normal(DIM).astype(np.float32)
    zmix[[1, 5, 9, 17]] = 0.0
    zmix[[2, 11]] = -0.0
    add("signed_zero_mix", zmix, [2, 3, 4])
    add("tiny", (rng.standard_normal(DIM) * 1e-30).astype(np.float32), [2, 3])
    add("subnormal", (rng.standard_normal(DIM) * 1e-41).astype(np.float32), [2])
    add("large", (rng.standard_normal(DIM) * 1e30).astype(np.float32), [2, 3])
    add("one_hot", np.eye(DIM, dtype=np.float32)[7] * 3.0, [2, 3, 4])
    return cases


def lattice_cases(ref, rng: random.Random) -> list[dict]:
    """Rows that are lattice points y/sqrt(8), and midpoints of two shell-2
    points (exact score ties broken by the loop order)."""
    q = ref.LeechLatticeVectorQuantizer(max_shell=3, use_cache=False)
    out = []
    s = ref.LATTICE_SCALE
    for t in range(6):
        idx = rng.randrange(q.total_count)
        y = np.array(q.codeword(idx), dtype=np.float64)
        out.append({"name": f"lattice_point_{t}", "x": _f32_bits((y * s).astype(np.float32)), "shells": [2, 3]})
    for t in range(6):
        a = np.array(q.codeword(rng.randrange(196560)), dtype=np.float64)
        b = np.array(q.codeword(rng.randrange(196560)), dtype=np.float64)
        out.append({"name": f"midpoint_{t}", "x": _f32_bits(((a + b) / 2.0).astype(np.float32)), "shells": [2, 3]})
    return out


def tables(ref, shells=(2, 3, 4, 5, 8, 13)) -> dict:
    out = {}
    for m in shells:
        q = ref.LeechLatticeVectorQuantizer(max_shell=m, use_cache=False)
        rows = []
        for shell in range(2, m + 1):
            for st in q.local_structures[shell]:
                rows.append({
                    "shell": shell,
                    "parity": st.leader.parity,
                    "leader": list(st.leader.leader),
                    "count": st.leader.count,
                    "golay_count": len(st.golay_codeword_indices),
                    "sign_count": st.sign_count,
                    "permutation_count": st.permutation_count,
                    "start": q.shell_offsets[shell] + q.class_offsets[shell][st.class_index],
                })
        out[str(m)] = {
            "total_count": q.total_count,
            "shape_bits": q.shape_bits,
            "shell_counts": {str(k): v for k, v in q.shell_counts.items()},
            "classes": rows,
        }
    return out


def codewords(ref, rng: random.Random) -> list[dict]:
    q = ref.LeechLatticeVectorQuantizer(max_shell=13, use_cache=False)
    picks = [0, 1103, 1104, 196559, 196560, q.total_count - 1]
    offs = [q.shell_offsets[m] for m in range(3, 14)]
    picks += offs + [o - 1 for o in offs]
    while len(picks) < 120:
        picks.append(rng.randrange(q.total_count))
    return [{"max_shell": 13, "index": i, "codeword": list(q.codeword(i))} for i in picks]


def metadata(root: str, shells=(4, 13)) -> dict:
    """The device metadata dicts the reference's GPU API hands its two CUDA
    launchers (_quantize_cuda_metadata / _codeword_cuda_metadata), built on a
    CPU device, with every tensor stored as a nested list plus its dtype."""
    sys.path.insert(0, root)
    from impl import leech_lattice_vector_quantizer_gpu as gpu  # noqa: E402

    def dump(d):
        out = {}
        for k, v in d.items():
            if k == "golay_indices":  # ~1M entries, a pure function of the Golay order; tests rebuild it
                continue
            if hasattr(v, "tolist"):
                out[k] = {"dtype": str(v.dtype).replace("torch.", ""), "data": v.tolist()}
            else:
                out[k] = v
        return out

    res = {}
    for m in shells:
        q = gpu.LeechLatticeVectorQuantizerGpu(max_shell=m, use_cache=False, device="cpu")
        res[str(m)] = {"quantize_meta": dump(q._quantize_cuda_metadata()),
                       "codeword_meta": dump(q._codeword_cuda_metadata()),
                       "comb": q._binom.tolist()}
    return res


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", default=os.environ.get("LLVQ_REFERENCE_ROOT"),
                    help="root of the reference checkout (default: $LLVQ_REFERENCE_ROOT)")
    ap.add_argument("--procs", type=int, default=8)
    ap.add_argument("--only-metadata", action="store_true")
    args = ap.parse_args()
    if not args.reference:
        ap.error("give --reference or set LLVQ_REFERENCE_ROOT")
    (HERE / "reference_metadata.json").write_text(json.dumps({
        "source": "impl/leech_lattice_vector_quantizer_gpu.py _quantize_cuda_metadata / _codeword_cuda_metadata",
        "shells": metadata(args.reference),
    }))
    if args.only_metadata:
        return
    ref = _reference_module(args.reference)
    rng = random.Random(7)

    t0 = time.time()
    cases = build_inputs() + lattice_cases(ref, rng)
    jobs = [(m, c["x"]) for c in cases for m in c["shells"]]
    ctx = mp.get_context("spawn")
    with ctx.Pool(args.procs, initializer=_worker_init, initargs=(args.reference,)) as pool:
        results = pool.map(_quantize_job, jobs, chunksize=1)
    it = iter(results)
    for c in cases:
        c["results"] = {}
        for m in c["shells"]:
            index, cw = next(it)
            c["results"][str(m)] = {"index": index, "codeword": cw}
    (HERE / "reference_quantize.json").write_text(json.dumps({
        "source": "impl/leech_lattice_vector_quantizer.py LeechLatticeVectorQuantizer.quantize (CPython "
                  + sys.version.split()[0] + ")",
        "cases": cases,
    }, indent=0))
    print(f"quantize fixtures: {len(jobs)} calls in {time.time() - t0:.1f}s")

    t0 = time.time()
    (HERE / "reference_tables.json").write_text(json.dumps({
        "source": "impl/leech_lattice_vector_quantizer.py local_structures / offsets",
        "tables": tables(ref),
        "codewords": codewords(ref, rng),
    }, indent=0))
    print(f"table fixtures in {time.time() - t0:.1f}s")


if __name__ == "__main__":
    main()
