"""Build the sm_100a CUDA library in-tree.

1. csrc/gen_search.py emits the straight-line scoring code of the codebooks
   that get a generated search kernel (csrc/_gen/search_gen.cuh).
2. nvcc compiles every csrc/*.cu for sm_100a and links
   llvq_paper_reproduction_b200/_lib/libllvq_b200.so (static CUDA runtime, no
   torch dependency; the C ABI is include/llvq_b200.h).

Usage: python -m llvq_paper_reproduction_b200.build [--force] [--jobs N] [--verbose]
"""
from __future__ import annotations

import argparse
import concurrent.futures as cf
import os
import shutil
import subprocess
import sys
from pathlib import Path

PKG = Path(__file__).resolve().parent
CSRC = PKG / "csrc"
GEN = CSRC / "_gen" / "search_gen.cuh"
BUILD = PKG / "_build"
LIB = PKG / "_lib" / "libllvq_b200.so"
INCLUDE = PKG.parent / "include"

# Codebooks with generated search code: name, min shell, max shell.
# 2..13 is the reference's 48-bit (2 bits/dim) codebook; 2..4 a small
# codebook for fast parity tests of the generated path; single shells 2, 5,
# 11, 23 and 32 are the shape codebooks of the shape-gain quantizer (1, 1.5,
# 2, 2.5 and 3 bits/dim) and 13 is the largest shell that fits 48 bits.
# Other codebooks run the table-driven chains.
SPECS = (("m2_4", 2, 4), ("m2_13", 2, 13), ("s2", 2, 2), ("s5", 5, 5), ("s11", 11, 11), ("s13", 13, 13),
         ("s23", 23, 23), ("s32", 32, 32))
# Angular specs: the multi-shell shape search of shape-gain quantization
# (correlation per unit norm over shells 2..max): 2..4 for fast parity tests,
# 2..5 (33 shape bits, 1.5 bits/dim with 3 gain bits) and 2..10 (44 shape
# bits, 2 bits/dim with 4 gain bits).
ANGULAR_SPECS = (("a2_4", 2, 4), ("a2_5", 2, 5), ("a2_10", 2, 10))

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
NVCC_FLAGS = ["-O3", "-lineinfo", "-std=c++17", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
              "-I", str(CSRC), "-I", str(INCLUDE)]


def nvcc() -> str:
    for cand in (os.environ.get("NVCC"), shutil.which("nvcc"), "/usr/local/cuda/bin/nvcc"):
        if cand and Path(cand).exists():
            return cand
    raise RuntimeError("nvcc not found")


def generate() -> None:
    args = [sys.executable, str(CSRC / "gen_search.py"), str(GEN)] + [f"{n}:{lo}:{hi}" for n, lo, hi in SPECS] + \
        [f"{n}:{lo}:{hi}:a" for n, lo, hi in ANGULAR_SPECS]
    subprocess.run(args, check=True)


def _compile(src: Path, obj: Path, verbose: bool) -> str:
    cmd = [nvcc(), *ARCH, *NVCC_FLAGS, "-c", str(src), "-o", str(obj)]
    if verbose:
        cmd += ["-Xptxas", "-v"]
    res = subprocess.run(cmd, capture_output=True, text=True)
    if res.returncode:
        raise RuntimeError(f"nvcc failed for {src.name}:\n{res.stderr}")
    return res.stderr


def build(force: bool = False, jobs: int | None = None, verbose: bool = False) -> Path:
    generate()
    BUILD.mkdir(exist_ok=True)
    LIB.parent.mkdir(exist_ok=True)
    headers = list(CSRC.glob("*.cuh")) + list(CSRC.glob("*.h")) + [GEN, INCLUDE / "llvq_b200.h"]
    newest_header = max(h.stat().st_mtime for h in headers)
    sources = sorted(CSRC.glob("*.cu"))
    todo = []
    for src in sources:
        obj = BUILD / (src.stem + ".o")
        if force or verbose or not obj.exists() or obj.stat().st_mtime < max(src.stat().st_mtime, newest_header):
            todo.append((src, obj))
    logs = {}
    with cf.ThreadPoolExecutor(max_workers=jobs or os.cpu_count() or 4) as ex:
        futs = {ex.submit(_compile, s, o, verbose): s for s, o in todo}
        for f in cf.as_completed(futs):
            logs[futs[f].name] = f.result()
    objs = [BUILD / (s.stem + ".o") for s in sources]
    if force or todo or not LIB.exists():
        tmp = LIB.with_name(LIB.name + ".tmp")
        subprocess.run([nvcc(), *ARCH, "-shared", "-o", str(tmp), *map(str, objs)], check=True)
        tmp.replace(LIB)
    if verbose:
        for name, log in sorted(logs.items()):
            print(f"== {name}\n{log}")
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--force", action="store_true")
    ap.add_argument("--jobs", type=int, default=None)
    ap.add_argument("--verbose", action="store_true")
    a = ap.parse_args()
    print(build(a.force, a.jobs, a.verbose))
