"""Generate the full-size index fixture of the 65,536-block Gaussian workload.

Workload: 65,536 blocks x 24 i.i.d. N(0, 1) fp32 values from
``torch.randn((65536, 24), generator=torch.Generator().manual_seed(0))`` on the
CPU.  For every block the oracle (the C restatement of the reference CPU
quantizer, impl/leech_lattice_vector_quantizer.py:282-314, in its hoisted
mode, which returns exactly the reference's argmax) gives

  * ``ball``:  the index over shells 2..13 (the 48-bit codebook, the
    reference's own quantize semantics);
  * ``shape``: the index over shell 11 alone (the shape part of the 2
    bits/dim shape-gain code: 45 shape bits + 3 gain bits = 48 bits).

Both are stored as 6-byte little-endian integers (``<u8`` truncated) in
``config1_indices.npz`` with a SHA-256 of the input bytes, so that a test can
tell a changed random generator from a changed quantizer.

    python tests/golden/make_config1.py [--threads N]

Takes about 12 minutes on 8 cores (shells 2..13 dominate).  The test suite
only reads the fixture.
"""
from __future__ import annotations

import argparse
import hashlib
import sys
import time
from pathlib import Path

import numpy as np

HERE = Path(__file__).resolve().parent
ROOT = HERE.parent.parent
N_BLOCKS = 65536
SEED = 0


def workload() -> np.ndarray:
    import torch

    x = torch.randn((N_BLOCKS, 24), generator=torch.Generator().manual_seed(SEED), dtype=torch.float32)
    return x.numpy()


def digest(x: np.ndarray) -> str:
    return hashlib.sha256(np.ascontiguousarray(x, dtype=np.float32).tobytes()).hexdigest()


def pack6(idx: np.ndarray) -> np.ndarray:
    assert int(idx.min()) >= 0 and int(idx.max()) < (1 << 48)
    return np.ascontiguousarray(idx.astype("<u8")).view(np.uint8).reshape(-1, 8)[:, :6].copy()


def unpack6(b: np.ndarray) -> np.ndarray:
    out = np.zeros((b.shape[0], 8), dtype=np.uint8)
    out[:, :6] = b
    return out.view("<u8").reshape(-1).astype(np.int64)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--threads", type=int, default=0)
    args = ap.parse_args()
    sys.path.insert(0, str(ROOT))
    from oracle.oracle import OracleBook

    x = workload()
    out = {"sha256": np.array(digest(x))}
    for name, lo, hi in (("shape", 11, 11), ("ball", 2, 13)):
        t0 = time.time()
        idx = OracleBook(hi, min_shell=lo).quantize_batch(x, mode=1, threads=args.threads or None)[0]
        print(f"{name}: shells {lo}..{hi}, {time.time() - t0:.0f} s", flush=True)
        out[name] = pack6(idx)
    np.savez_compressed(HERE / "config1_indices.npz", **out)


if __name__ == "__main__":
    main()
