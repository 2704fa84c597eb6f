"""ctypes front end of the CPU oracle (test infrastructure only).

The oracle is a C restatement of the reference quantizer
(impl/leech_lattice_vector_quantizer.py of dmnunez1993/llvq-paper-reproduction);
see llvq_oracle.c for the function-by-function citations.  Only the test suite,
``__graft_entry__.smoke()`` and the CPU-baseline leg of ``bench.py`` use it, as
the checker -- the product library never imports it.
"""
from __future__ import annotations

import ctypes
import os
import subprocess
from pathlib import Path

import numpy as np

_HERE = Path(__file__).resolve().parent
_LIB_PATH = _HERE / "_build" / "liboracle.so"
_lib = None

DIM = 24
NGOLAY = 4096


def build(force: bool = False) -> Path:
    """Compile the oracle with its Makefile (gcc only)."""
    if force or not _LIB_PATH.exists() or _LIB_PATH.stat().st_mtime < (_HERE / "llvq_oracle.c").stat().st_mtime:
        subprocess.run(["make", "-s", "-C", str(_HERE)], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not _LIB_PATH.exists():
        build()
    lib = ctypes.CDLL(str(_LIB_PATH))
    vp, i32, i64, u64, dbl = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64, ctypes.c_uint64, ctypes.c_double
    p = ctypes.POINTER
    lib.oracle_create.restype = vp
    lib.oracle_create.argtypes = [ctypes.c_int, ctypes.c_int]
    lib.oracle_destroy.argtypes = [vp]
    lib.oracle_num_classes.restype = ctypes.c_int
    lib.oracle_num_classes.argtypes = [vp]
    lib.oracle_total.restype = u64
    lib.oracle_total.argtypes = [vp]
    lib.oracle_golay_words.argtypes = [vp]
    lib.oracle_class_info.restype = ctypes.c_int
    lib.oracle_class_info.argtypes = [vp, ctypes.c_int, p(i32), p(i32), vp, p(u64), p(u64), p(u64), p(i32), p(i64)]
    lib.oracle_quantize.restype = i64
    lib.oracle_quantize.argtypes = [vp, vp, ctypes.c_int, p(i32), p(i32), p(dbl), vp]
    lib.oracle_quantize_batch.restype = ctypes.c_int
    lib.oracle_quantize_batch.argtypes = [vp, vp, i64, ctypes.c_int, ctypes.c_int, vp, vp, vp, vp]
    lib.oracle_codeword.restype = ctypes.c_int
    lib.oracle_codeword.argtypes = [vp, i64, vp]
    lib.oracle_codeword_batch.restype = i64
    lib.oracle_codeword_batch.argtypes = [vp, vp, i64, vp]
    lib.oracle_codeword_batch_mt.restype = i64
    lib.oracle_codeword_batch_mt.argtypes = [vp, vp, i64, vp, ctypes.c_int]
    lib.oracle_encode.restype = i64
    lib.oracle_encode.argtypes = [vp, vp]
    lib.oracle_rank_even_signs.restype = i64
    lib.oracle_rank_even_signs.argtypes = [vp]
    lib.oracle_rank_even_signs_enumerate.restype = i64
    lib.oracle_rank_even_signs_enumerate.argtypes = [vp]
    lib.oracle_pair_score.restype = dbl
    lib.oracle_pair_score.argtypes = [vp, vp, ctypes.c_int, ctypes.c_int, vp]
    lib.oracle_ref_projection.restype = dbl
    lib.oracle_ref_projection.argtypes = [vp, vp]
    _lib = lib
    return lib


def golay_words() -> np.ndarray:
    """The 4096 extended Golay words in the reference's lexicographic order
    (bit d of each uint32 = coordinate d)."""
    lib = _load()
    out = np.zeros(NGOLAY, dtype=np.uint32)
    lib.oracle_golay_words(out.ctypes.data)
    return out


def ref_projection(x, y) -> float:
    """x.y with CPython 3.12's compensated float sum (reference dot_product)."""
    lib = _load()
    xd = np.ascontiguousarray(x, dtype=np.float64)
    yi = np.ascontiguousarray(y, dtype=np.int32)
    return float(lib.oracle_ref_projection(xd.ctypes.data, yi.ctypes.data))


def rank_even_signs(y, enumerate_masks: bool = False) -> int:
    lib = _load()
    yi = np.ascontiguousarray(y, dtype=np.int32)
    fn = lib.oracle_rank_even_signs_enumerate if enumerate_masks else lib.oracle_rank_even_signs
    return int(fn(yi.ctypes.data))


class OracleBook:
    """The implicit codebook over shells [min_shell, max_shell] (reference: 2..max_shell)."""

    def __init__(self, max_shell: int, min_shell: int = 2):
        self._lib = _load()
        self._h = self._lib.oracle_create(min_shell, max_shell)
        if not self._h:
            raise ValueError(f"oracle cannot build shells {min_shell}..{max_shell}")
        self.min_shell = min_shell
        self.max_shell = max_shell

    def __del__(self):
        h = getattr(self, "_h", None)
        if h:
            self._lib.oracle_destroy(h)
            self._h = None

    @property
    def n_classes(self) -> int:
        return int(self._lib.oracle_num_classes(self._h))

    @property
    def total_count(self) -> int:
        return int(self._lib.oracle_total(self._h))

    def class_info(self, k: int) -> dict:
        shell, parity, gc = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        cnt, sc, pc = ctypes.c_uint64(), ctypes.c_uint64(), ctypes.c_uint64()
        start = ctypes.c_int64()
        leader = np.zeros(DIM, dtype=np.int32)
        r = self._lib.oracle_class_info(self._h, k, ctypes.byref(shell), ctypes.byref(parity), leader.ctypes.data,
                                        ctypes.byref(cnt), ctypes.byref(sc), ctypes.byref(pc), ctypes.byref(gc),
                                        ctypes.byref(start))
        if r:
            raise IndexError(k)
        return {
            "shell": shell.value, "parity": "odd" if parity.value else "even", "leader": tuple(int(v) for v in leader),
            "count": cnt.value, "sign_count": sc.value, "permutation_count": pc.value, "golay_count": gc.value,
            "start": start.value,
        }

    def quantize(self, x, mode: int = 1) -> dict:
        xd = np.ascontiguousarray(x, dtype=np.float64).reshape(DIM)
        g, k = ctypes.c_int32(), ctypes.c_int32()
        s = ctypes.c_double()
        y = np.zeros(DIM, dtype=np.int32)
        idx = self._lib.oracle_quantize(self._h, xd.ctypes.data, mode, ctypes.byref(g), ctypes.byref(k),
                                        ctypes.byref(s), y.ctypes.data)
        return {"index": int(idx), "golay": g.value, "class": k.value, "score": s.value, "codeword": y}

    def quantize_batch(self, x, mode: int = 1, threads: int | None = None):
        """fp32 rows [n,24] -> (index int64[n], golay int32[n], class int32[n], score f64[n])."""
        xf = np.ascontiguousarray(x, dtype=np.float32).reshape(-1, DIM)
        n = xf.shape[0]
        idx = np.zeros(n, dtype=np.int64)
        g = np.zeros(n, dtype=np.int32)
        k = np.zeros(n, dtype=np.int32)
        s = np.zeros(n, dtype=np.float64)
        threads = threads or os.cpu_count() or 1
        self._lib.oracle_quantize_batch(self._h, xf.ctypes.data, n, mode, threads, idx.ctypes.data, g.ctypes.data,
                                        k.ctypes.data, s.ctypes.data)
        return idx, g, k, s

    def codeword(self, index: int) -> tuple[int, ...]:
        """Indices are unsigned 64-bit: pass a Python int below total_count
        (or its two's-complement int64 image)."""
        y = np.zeros(DIM, dtype=np.int32)
        i = int(index) & ((1 << 64) - 1)
        if self._lib.oracle_codeword(self._h, i - (1 << 64) if i >> 63 else i, y.ctypes.data):
            raise IndexError(index)
        return tuple(int(v) for v in y)

    def codeword_batch(self, indices, threads: int = 1) -> np.ndarray:
        """Integer codewords [n, 24] (int32) of int64 indices; threads > 1
        splits the rows over that many POSIX threads (0: all host cores)."""
        idx = np.ascontiguousarray(indices, dtype=np.int64).reshape(-1)
        out = np.zeros((idx.shape[0], DIM), dtype=np.int32)
        threads = threads or os.cpu_count() or 1
        if threads > 1:
            bad = self._lib.oracle_codeword_batch_mt(self._h, idx.ctypes.data, idx.shape[0], out.ctypes.data,
                                                     threads)
        else:
            bad = self._lib.oracle_codeword_batch(self._h, idx.ctypes.data, idx.shape[0], out.ctypes.data)
        if bad:
            raise IndexError(f"{bad} indices out of range")
        return out

    def encode(self, y) -> int:
        yi = np.ascontiguousarray(y, dtype=np.int32).reshape(DIM)
        return int(self._lib.oracle_encode(self._h, yi.ctypes.data))

    def pair_score(self, x, golay: int, cls: int):
        xd = np.ascontiguousarray(x, dtype=np.float64).reshape(DIM)
        y = np.zeros(DIM, dtype=np.int32)
        s = self._lib.oracle_pair_score(self._h, xd.ctypes.data, golay, cls, y.ctypes.data)
        return float(s), y
