"""ctypes binding of the in-tree CUDA library (include/llvq_b200.h).

The library is the only compute path: if it is missing this module raises at
import time instead of falling back to anything else.  Status codes map to
the exception types the reference raises (ValueError, RuntimeError,
IndexError).
"""
from __future__ import annotations

import ctypes
import threading
from pathlib import Path
from typing import Sequence

import numpy as np

LIB_PATH = Path(__file__).resolve().parent / "_lib" / "libllvq_b200.so"

OK = 0
ERR_INVALID_ARGUMENT = 1
ERR_CUDA = 2
ERR_UNSUPPORTED = 3
ERR_OUT_OF_MEMORY = 4
ERR_INDEX_RANGE = 5
ERR_NOT_A_CODEWORD = 6

OUT_INT64 = 0
OUT_F32 = 1
OUT_F32_DOUBLE = 2
OUT_BF16_ROWSCALE = 3
FLAG_TABLE_DRIVEN = 1
GAIN_PACK = 1
GAIN_ANGULAR = 2

# Every symbol the public header declares (checked by the CPU test suite).
EXPORTS = (
    "llvq_codebook_create", "llvq_codebook_destroy", "llvq_codebook_info", "llvq_quantize", "llvq_quantize_ex",
    "llvq_dequantize_lattice", "llvq_dequantize", "llvq_dequantize_bf16", "llvq_codeword_host",
    "llvq_encode_host", "llvq_status_string", "llvq_last_error", "llvq_version", "llvq_gemm",
    "llvq_hadamard", "llvq_gemm_noalloc", "llvq_pack_indices", "llvq_unpack_indices", "llvq_dequantize_packed",
    "llvq_gemm_packed", "llvq_hadamard_ex", "llvq_codeword_batch_host", "llvq_codebook_tables",
    "llvq_quantize_gain", "llvq_rotate_scale",
)

_lib = None
_lock = threading.Lock()


def load() -> ctypes.CDLL:
    global _lib
    if _lib is not None:
        return _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not LIB_PATH.exists():
            raise ImportError(f"{LIB_PATH} is missing: build it with `python -m llvq_paper_reproduction_b200.build`")
        lib = ctypes.CDLL(str(LIB_PATH))
        vp, i32, i64 = ctypes.c_void_p, ctypes.c_int32, ctypes.c_int64
        P = ctypes.POINTER
        sig = {
            "llvq_codebook_create": (ctypes.c_int, [i32, vp, vp, vp, ctypes.c_int, P(vp)]),
            "llvq_codebook_destroy": (None, [vp]),
            "llvq_codebook_info": (ctypes.c_int, [vp, P(i64), P(i32), P(i32), P(i32), P(i32)]),
            "llvq_quantize": (ctypes.c_int, [vp, vp, i64, vp, vp, vp, vp]),
            "llvq_quantize_ex": (ctypes.c_int, [vp, vp, i64, vp, vp, vp, ctypes.c_uint32, vp]),
            "llvq_quantize_gain": (ctypes.c_int, [vp, vp, i64, vp, vp, vp, vp, i32, vp, i64, vp, ctypes.c_uint32,
                                                  vp]),
            "llvq_dequantize_lattice": (ctypes.c_int, [vp, vp, i64, vp, vp, vp]),
            "llvq_dequantize": (ctypes.c_int, [vp, vp, i64, vp, i32, vp, vp]),
            "llvq_dequantize_bf16": (ctypes.c_int, [vp, vp, i64, vp, i64, vp, vp, vp]),
            "llvq_gemm": (ctypes.c_int, [vp, vp, i64, i64, vp, vp, i64, i64, vp, vp, vp]),
            "llvq_gemm_noalloc": (ctypes.c_int, [vp, vp, i64, i64, vp, vp, i64, i64, vp, vp, vp]),
            "llvq_hadamard": (ctypes.c_int, [vp, i32, vp, i64, i64, i32, vp, i32, vp]),
            "llvq_hadamard_ex": (ctypes.c_int, [vp, i32, vp, i32, i64, i64, i32, vp, i32, vp]),
            "llvq_rotate_scale": (ctypes.c_int, [vp, i64, i64, i64, i32, vp, vp, vp, vp]),
            "llvq_pack_indices": (ctypes.c_int, [vp, i64, i32, vp, vp, vp]),
            "llvq_unpack_indices": (ctypes.c_int, [vp, i64, i32, vp, vp]),
            "llvq_dequantize_packed": (ctypes.c_int, [vp, vp, i32, i64, vp, i32, vp, i64, vp, vp]),
            "llvq_gemm_packed": (ctypes.c_int, [vp, vp, i32, i64, i64, vp, vp, i64, i64, vp, vp, vp]),
            "llvq_codeword_host": (ctypes.c_int, [vp, i64, vp]),
            "llvq_codeword_batch_host": (ctypes.c_int, [vp, vp, i64, vp, P(i64)]),
            "llvq_codebook_tables": (ctypes.c_int, [vp, P(i32), P(i64), P(i32)]),
            "llvq_encode_host": (ctypes.c_int, [vp, vp, P(i64)]),
            "llvq_status_string": (ctypes.c_char_p, [ctypes.c_int]),
            "llvq_last_error": (ctypes.c_char_p, []),
            "llvq_version": (ctypes.c_int, []),
        }
        for name, (res, args) in sig.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        _lib = lib
        return lib


def as_int64(index: int) -> int:
    """The int64 image of an unsigned 64-bit index (negative from 2^63 on)."""
    i = int(index) & ((1 << 64) - 1)
    return i - (1 << 64) if i >> 63 else i


def check(status: int, what: str) -> None:
    """Raise the exception type the reference raises for this failure."""
    if status == OK:
        return
    lib = load()
    msg = f"{what}: {lib.llvq_status_string(status).decode()}: {lib.llvq_last_error().decode()}"
    if status == ERR_INDEX_RANGE:
        raise IndexError(msg)
    if status in (ERR_INVALID_ARGUMENT, ERR_NOT_A_CODEWORD, ERR_UNSUPPORTED):
        raise ValueError(msg)
    if status == ERR_OUT_OF_MEMORY:
        raise MemoryError(msg)
    raise RuntimeError(msg)


class NativeCodebook:
    """Owner of one llvq_codebook handle (tables on one device, or host-only
    when device < 0)."""

    def __init__(self, shells: Sequence[int], parities: Sequence[int], leaders: Sequence[Sequence[int]],
                 device: int = -1):
        lib = load()
        n = len(shells)
        sh = np.ascontiguousarray(shells, dtype=np.int32)
        pa = np.ascontiguousarray(parities, dtype=np.int32)
        le = np.ascontiguousarray(leaders, dtype=np.int32).reshape(n, 24)
        h = ctypes.c_void_p()
        check(lib.llvq_codebook_create(n, sh.ctypes.data, pa.ctypes.data, le.ctypes.data, int(device),
                                       ctypes.byref(h)), "llvq_codebook_create")
        self._lib = lib
        self.handle = h.value
        self.device = int(device)
        total, ncls, lo, hi, spec = ctypes.c_int64(), ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32(), \
            ctypes.c_int32()
        check(lib.llvq_codebook_info(self.handle, ctypes.byref(total), ctypes.byref(ncls), ctypes.byref(lo),
                                     ctypes.byref(hi), ctypes.byref(spec)), "llvq_codebook_info")
        self.total_count = total.value & ((1 << 64) - 1)  # unsigned: codebooks past 2^63 use the full range
        self.n_classes = ncls.value
        self.min_shell = lo.value
        self.max_shell = hi.value
        self.specialized = bool(spec.value)

    def __del__(self):
        h = getattr(self, "handle", None)
        if h:
            try:
                self._lib.llvq_codebook_destroy(h)
            except Exception:  # interpreter teardown
                pass
            self.handle = None

    # ---- host paths (indices are unsigned 64-bit: Python ints in
    # [0, total_count); the int64 arguments carry their two's-complement image)
    def codeword(self, index: int) -> tuple[int, ...]:
        out = (ctypes.c_int32 * 24)()
        check(self._lib.llvq_codeword_host(self.handle, as_int64(index), out), "llvq_codeword_host")
        return tuple(out)

    def codeword_batch(self, indices) -> tuple[np.ndarray, int]:
        """Integer codewords [n, 24] of int64 indices on the host with the
        table-driven decoder the kernels use; (codewords, count out of range)."""
        idx = np.ascontiguousarray(indices, dtype=np.int64).reshape(-1)
        out = np.zeros((idx.shape[0], 24), dtype=np.int32)
        bad = ctypes.c_int64()
        check(self._lib.llvq_codeword_batch_host(self.handle, idx.ctypes.data, idx.shape[0], out.ctypes.data,
                                                 ctypes.byref(bad)), "llvq_codeword_batch_host")
        return out, bad.value

    def tables(self) -> dict:
        """Whether the decoder is table-driven, its table bytes and the most
        lookups one index takes."""
        tab, nbytes, jobs = ctypes.c_int32(), ctypes.c_int64(), ctypes.c_int32()
        check(self._lib.llvq_codebook_tables(self.handle, ctypes.byref(tab), ctypes.byref(nbytes),
                                             ctypes.byref(jobs)), "llvq_codebook_tables")
        return {"tabulated": bool(tab.value), "bytes": nbytes.value, "max_lookups": jobs.value}

    def encode(self, vector: Sequence[int]) -> int:
        v = (ctypes.c_int32 * 24)(*[int(a) for a in vector])
        idx = ctypes.c_int64()
        check(self._lib.llvq_encode_host(self.handle, v, ctypes.byref(idx)), "llvq_encode_host")
        return idx.value & ((1 << 64) - 1)

    # ---- device paths (raw pointers; the callers own allocation and streams)
    def quantize(self, x_ptr: int, n: int, idx_ptr: int, pair_ptr: int, score_ptr: int, stream: int,
                 flags: int = 0) -> None:
        check(self._lib.llvq_quantize_ex(self.handle, x_ptr, n, idx_ptr, pair_ptr, score_ptr, flags, stream),
              "llvq_quantize")

    def quantize_gain(self, x_ptr: int, n: int, idx_ptr: int, pair_ptr: int, score_ptr: int, thr_ptr: int,
                      gain_bits: int, sigma_ptr: int | None, blocks_per_row: int, gain_ptr: int | None, pack: bool,
                      stream: int, angular: bool = False) -> None:
        flags = (GAIN_PACK if pack else 0) | (GAIN_ANGULAR if angular else 0)
        check(self._lib.llvq_quantize_gain(self.handle, x_ptr, n, idx_ptr, pair_ptr, score_ptr, thr_ptr, gain_bits,
                                           sigma_ptr, blocks_per_row, gain_ptr, flags, stream),
              "llvq_quantize_gain")

    def dequantize_lattice(self, idx_ptr: int, n: int, out_ptr: int, err_ptr: int | None, stream: int) -> None:
        check(self._lib.llvq_dequantize_lattice(self.handle, idx_ptr, n, out_ptr, err_ptr, stream),
              "llvq_dequantize_lattice")

    def dequantize(self, idx_ptr: int, n: int, out_ptr: int, kind: int, err_ptr: int | None, stream: int) -> None:
        check(self._lib.llvq_dequantize(self.handle, idx_ptr, n, out_ptr, kind, err_ptr, stream), "llvq_dequantize")

    def gemm(self, idx_ptr: int, n_out: int, blocks_per_row: int, scale_ptr: int | None, a_ptr: int, m: int, k: int,
             y_ptr: int, err_ptr: int | None, stream: int) -> None:
        check(self._lib.llvq_gemm(self.handle, idx_ptr, n_out, blocks_per_row, scale_ptr, a_ptr, m, k, y_ptr, err_ptr,
                                  stream), "llvq_gemm")

    def gemm_noalloc(self, idx_ptr: int, n_out: int, blocks_per_row: int, scale_ptr: int | None, a_ptr: int, m: int,
                     k: int, y_ptr: int, err_ptr: int | None, stream: int) -> None:
        """llvq_gemm with a static 16 MiB staging array per device instead of a
        stream-ordered allocation (blocks_per_row <= 2730)."""
        check(self._lib.llvq_gemm_noalloc(self.handle, idx_ptr, n_out, blocks_per_row, scale_ptr, a_ptr, m, k, y_ptr,
                                          err_ptr, stream), "llvq_gemm_noalloc")

    def dequantize_packed(self, packed_ptr: int, index_bytes: int, n: int, out_ptr: int, kind: int,
                          scale_ptr: int | None, blocks_per_row: int, err_ptr: int | None, stream: int) -> None:
        check(self._lib.llvq_dequantize_packed(self.handle, packed_ptr, index_bytes, n, out_ptr, kind, scale_ptr,
                                               blocks_per_row, err_ptr, stream), "llvq_dequantize_packed")

    def gemm_packed(self, packed_ptr: int, index_bytes: int, n_out: int, blocks_per_row: int, scale_ptr: int | None,
                    a_ptr: int, m: int, k: int, y_ptr: int, err_ptr: int | None, stream: int) -> None:
        check(self._lib.llvq_gemm_packed(self.handle, packed_ptr, index_bytes, n_out, blocks_per_row, scale_ptr,
                                         a_ptr, m, k, y_ptr, err_ptr, stream), "llvq_gemm_packed")

    def dequantize_bf16(self, idx_ptr: int, n: int, scale_ptr: int, blocks_per_row: int, out_ptr: int,
                        err_ptr: int | None, stream: int) -> None:
        check(self._lib.llvq_dequantize_bf16(self.handle, idx_ptr, n, scale_ptr, blocks_per_row, out_ptr, err_ptr,
                                             stream), "llvq_dequantize_bf16")


def pack_indices(idx_ptr: int, n: int, index_bytes: int, out_ptr: int, err_ptr: int | None, stream: int) -> None:
    check(load().llvq_pack_indices(idx_ptr, n, index_bytes, out_ptr, err_ptr, stream), "llvq_pack_indices")


def unpack_indices(packed_ptr: int, n: int, index_bytes: int, out_ptr: int, stream: int) -> None:
    check(load().llvq_unpack_indices(packed_ptr, n, index_bytes, out_ptr, stream), "llvq_unpack_indices")


DT_F32, DT_F16, DT_BF16 = 0, 1, 2


def hadamard_ex(in_ptr: int, in_type: int, out_ptr: int, out_type: int, rows: int, cols: int, block: int,
                signs_ptr: int, inverse: bool, stream: int) -> None:
    check(load().llvq_hadamard_ex(in_ptr, in_type, out_ptr, out_type, rows, cols, block, signs_ptr, int(inverse),
                                  stream), "llvq_hadamard_ex")


def rotate_scale(in_ptr: int, rows: int, cols: int, ld: int, block: int, signs_ptr: int, out_ptr: int,
                 scale_ptr: int, stream: int) -> None:
    check(load().llvq_rotate_scale(in_ptr, rows, cols, ld, block, signs_ptr, out_ptr, scale_ptr, stream),
          "llvq_rotate_scale")


def hadamard(in_ptr: int, in_is_half: bool, out_ptr: int, rows: int, cols: int, block: int, signs_ptr: int,
             inverse: bool, stream: int) -> None:
    lib = load()
    check(lib.llvq_hadamard(in_ptr, int(in_is_half), out_ptr, rows, cols, block, signs_ptr, int(inverse), stream),
          "llvq_hadamard")


_CACHE: dict = {}


class MetadataBooks:
    """Codebooks of the reference's metadata dicts, for the launcher shims.

    The dicts hold device tensors; reading them back to build a content key
    would synchronise the host on every launch, which the reference's
    launchers never do.  An entry is therefore reused only while every
    tensor it was built from is the very same live object, unmodified
    (same ``_version``): a new dict whose tensors happen to reuse freed
    device memory at the same addresses gets its own codebook, and the
    codebook itself is shared by content through ``codebook_for``."""

    def __init__(self, keys: Sequence[str], classes_from_meta):
        self._keys = tuple(keys)
        self._classes = classes_from_meta
        self._entries: dict = {}
        self._mu = threading.Lock()

    def get(self, meta: dict, device: int) -> "NativeCodebook":
        import weakref

        tensors = [meta[k] for k in self._keys]
        key = (tuple(t.data_ptr() for t in tensors), int(device))
        with self._mu:
            hit = self._entries.get(key)
            if hit is not None:
                refs, versions, book = hit
                if all(r() is t for r, t in zip(refs, tensors)) and \
                        all(v == t._version for v, t in zip(versions, tensors)):
                    return book
        shell, parity, leaders = self._classes(meta)
        book = codebook_for(shell, parity, leaders, device)
        with self._mu:
            self._entries = {k: e for k, e in self._entries.items() if all(r() is not None for r in e[0])}
            self._entries[key] = ([weakref.ref(t) for t in tensors], [t._version for t in tensors], book)
        return book


def codebook_for(shells, parities, leaders, device: int) -> NativeCodebook:
    """Codebooks are cached per (class list, device): building one uploads
    its tables once."""
    key = (np.asarray(shells, dtype=np.int32).tobytes(), np.asarray(parities, dtype=np.int32).tobytes(),
           np.asarray(leaders, dtype=np.int32).tobytes(), int(device))
    cb = _CACHE.get(key)
    if cb is None:
        cb = NativeCodebook(shells, parities, leaders, device)
        _CACHE[key] = cb
    return cb
