"""Drop-in replacement of LeechLatticeVectorQuantizerGpu
(impl/leech_lattice_vector_quantizer_gpu.py:145-567 of
dmnunez1993/llvq-paper-reproduction).

Same constructor, attributes and methods; tensor quantize/dequantize run the
sm_100a kernels of the in-tree CUDA library on torch's current stream.  There
is no CPU fallback: tensor paths on a non-CUDA device raise ValueError, as the
reference does.  Scalar host paths (codeword, unrank, encode_codeword) run the
library's host code.
"""
from __future__ import annotations

from bisect import bisect_right
from math import ceil, log2
from pathlib import Path
from typing import Sequence

import torch

from . import _native
from .tables import (DIM, LATTICE_SCALE, ClassLeader, ClassLocalStructure, LocalDecomposition, RankedCodeword,
                     build_local_structure, extended_golay_codewords, generate_class_leaders, leech_shell_counts)


class LeechLatticeVectorQuantizerGpu:
    """Implicit shell -> class -> local-symmetry database for Leech codewords,
    with the quantizer and dequantizer on the GPU."""

    def __init__(self, max_shell: int = 4, leaders: Sequence[ClassLeader] | None = None,
                 cache_dir: str | Path | None = ".llvq_cache", use_cache: bool = True, verbose: bool = False,
                 device: str | torch.device | None = None, dtype: torch.dtype = torch.float32,
                 min_shell: int = 2):
        if max_shell < 2:
            raise ValueError("max_shell must be at least 2")
        if min_shell < 2 or min_shell > max_shell:
            raise ValueError("min_shell must be in 2..max_shell")
        self.device = torch.device(device or ("cuda" if torch.cuda.is_available() else "cpu"))
        self.dtype = dtype
        if leaders is None:
            leaders = generate_class_leaders(max_shell, cache_dir=cache_dir, use_cache=use_cache, verbose=verbose,
                                             min_shell=min_shell)
        shells = {row.shell for row in leaders}
        missing = [m for m in range(min_shell, max_shell + 1) if m not in shells]
        if missing:
            raise ValueError(f"no class leaders are available for shells: {missing}")
        self.min_shell = min_shell
        self.max_shell = max_shell
        self.golay_codewords = extended_golay_codewords()
        self.golay_index_by_codeword = {c: i for i, c in enumerate(self.golay_codewords)}
        key = lambda r: (r.leader, 0 if r.parity == "even" else 1, r.count)  # noqa: E731
        self.classes_by_shell = {
            s: tuple(sorted((r for r in leaders if r.shell == s), key=key)) for s in range(min_shell, max_shell + 1)
        }
        self.shell_offsets = {}
        self.class_offsets = {}
        cursor = 0
        for s, rows in self.classes_by_shell.items():
            self.shell_offsets[s] = cursor
            offs, c = [], 0
            for r in rows:
                offs.append(c)
                c += r.count
            self.class_offsets[s] = tuple(offs)
            cursor += c
        self.local_structures = {
            s: tuple(build_local_structure(s, i, r, self.golay_codewords) for i, r in enumerate(rows))
            for s, rows in self.classes_by_shell.items()
        }
        self.class_index_by_shell_and_key = {
            s: {(r.leader, r.parity): i for i, r in enumerate(rows)} for s, rows in self.classes_by_shell.items()
        }
        self.shell_counts = {s: sum(r.count for r in rows) for s, rows in self.classes_by_shell.items()}
        self.cumulative_shell_counts = {s: self.shell_offsets[s] + self.shell_counts[s] for s in self.classes_by_shell}
        self.total_count = self.cumulative_shell_counts[max_shell]
        self.shape_bits = ceil(log2(self.total_count)) if self.total_count > 1 else 1
        self._validate()
        flat = [st for s in self.classes_by_shell for st in self.local_structures[s]]
        self._class_shell = [st.shell for st in flat]
        self._class_parity = [0 if st.leader.parity == "even" else 1 for st in flat]
        self._class_leader = [st.leader.leader for st in flat]
        self._host_book = None
        self._device_book = None

    # ------------------------------------------------------------ native books
    def _host(self) -> _native.NativeCodebook:
        if self._host_book is None:
            self._host_book = _native.codebook_for(self._class_shell, self._class_parity, self._class_leader, -1)
        return self._host_book

    def _book(self) -> _native.NativeCodebook:
        if self._device_book is None:
            index = self.device.index if self.device.index is not None else torch.cuda.current_device()
            self._device_book = _native.codebook_for(self._class_shell, self._class_parity, self._class_leader,
                                                     index)
            if self._device_book.total_count != self.total_count:
                raise RuntimeError("native codebook disagrees with the host tables")
        return self._device_book

    @property
    def specialized(self) -> bool:
        """True when generated search code exists for this class list."""
        return self._host().specialized

    # ------------------------------------------------------------ host API
    def rank_class(self, shell: int, class_index: int, class_local_index: int = 0) -> int:
        classes = self.classes_by_shell[shell]
        if class_index < 0 or class_index >= len(classes):
            raise IndexError(class_index)
        if class_local_index < 0 or class_local_index >= classes[class_index].count:
            raise IndexError(class_local_index)
        return self.shell_offsets[shell] + self.class_offsets[shell][class_index] + class_local_index

    def shell_for_index(self, global_index: int) -> int:
        ends = [self.cumulative_shell_counts[s] for s in self.classes_by_shell]
        return self.min_shell + bisect_right(ends, global_index)

    def unrank(self, global_index: int) -> RankedCodeword:
        if global_index < 0 or global_index >= self.total_count:
            raise IndexError(global_index)
        shell = self.shell_for_index(global_index)
        local = global_index - self.shell_offsets[shell]
        offs = self.class_offsets[shell]
        ci = bisect_right(offs, local) - 1
        return RankedCodeword(global_index, shell, local, ci, local - offs[ci], offs[ci],
                              self.classes_by_shell[shell][ci])

    def decompose_local_index(self, ranked: RankedCodeword) -> LocalDecomposition:
        st = self.local_structures[ranked.shell][ranked.class_index]
        cur = ranked.class_local_index
        perm = cur % st.permutation_count
        cur //= st.permutation_count
        sign = cur % st.sign_count
        golay = cur // st.sign_count
        return LocalDecomposition(golay, self.golay_codewords[st.golay_codeword_indices[golay]], sign, perm)

    def codeword(self, global_index: int) -> tuple[int, ...]:
        if global_index < 0 or global_index >= self.total_count:
            raise IndexError(global_index)
        return self._host().codeword(int(global_index))

    def encode_codeword(self, vector: Sequence[int]) -> int:
        """Exact index of a codeword of this database (CPU module :247-280)."""
        values = tuple(int(v) for v in vector)
        if len(values) != DIM:
            raise ValueError(f"expected {DIM} coordinates, got {len(values)}")
        return self._host().encode(values)

    # ------------------------------------------------------------ dequantize
    def dequantize_lattice(self, global_index):
        """Integer Leech representative(s) before the 1/sqrt(8) scale."""
        if not torch.is_tensor(global_index) and isinstance(global_index, int):
            return self.codeword(global_index)
        indices = torch.as_tensor(global_index, dtype=torch.long, device=self.device)
        shape = indices.shape
        return self._dequantize_lattice_cuda(indices.reshape(-1)).reshape(*shape, DIM)

    dequantize_lattice_cuda = dequantize_lattice

    def dequantize(self, global_index):
        """Scaled Leech lattice vector(s): fp32(1/sqrt 8) * k in the API dtype."""
        if not torch.is_tensor(global_index) and isinstance(global_index, int):
            return tuple(LATTICE_SCALE * v for v in self.codeword(global_index))
        indices = torch.as_tensor(global_index, dtype=torch.long, device=self.device)
        shape = indices.shape
        flat = indices.reshape(-1).contiguous()
        if self.dtype != torch.float32:
            return LATTICE_SCALE * self._dequantize_lattice_cuda(flat).reshape(*shape, DIM).to(self.dtype)
        self._require_cuda("dequantize")
        out = torch.empty((flat.shape[0], DIM), dtype=torch.float32, device=self.device)
        err = self._error_counter()
        with torch.cuda.device(self.device):
            self._book().dequantize(flat.data_ptr(), flat.shape[0], out.data_ptr(), _native.OUT_F32, err.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream)
        self._raise_if_bad(err)
        return out.reshape(*shape, DIM)

    # ---------------------------------------------------------- packed indices
    @property
    def index_bytes(self) -> int:
        """Bytes per packed index: the smallest count whose all-ones value
        (the invalid-index marker) lies above every index (6 at shells 2..13)."""
        return max(1, (self.total_count.bit_length() + 7) // 8)

    def pack_indices(self, indices: torch.Tensor, check: bool = False) -> torch.Tensor:
        """int64 indices [...] -> uint8 [..., index_bytes] little-endian; -1
        (a NaN/Inf row) becomes all-ones.  An index that does not fit is
        stored as all-ones and counted in the pending error flags (see
        ``raise_pending_errors``); ``check=True`` synchronises and raises
        IndexError at once.  No reference counterpart."""
        self._require_cuda("pack_indices")
        idx = indices.to(device=self.device, dtype=torch.long).contiguous()
        b = self.index_bytes
        out = torch.empty((*idx.shape, b), dtype=torch.uint8, device=self.device)
        flags = self._flags()
        with torch.cuda.device(self.device):
            _native.pack_indices(idx.data_ptr(), idx.numel(), b, out.data_ptr(), flags[self.FLAG_RANGE].data_ptr(),
                                 torch.cuda.current_stream().cuda_stream)
        if check:
            self.raise_pending_errors()
        return out

    def unpack_indices(self, packed: torch.Tensor) -> torch.Tensor:
        """uint8 [..., index_bytes] -> int64 [...] (all-ones -> -1)."""
        self._require_cuda("unpack_indices")
        pk = self._packed(packed)
        out = torch.empty(pk.shape[:-1], dtype=torch.long, device=self.device)
        with torch.cuda.device(self.device):
            _native.unpack_indices(pk.data_ptr(), out.numel(), self.index_bytes, out.data_ptr(),
                                   torch.cuda.current_stream().cuda_stream)
        return out

    def _packed(self, packed: torch.Tensor) -> torch.Tensor:
        if packed.dtype != torch.uint8 or packed.dim() < 1 or packed.shape[-1] != self.index_bytes:
            raise ValueError(f"packed indices must be uint8 [..., {self.index_bytes}]")
        return packed.to(self.device).contiguous()

    def dequantize_bf16(self, indices: torch.Tensor, row_scale: torch.Tensor, check: bool = False) -> torch.Tensor:
        """bf16 weights: bf16(dequantize(indices) * row_scale[row]) for indices
        [rows, blocks_per_row] (int64, or packed uint8 [rows, blocks_per_row,
        index_bytes]) and fp16 row_scale [rows] (no reference counterpart).
        Asynchronous: an out-of-range index gives a zero block and is counted
        in the pending error flags (``raise_pending_errors``); ``check=True``
        synchronises and raises IndexError at once."""
        self._require_cuda("dequantize_bf16")
        packed = indices.dtype == torch.uint8
        rows_blocks = indices.shape[:-1] if packed else indices.shape
        if len(rows_blocks) != 2 or row_scale.shape != (rows_blocks[0],) or row_scale.dtype != torch.float16:
            raise ValueError("expected indices [rows, blocks] and fp16 row_scale [rows]")
        rows, bpr = rows_blocks
        sc = row_scale.to(self.device).contiguous()
        out = torch.empty((rows, bpr * DIM), dtype=torch.bfloat16, device=self.device)
        err = self._flags()[self.FLAG_RANGE]
        stream = torch.cuda.current_stream(self.device).cuda_stream
        with torch.cuda.device(self.device):
            if packed:
                pk = self._packed(indices)
                self._book().dequantize_packed(pk.data_ptr(), self.index_bytes, rows * bpr, out.data_ptr(),
                                               _native.OUT_BF16_ROWSCALE, sc.data_ptr(), bpr, err.data_ptr(), stream)
            else:
                idx = indices.to(device=self.device, dtype=torch.long).contiguous()
                self._book().dequantize_bf16(idx.data_ptr(), idx.numel(), sc.data_ptr(), bpr, out.data_ptr(),
                                             err.data_ptr(), stream)
        if check:
            self.raise_pending_errors()
        return out

    def gemm(self, a: torch.Tensor, indices: torch.Tensor, row_scale: torch.Tensor | None = None,
             rotation: tuple[int, torch.Tensor] | None = None, check: bool = False) -> torch.Tensor:
        """Dequant-GEMM: ``a @ W.T`` in fp32 for bf16 activations ``a`` [m, k]
        and a weight given by its indices [n, blocks] (int64, or packed uint8
        [n, blocks, index_bytes]; W[n] = dequantize(indices[n]).flatten()[:k]
        * row_scale[n]).  For m <= 4 one kernel decodes each weight block in
        registers and multiplies it there (one warp per output row, a fixed
        reduction order); larger m decode into a bf16 staging buffer
        (stream-ordered, at most 256 MiB, chunk by chunk beyond that) that a
        pipelined tcgen05 GEMM reads.  ``rotation=(block, signs)`` first
        rotates the activations with the seeded Hadamard transform the weight
        was quantized under (int8 +-1 signs [k], block a power of two dividing
        k), rounding them to bf16 once: x W^T = (x R)(W R)^T.  The call is
        asynchronous on the current stream (no host synchronisation): a
        tensor-core wait that timed out sets the pending error flags
        (``raise_pending_errors``); ``check=True`` synchronises and raises
        RuntimeError at once.  No reference counterpart."""
        self._require_cuda("gemm")
        packed = indices.dtype == torch.uint8
        if a.dim() != 2 or indices.dim() != (3 if packed else 2):
            raise ValueError("expected a [m, k] and indices [n, blocks] (packed: [n, blocks, index_bytes])")
        m, k = a.shape
        n, bpr = indices.shape[:2]
        a16 = a.to(device=self.device, dtype=torch.bfloat16).contiguous()
        if rotation is not None:
            block, signs = rotation
            signs = signs.to(device=self.device, dtype=torch.int8).contiguous()
            if signs.shape != (k,):
                raise ValueError("rotation signs must have one entry per activation column")
            rot = torch.empty_like(a16)
            with torch.cuda.device(self.device):
                _native.hadamard_ex(a16.data_ptr(), _native.DT_BF16, rot.data_ptr(), _native.DT_BF16, m, k, int(block),
                                    signs.data_ptr(), False, torch.cuda.current_stream().cuda_stream)
            a16 = rot
        idx = self._packed(indices) if packed else indices.to(device=self.device, dtype=torch.long).contiguous()
        sc = None
        if row_scale is not None:
            if row_scale.shape != (n,):
                raise ValueError("row_scale must have one entry per weight row")
            sc = row_scale.to(device=self.device, dtype=torch.float16).contiguous()
        y = torch.empty((m, n), dtype=torch.float32, device=self.device)
        err = self._flags()[self.FLAG_GEMM]
        with torch.cuda.device(self.device):
            stream = torch.cuda.current_stream().cuda_stream
            sp = sc.data_ptr() if sc is not None else None
            if packed:
                self._book().gemm_packed(idx.data_ptr(), self.index_bytes, n, bpr, sp, a16.data_ptr(), m, k,
                                         y.data_ptr(), err.data_ptr(), stream)
            else:
                self._book().gemm(idx.data_ptr(), n, bpr, sp, a16.data_ptr(), m, k, y.data_ptr(), err.data_ptr(),
                                  stream)
        if check:
            self.raise_pending_errors()
        return y

    def _dequantize_lattice_cuda(self, indices: torch.Tensor) -> torch.Tensor:
        self._require_cuda("dequantize_lattice_cuda")
        flat = indices.contiguous()
        out = torch.empty((flat.shape[0], DIM), dtype=torch.long, device=self.device)
        err = self._error_counter()
        with torch.cuda.device(self.device):
            self._book().dequantize_lattice(flat.data_ptr(), flat.shape[0], out.data_ptr(), err.data_ptr(),
                                            torch.cuda.current_stream().cuda_stream)
        self._raise_if_bad(err)
        return out

    def _error_counter(self) -> torch.Tensor:
        return torch.zeros((1,), dtype=torch.int32, device=self.device)

    # Sticky device-side error flags of the asynchronous (non-reference)
    # paths: [0] indices outside the codebook or the packed width
    # (dequantize_bf16, pack_indices), [1] a timed-out tensor-core wait (gemm).
    FLAG_RANGE = 0
    FLAG_GEMM = 1

    def _flags(self) -> torch.Tensor:
        f = getattr(self, "_pending", None)
        if f is None:
            f = self._pending = torch.zeros((2,), dtype=torch.int32, device=self.device)
        return f

    def pending_errors(self) -> dict:
        """Counts recorded by the asynchronous paths since the last reset
        (synchronises the host with the device)."""
        v = self._flags().tolist()
        return {"index_range": int(v[self.FLAG_RANGE]), "gemm_timeout": int(v[self.FLAG_GEMM])}

    def raise_pending_errors(self) -> None:
        """Read and clear the pending error flags; raise IndexError for
        indices outside the codebook (or the packed width), RuntimeError for
        a timed-out dequant-GEMM."""
        errs = self.pending_errors()
        if errs["index_range"] or errs["gemm_timeout"]:
            self._flags().zero_()
        if errs["gemm_timeout"]:
            raise RuntimeError("tensor-core wait timed out in the dequant-GEMM")
        if errs["index_range"]:
            raise IndexError("global index outside codebook range (or the packed index width)")

    @staticmethod
    def _raise_if_bad(err: torch.Tensor) -> None:
        # Same host sync and exception as the reference's range check (_gpu.py:418-419).
        if int(err.item()):
            raise IndexError("global index outside codebook range")

    def _require_cuda(self, what: str) -> None:
        if self.device.type != "cuda":
            raise ValueError(f"{what} requires a CUDA device")

    # ------------------------------------------------------------ quantize
    def quantize(self, vector):
        """Quantize real-valued 24-D vector(s) on the GPU (tensor in, int64
        tensor out; a sequence input returns an int)."""
        return self.quantize_cuda(vector)

    # rows per chunk when a large batch comes from host memory
    HOST_CHUNK_ROWS = 1 << 20

    def quantize_cuda(self, vector, return_details: bool = False, table_driven: bool = False):
        self._require_cuda("quantize_cuda")
        tensor_input = torch.is_tensor(vector)
        if (tensor_input and vector.device.type == "cpu" and not return_details and not table_driven
                and vector.dim() >= 2 and vector.shape[-1] == DIM and vector.numel() // DIM > 2 * self.HOST_CHUNK_ROWS):
            return self._quantize_from_host(vector)
        x = torch.as_tensor(vector, dtype=self.dtype, device=self.device)
        if x.shape[-1] != DIM:
            raise ValueError(f"expected last dimension {DIM}, got {x.shape[-1]}")
        single = x.ndim == 1
        shape = x.shape[:-1]
        xs = x.reshape(-1, DIM).to(torch.float32).contiguous()
        n = xs.shape[0]
        indices = torch.empty((n,), dtype=torch.long, device=self.device)
        best_pair = torch.empty((n,), dtype=torch.long, device=self.device)
        best_score = torch.empty((n,), dtype=torch.float32, device=self.device)
        with torch.cuda.device(self.device):
            self._book().quantize(xs.data_ptr(), n, indices.data_ptr(), best_pair.data_ptr(), best_score.data_ptr(),
                                  torch.cuda.current_stream().cuda_stream,
                                  _native.FLAG_TABLE_DRIVEN if table_driven else 0)
        indices = indices.reshape(shape)
        if single:
            indices = indices.reshape(())
        if return_details:
            return indices, best_pair.reshape(shape), best_score.reshape(shape)
        if not tensor_input:
            return int(indices.item())
        return indices

    def _quantize_from_host(self, vector: torch.Tensor) -> torch.Tensor:
        """Large host batches: copy chunk i+1 to the device on a side stream
        while chunk i is quantized on the current stream (two device buffers,
        events in both directions), so the host->device copy hides behind the
        search.  Same indices as the single-copy path (rows are independent)."""
        shape = vector.shape[:-1]
        x = vector.reshape(-1, DIM)
        if x.dtype != torch.float32:
            x = x.to(torch.float32)
        x = x.contiguous()
        n, c = x.shape[0], self.HOST_CHUNK_ROWS
        indices = torch.empty((n,), dtype=torch.long, device=self.device)
        pair = torch.empty((c,), dtype=torch.long, device=self.device)
        score = torch.empty((c,), dtype=torch.float32, device=self.device)
        bufs = [torch.empty((c, DIM), dtype=torch.float32, device=self.device) for _ in range(2)]
        compute = torch.cuda.current_stream(self.device)
        copy = torch.cuda.Stream(device=self.device)
        copied = [torch.cuda.Event() for _ in range(2)]
        used = [None, None]
        book = self._book()
        # the buffers may be memory that earlier work on the current stream
        # still reads (the caching allocator recycles it in stream order)
        copy.wait_stream(compute)
        with torch.cuda.device(self.device):
            for i, r0 in enumerate(range(0, n, c)):
                rows, b = min(c, n - r0), i & 1
                with torch.cuda.stream(copy):
                    if used[b] is not None:
                        copy.wait_event(used[b])
                    bufs[b][:rows].copy_(x[r0: r0 + rows], non_blocking=True)
                    copied[b].record(copy)
                compute.wait_event(copied[b])
                book.quantize(bufs[b].data_ptr(), rows, indices[r0:].data_ptr(), pair.data_ptr(), score.data_ptr(),
                              compute.cuda_stream, 0)
                used[b] = torch.cuda.Event()
                used[b].record(compute)
        return indices.reshape(shape)

    # ------------------------------------------------------------ checks
    def _validate(self) -> None:
        theta = leech_shell_counts(self.max_shell)
        for shell, rows in self.classes_by_shell.items():
            if sum(r.count for r in rows) != theta[shell]:
                raise ValueError(f"shell {shell} leaders sum to {sum(r.count for r in rows)}, "
                                 f"theta series gives {theta[shell]}")
            for st in self.local_structures[shell]:
                if st.count != st.leader.count:
                    raise ValueError(f"shell {shell}, class {st.class_index} has local count {st.count}, "
                                     f"leader count {st.leader.count}")


__all__ = ["LeechLatticeVectorQuantizerGpu", "ClassLeader", "ClassLocalStructure", "LocalDecomposition",
           "RankedCodeword", "LATTICE_SCALE", "DIM"]
