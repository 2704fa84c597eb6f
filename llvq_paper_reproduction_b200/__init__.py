"""B200 (sm_100a) Leech-lattice (Λ24) vector quantizer: a drop-in for the
GPU quantizer API of dmnunez1993/llvq-paper-reproduction.

The compute path is the in-tree CUDA library (``_lib/libllvq_b200.so``, C ABI
in ``include/llvq_b200.h``); it is loaded lazily and its absence is an error,
never a fallback.
"""
from .tables import (DIM, LATTICE_SCALE, ClassLeader, ClassLocalStructure, LocalDecomposition, RankedCodeword,
                     build_local_structure, compare_with_reference, extended_golay_codewords,
                     generate_class_leaders, leech_shell_counts)


def __getattr__(name):
    if name == "LeechLatticeVectorQuantizerGpu":
        from .quantizer import LeechLatticeVectorQuantizerGpu
        return LeechLatticeVectorQuantizerGpu
    raise AttributeError(name)


__all__ = ["DIM", "LATTICE_SCALE", "ClassLeader", "ClassLocalStructure", "LocalDecomposition", "RankedCodeword",
           "LeechLatticeVectorQuantizerGpu", "build_local_structure", "compare_with_reference",
           "extended_golay_codewords", "generate_class_leaders", "leech_shell_counts"]
