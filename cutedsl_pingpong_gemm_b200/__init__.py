"""B200-native (sm_100a) GEMM with the Python surface of the CuTe-DSL "pingpong" GEMM.

Public modules mirror the reference's files:

* ``gemm_base``      -- ``GemmSM90`` (alias ``GemmSM100``) and ``compile``
* ``tile_scheduler`` -- ``RasterOrder``, ``SimpleTileSchedulerArguments``, ``SimpleTileScheduler``,
                        ``get_max_active_clusters``
* ``fast_math``      -- ``FastDivmod``

All compute runs in ``libcpgemm.so`` (hand-written CUDA for sm_100a, C ABI in
``include/cpgemm.h``).
"""
from . import _lib
from ._lib import CpgError
from .fast_math import FastDivmod
from .gemm_base import CompiledGemm, GemmSM90, GemmSM100, compile
from .tile_scheduler import (RasterOrder, SimpleTileScheduler, SimpleTileSchedulerArguments,
                             get_max_active_clusters)

__all__ = [
    "CpgError", "FastDivmod", "CompiledGemm", "GemmSM90", "GemmSM100", "compile", "RasterOrder",
    "SimpleTileScheduler", "SimpleTileSchedulerArguments", "get_max_active_clusters",
]


def library_path() -> str:
    return _lib.lib_path()
