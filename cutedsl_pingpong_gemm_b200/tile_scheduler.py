"""Tile scheduler with the interface of the reference's ``tile_scheduler.py``.

Same names and meaning as the reference: ``RasterOrder`` (tile_scheduler.py:24-27),
``SimpleTileSchedulerArguments`` (:29-35), ``SimpleTileScheduler.Params`` / ``to_underlying_arguments``
(:38-78, :89-91), ``get_grid_shape`` (:110-123), ``_map_cta_coords`` (:125-146) and
``get_max_active_clusters`` (:20-22).  The computation lives in the shared C++ header
``csrc/tile_scheduler.h``, which the GEMM kernels execute on the device; this module reaches it
through the C ABI.  ``cluster_map_device`` runs the device copy for verification, and
``schedule`` lists the per-CTA tile sequence the persistent kernel walks.
"""
import ctypes
from dataclasses import dataclass
from enum import IntEnum
from functools import lru_cache
from typing import Dict, List, Tuple

import numpy as np

from . import _lib
from .fast_math import FastDivmod


class RasterOrder(IntEnum):
    """Set M/N as fast dimension (tile_scheduler.py:24-27)."""
    AlongM = 0
    AlongN = 1


@lru_cache
def get_max_active_clusters(cluster_size: int) -> int:
    """Clusters of ``cluster_size`` CTAs of the GEMM kernel resident at once on the current GPU."""
    lib = _lib.load()
    out = ctypes.c_int32()
    _lib.check(lib.cpg_max_active_clusters(int(cluster_size), ctypes.byref(out)),
               "get_max_active_clusters")
    return out.value


@dataclass
class SimpleTileSchedulerArguments:
    """tile_scheduler.py:29-35."""
    ntiles_mnl: Tuple[int, int, int]
    raster_order: RasterOrder
    group_size: int
    cluster_shape_mnk: Tuple[int, int, int]
    is_persistent: bool


def _fdm(c: "_lib.FastDivmodC") -> FastDivmod:
    return FastDivmod(c.divisor, c.multiplier, c.shift_right)


class SimpleTileScheduler:
    @dataclass
    class Params:
        """tile_scheduler.py:38-48 (plus the raw C struct used by the kernels)."""
        ncluster_mnl: Tuple[int, int, int]
        raster_order: RasterOrder
        dm_clusters_per_problem: FastDivmod
        num_groups_regular: int
        dm_group_size: FastDivmod
        dm_group_size_tail: FastDivmod
        dm_num_clusters_in_group: FastDivmod
        cluster_shape_mn: Tuple[int, int]
        is_persistent: bool
        c_struct: object = None

        @staticmethod
        def create(args: SimpleTileSchedulerArguments) -> "SimpleTileScheduler.Params":
            lib = _lib.load()
            c = _lib.SchedParamsC()
            ntm, ntn, ntl = (int(x) for x in args.ntiles_mnl)
            cm, cn, ck = (int(x) for x in args.cluster_shape_mnk)
            _lib.check(lib.cpg_sched_params_create(ntm, ntn, ntl, int(args.raster_order),
                                                   int(args.group_size), cm, cn, ck,
                                                   int(bool(args.is_persistent)), ctypes.byref(c)),
                       "SimpleTileScheduler.Params.create")
            return SimpleTileScheduler.Params.from_c(c)

        @staticmethod
        def from_c(c: "_lib.SchedParamsC") -> "SimpleTileScheduler.Params":
            return SimpleTileScheduler.Params(
                (c.ncluster_m, c.ncluster_n, c.ncluster_l), RasterOrder(c.raster_order),
                _fdm(c.dm_clusters_per_problem), c.num_groups_regular, _fdm(c.dm_group_size),
                _fdm(c.dm_group_size_tail), _fdm(c.dm_num_clusters_in_group),
                (c.cluster_m, c.cluster_n), bool(c.is_persistent), c)

    @staticmethod
    def to_underlying_arguments(args: SimpleTileSchedulerArguments) -> "SimpleTileScheduler.Params":
        """tile_scheduler.py:89-91."""
        return SimpleTileScheduler.Params.create(args)

    @staticmethod
    def get_grid_shape(params: "SimpleTileScheduler.Params", max_active_clusters: int) -> Tuple[int, int, int]:
        """tile_scheduler.py:110-123."""
        lib = _lib.load()
        grid = (ctypes.c_int32 * 3)()
        _lib.check(lib.cpg_sched_grid_shape(ctypes.byref(params.c_struct), int(max_active_clusters),
                                            grid), "get_grid_shape")
        return (grid[0], grid[1], grid[2])

    @staticmethod
    def num_clusters(params: "SimpleTileScheduler.Params") -> int:
        return params.ncluster_mnl[0] * params.ncluster_mnl[1]

    @staticmethod
    def _map_cta_coords(params: "SimpleTileScheduler.Params", cluster_id_in_problem: int) -> Tuple[int, int]:
        """tile_scheduler.py:125-146 for one linear cluster id, in O(1): the group and the
        position in it come from the params' FastDivmods (the kernels' host/device arithmetic),
        every second group runs its slow coordinate backwards."""
        group_id, id_in_group = params.dm_num_clusters_in_group.divmod(int(cluster_id_in_problem))
        dm = params.dm_group_size if group_id < params.num_groups_regular else params.dm_group_size_tail
        slow, fast_in_group = dm.divmod(id_in_group)
        if group_id % 2 == 1:
            nslow = params.ncluster_mnl[1] if params.raster_order == RasterOrder.AlongM else params.ncluster_mnl[0]
            slow = nslow - 1 - slow
        fast = group_id * params.dm_group_size.divisor + fast_in_group
        return (slow, fast) if params.raster_order == RasterOrder.AlongN else (fast, slow)

    @staticmethod
    def cluster_map(params: "SimpleTileScheduler.Params", n: int = None) -> np.ndarray:
        """(n, 2) int32 array: cluster (m, n) of linear cluster ids 0..n-1 (host C++)."""
        n = SimpleTileScheduler.num_clusters(params) if n is None else int(n)
        out = np.zeros((n, 2), dtype=np.int32)
        lib = _lib.load()
        _lib.check(lib.cpg_sched_cluster_map(ctypes.byref(params.c_struct),
                                             out.ctypes.data_as(ctypes.POINTER(ctypes.c_int32)), n),
                   "cluster_map")
        return out

    @staticmethod
    def cluster_map_device(params: "SimpleTileScheduler.Params", n: int = None, device=None):
        """Same map computed on the GPU by the kernels' scheduler code; returns a CUDA tensor."""
        import torch
        n = SimpleTileScheduler.num_clusters(params) if n is None else int(n)
        dev = torch.device("cuda", torch.cuda.current_device() if device is None else device)
        out = torch.zeros((n, 2), dtype=torch.int32, device=dev)
        lib = _lib.load()
        stream = torch.cuda.current_stream(dev).cuda_stream
        _lib.check(lib.cpg_sched_cluster_map_device(ctypes.byref(params.c_struct), out.data_ptr(), n,
                                                    stream), "cluster_map_device")
        return out

    @staticmethod
    def schedule(params: "SimpleTileScheduler.Params", grid: Tuple[int, int, int]) -> Dict[Tuple[int, int, int], List[Tuple[int, ...]]]:
        """Per-CTA tile sequence for a launch of ``grid`` (tile_scheduler.py:94-183).

        With one batch (L = 1) the entries are ``(pid_m, pid_n)``, exactly the reference's
        schedule.  With L > 1 they are ``(pid_m, pid_n, l)``: a persistent CTA's linear cluster
        id is first split into (batch l, id within the problem) with ``dm_clusters_per_problem``,
        as the sm_100a kernels do (the reference fixes the batch at 0, tile_scheduler.py:96, and
        so never runs past one problem); a non-persistent CTA's batch is ``blockIdx.z``."""
        cmap = SimpleTileScheduler.cluster_map(params)
        cm, cn = params.cluster_shape_mn
        per_problem = params.ncluster_mnl[0] * params.ncluster_mnl[1]
        nl = params.ncluster_mnl[2]
        total = per_problem * nl
        out = {}
        for bz in range(grid[2]):
            for by in range(grid[1]):
                for bx in range(grid[0]):
                    if params.is_persistent:
                        work = [divmod(c, per_problem) for c in range(bz, total, grid[2])]
                    else:
                        work = [(bz, (bx // cm) + (by // cn) * (grid[0] // cm))]
                    tiles = []
                    for l, c in work:
                        t = (int(cmap[c, 0]) * cm + bx % cm, int(cmap[c, 1]) * cn + by % cn)
                        tiles.append(t if nl == 1 else t + (l,))
                    out[(bx, by, bz)] = tiles
        return out
