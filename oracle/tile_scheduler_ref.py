"""Pure-Python restatement of the reference's tile scheduler -- TEST ORACLE ONLY.

Follows adelmuursepp/cutedsl_pingpong_gemm ``tile_scheduler.py``:

* ``RasterOrder``                tile_scheduler.py:24-27
* ``Params.create``              tile_scheduler.py:50-78
* ``get_grid_shape``             tile_scheduler.py:110-123
* ``create`` (start work id)     tile_scheduler.py:94-107
* ``_map_cta_coords``            tile_scheduler.py:125-146
* ``get_current_work``           tile_scheduler.py:148-166
* ``advance_to_next_work``       tile_scheduler.py:175-183

and the caller side in gemm_base.py: tile counts ``ceil(M/tile_m), ceil(N/tile_n)`` with the
fixed group size 8 (gemm_base.py:65, :464-478).

The device intrinsics the reference reads (``cluster_idx``, ``cluster_dim`` = number of
clusters in the grid, ``block_idx``, ``block_in_cluster_idx``, ``grid_dim``) are restated as
explicit loops over the launch grid in ``schedule``.  ``_map_cta_coords`` and the Params are
pinned bit-exact against ``tests/golden/tile_maps.{json,npz}``, which were produced by running
the reference's own code.
"""
from dataclasses import dataclass
from typing import List, Tuple

from .fast_math_ref import FastDivmod

ALONG_M = 0
ALONG_N = 1


def ceil_div(a: int, b: int) -> int:
    return -(-a // b)


@dataclass
class Params:
    ncluster_mnl: Tuple[int, int, int]
    raster_order: int
    dm_clusters_per_problem: FastDivmod
    num_groups_regular: int
    dm_group_size: FastDivmod
    dm_group_size_tail: FastDivmod
    dm_num_clusters_in_group: FastDivmod
    cluster_shape_mn: Tuple[int, int]
    is_persistent: bool


def params_create(ntiles_mnl, raster_order, group_size, cluster_shape_mnk, is_persistent) -> Params:
    """tile_scheduler.py:50-78."""
    assert cluster_shape_mnk[2] == 1
    cm, cn = cluster_shape_mnk[0], cluster_shape_mnk[1]
    ncm, ncn = ceil_div(ntiles_mnl[0], cm), ceil_div(ntiles_mnl[1], cn)
    ncluster_mnl = (ncm, ncn, ntiles_mnl[2])
    clusters_per_problem = ncm * ncn
    fast = ncm if raster_order == ALONG_M else ncn
    slow = ncn if raster_order == ALONG_M else ncm
    g = min(group_size, fast)
    tail = fast % g
    nreg = fast // g
    nig = g * slow
    return Params(ncluster_mnl, raster_order, FastDivmod.create(clusters_per_problem), nreg,
                  FastDivmod.create(g), FastDivmod.create(tail if tail > 0 else 1),
                  FastDivmod.create(nig), (cm, cn), is_persistent)


def get_grid_shape(p: Params, max_active_clusters: int) -> Tuple[int, int, int]:
    """tile_scheduler.py:110-123."""
    cm, cn = p.cluster_shape_mn
    num_ctas = (p.ncluster_mnl[0] * cm, p.ncluster_mnl[1] * cn, p.ncluster_mnl[2])
    if not p.is_persistent:
        return num_ctas
    in_problem = num_ctas[0] * num_ctas[1] * num_ctas[2]
    in_cluster = cm * cn
    per_wave = max_active_clusters * in_cluster
    persistent_ctas = min(in_problem, per_wave)
    return (cm, cn, persistent_ctas // in_cluster)


def map_cta_coords(p: Params, cluster_id: int) -> Tuple[int, int]:
    """tile_scheduler.py:125-146: linear cluster id -> (cluster_m, cluster_n)."""
    group_id, id_in_group = p.dm_num_clusters_in_group.divmod(cluster_id)
    if group_id < p.num_groups_regular:
        slow, fast_in_group = p.dm_group_size.divmod(id_in_group)
    else:
        slow, fast_in_group = p.dm_group_size_tail.divmod(id_in_group)
    if group_id % 2 == 1:
        nslow = p.ncluster_mnl[1] if p.raster_order == ALONG_M else p.ncluster_mnl[0]
        slow = nslow - 1 - slow
    fast = group_id * p.dm_group_size.divisor + fast_in_group
    if p.raster_order == ALONG_N:
        return slow, fast
    return fast, slow


def cluster_map(p: Params) -> List[Tuple[int, int]]:
    """_map_cta_coords for every cluster id of the problem (batch ignored, as the reference)."""
    return [map_cta_coords(p, c) for c in range(p.ncluster_mnl[0] * p.ncluster_mnl[1])]


def schedule(p: Params, grid: Tuple[int, int, int]):
    """Per-CTA tile sequence the reference's kernel walks for a launch of ``grid``.

    Returns ``{(bx, by, bz): [(pid_m, pid_n), ...]}``.  Restates create / get_current_work /
    advance_to_next_work (tile_scheduler.py:94-107, :148-166, :175-183): persistent CTAs
    start at cluster id ``blockIdx.z`` and stride by ``gridDim.z`` while the id is below the
    cluster count; non-persistent clusters do exactly one tile, the one at linear cluster id
    ``clusterid.x + clusterid.y * nclusterid.x``.  ``pid = cid * cluster_shape +
    block_in_cluster``.
    """
    cm, cn = p.cluster_shape_mn
    total = p.ncluster_mnl[0] * p.ncluster_mnl[1] * p.ncluster_mnl[2]
    out = {}
    for bz in range(grid[2]):
        for by in range(grid[1]):
            for bx in range(grid[0]):
                bic = (bx % cm, by % cn)
                if p.is_persistent:
                    cid = bz
                else:
                    nclx = grid[0] // cm
                    cid = (bx // cm) + (by // cn) * nclx
                seq = []
                first = True
                while (p.is_persistent and cid < total) or (not p.is_persistent and first):
                    m, n = map_cta_coords(p, cid)
                    seq.append((m * cm + bic[0], n * cn + bic[1]))
                    first = False
                    if p.is_persistent:
                        cid += grid[2]
                out[(bx, by, bz)] = seq
    return out
