"""Generate golden vectors by executing the reference's own scheduler and FastDivmod code.

This script is test infrastructure. It imports the reference implementation
(`fast_math.py`, `tile_scheduler.py` of adelmuursepp/cutedsl_pingpong_gemm) from a local
checkout and runs it on the host under the installed CuTe-DSL (nvidia-cutlass-dsl 4.5.0).
The outputs are committed next to this script so that the tests never need the reference:

* ``fast_divmod.json`` -- ``FastDivmod.create`` (fast_math.py:56-65) parameters for a set of
  divisors, and ``FastDivmod.divmod`` (fast_math.py:67-81) results on sampled dividends.
* ``tile_maps.npz`` / ``tile_maps.json`` -- ``SimpleTileScheduler.Params.create``
  (tile_scheduler.py:50-78), ``get_grid_shape`` (tile_scheduler.py:110-123) and the full
  cluster-id -> (cluster_m, cluster_n) map of ``_map_cta_coords`` (tile_scheduler.py:125-146)
  for every configuration listed in ``TILE_CONFIGS``.

The one substitution: ``fast_math.umulhi`` is inline PTX (``mul.hi.u32``, fast_math.py:34-47)
and cannot execute on a CPU, so it is replaced by its defining arithmetic
``(u64(a) * u64(b)) >> 32`` on unsigned 32-bit operands.  Everything else is the reference's
code as shipped.

Usage (needs the reference checkout and CuTe-DSL; not run by the tests)::

    PYTHONDONTWRITEBYTECODE=1 python tests/golden/gen_golden.py --reference <path-to-reference>
"""
import argparse
import hashlib
import json
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))

# (ntiles_m, ntiles_n, raster, cluster_m, cluster_n) -- raster 0 = AlongM, 1 = AlongN.
# Shapes come from the benchmark configurations (1024^3, 8192^3, the LLM FFN shape and its
# M-shards, FP8, small-M, tall-K) with 128x256 / 128x128 / 128x64 tiles, plus ragged shapes
# that exercise the group tail and the serpentine reversal.
TILE_CONFIGS = [
    (8, 4, 1, 2, 1),      # 1024^3, 128x256 tiles, cluster 2x1 (the parity config)
    (8, 4, 1, 1, 1),
    (8, 4, 0, 2, 1),
    (8, 8, 1, 1, 1),      # 1024^3, 128x128 tiles
    (64, 32, 1, 2, 1),    # 8192^3, 128x256 tiles
    (64, 32, 1, 1, 1),
    (64, 32, 0, 1, 1),
    (64, 32, 0, 2, 1),
    (64, 64, 1, 2, 1),    # 8192^3, 128x128 tiles
    (128, 112, 1, 2, 1),  # LLM FFN up 16384x28672, 128x256 tiles
    (128, 112, 1, 1, 1),
    (16, 112, 1, 2, 1),   # LLM shard M/8
    (32, 112, 1, 2, 1),   # LLM shard M/4
    (64, 112, 1, 2, 1),   # LLM shard M/2
    (128, 32, 1, 2, 1),   # FP8 16384x8192
    (128, 32, 1, 1, 1),
    (1, 32, 1, 1, 1),     # small M, 128x256
    (1, 64, 1, 1, 1),     # small M, 128x128
    (1, 128, 1, 1, 1),    # small M, 128x64
    (16, 8, 1, 2, 1),     # tall-K 2048x2048
    (16, 16, 1, 1, 1),
    (37, 53, 1, 1, 1),    # ragged
    (37, 53, 0, 1, 1),
    (37, 53, 1, 2, 1),
    (37, 53, 1, 1, 2),
    (37, 53, 0, 2, 2),
    (13, 7, 1, 1, 1),
    (13, 7, 0, 2, 1),
    (13, 7, 1, 2, 2),
    (1, 1, 1, 1, 1),
    (1, 1, 0, 2, 1),
    (3, 100, 1, 1, 1),
    (100, 3, 1, 1, 1),
    (100, 3, 0, 1, 2),
    (9, 17, 1, 2, 1),
    (17, 9, 0, 1, 1),
    (5, 200, 1, 1, 1),
]

# max_active_clusters values used for the persistent grid-shape goldens (tile_scheduler.py:110-123).
MAX_ACTIVE_CLUSTERS = [1, 7, 74, 148]

DIVISORS = (list(range(1, 65)) + [
    96, 100, 112, 127, 128, 255, 256, 257, 511, 512, 1000, 1023, 1024, 1025, 3584, 4096,
    7168, 9999, 14336, 28672, 65535, 65536, 65537, (1 << 20) - 1, (1 << 20), (1 << 24) + 1,
    123456789, (1 << 30) - 1, (1 << 30), (1 << 30) + 1, (1 << 31) - 1,
])


def _dividends(d, rng):
    base = [0, 1, 2, 3, d - 1, d, d + 1, 2 * d - 1, 2 * d, 2 * d + 1, 7 * d + 3,
            (1 << 31) - 1, (1 << 31) - 2, (1 << 30), (1 << 30) - 1, (1 << 16), (1 << 16) - 1]
    base += [int(x) for x in rng.integers(0, 1 << 31, size=24)]
    base += [int(x) for x in rng.integers(0, min(1 << 31, 64 * d + 64), size=8)]
    return sorted({x for x in base if 0 <= x < (1 << 31)})


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--reference", required=True, help="path of the reference checkout")
    ns = ap.parse_args()
    sys.dont_write_bytecode = True
    sys.path.insert(0, ns.reference)

    import cutlass
    import cutlass.cute as cute
    from cutlass import Int32, Uint32, Uint64
    from cutlass.cute.runtime import from_dlpack
    import fast_math
    import tile_scheduler as ts

    def host_umulhi(a, b, *, loc=None, ip=None):
        return Uint32((Uint64(Uint32(a)) * Uint64(Uint32(b))) >> 32)

    fast_math.umulhi = host_umulhi

    # ---------------- FastDivmod -----------------------------------------------------------
    @cute.jit
    def fdm_kernel(out: cute.Tensor, xs: cute.Tensor, n: cutlass.Constexpr, d: cutlass.Constexpr):
        f = fast_math.FastDivmod.create(d)
        out[0, 0] = Int32(f.multiplier)
        out[0, 1] = Int32(f.shift_right)
        for i in cutlass.range(n):
            q, r = f.divmod(xs[i])
            out[i + 1, 0] = q
            out[i + 1, 1] = r

    rng = np.random.default_rng(0)
    fdm = []
    for d in DIVISORS:
        xs = np.array(_dividends(d, rng), dtype=np.int32)
        out = np.zeros((len(xs) + 1, 2), dtype=np.int32)
        fdm_kernel(from_dlpack(out), from_dlpack(xs), len(xs), d)
        fdm.append({
            "divisor": d,
            "multiplier": int(np.uint32(out[0, 0])),
            "shift_right": int(np.uint32(out[0, 1])),
            "dividends": xs.tolist(),
            "quotients": out[1:, 0].tolist(),
            "remainders": out[1:, 1].tolist(),
        })
        print(f"fastdivmod d={d}: mult={fdm[-1]['multiplier']} shift={fdm[-1]['shift_right']}")
    with open(os.path.join(HERE, "fast_divmod.json"), "w") as f:
        json.dump({"generator": "tests/golden/gen_golden.py",
                   "source": "fast_math.py:56-81 (reference), umulhi as (u64(a)*u64(b))>>32",
                   "cases": fdm}, f, separators=(",", ":"))

    # ---------------- Tile scheduler --------------------------------------------------------
    @cute.jit
    def sched_kernel(out: cute.Tensor, grids: cute.Tensor,
                     ntm: cutlass.Constexpr, ntn: cutlass.Constexpr, raster: cutlass.Constexpr,
                     cm: cutlass.Constexpr, cn: cutlass.Constexpr, ncl: cutlass.Constexpr,
                     mac: cutlass.Constexpr):
        # Params.create via to_underlying_arguments, exactly as GemmSM90.__call__ does
        # (gemm_base.py:147-149), with the fixed group size 8 of gemm_base.py:65.
        args = ts.SimpleTileSchedulerArguments((ntm, ntn, 1), raster, Int32(8), (cm, cn, 1), True)
        p = ts.SimpleTileScheduler.to_underlying_arguments(args)
        sched = ts.SimpleTileScheduler(Int32(0), Int32(0), Int32(0), p)
        for i in cutlass.range(ncl):
            m, n = sched._map_cta_coords(Int32(i))
            out[i, 0] = m
            out[i, 1] = n
        # Params fields after the map rows.
        out[ncl, 0] = p.num_groups_regular
        out[ncl, 1] = p.dm_group_size.divisor
        out[ncl + 1, 0] = p.dm_group_size_tail.divisor
        out[ncl + 1, 1] = p.dm_num_clusters_in_group.divisor
        out[ncl + 2, 0] = p.dm_clusters_per_problem.divisor
        out[ncl + 2, 1] = p.ncluster_mnl[0]
        out[ncl + 3, 0] = p.ncluster_mnl[1]
        out[ncl + 3, 1] = p.ncluster_mnl[2]
        # Persistent grid shape for the given max_active_clusters.
        g = ts.SimpleTileScheduler.get_grid_shape(p, Int32(mac))
        grids[0] = g[0]
        grids[1] = g[1]
        grids[2] = g[2]

    @cute.jit
    def grid_np_kernel(grids: cute.Tensor, ntm: cutlass.Constexpr, ntn: cutlass.Constexpr,
                       raster: cutlass.Constexpr, cm: cutlass.Constexpr, cn: cutlass.Constexpr):
        args = ts.SimpleTileSchedulerArguments((ntm, ntn, 1), raster, Int32(8), (cm, cn, 1), False)
        p = ts.SimpleTileScheduler.to_underlying_arguments(args)
        g = ts.SimpleTileScheduler.get_grid_shape(p, Int32(1))
        grids[0] = g[0]
        grids[1] = g[1]
        grids[2] = g[2]

    maps = {}
    index = []
    for (ntm, ntn, raster, cm, cn) in TILE_CONFIGS:
        ncm = -(-ntm // cm)
        ncn = -(-ntn // cn)
        ncl = ncm * ncn
        key = f"m{ntm}_n{ntn}_r{raster}_c{cm}x{cn}"
        persistent_grids = {}
        mp = None
        params = None
        for mac in MAX_ACTIVE_CLUSTERS:
            out = np.zeros((ncl + 4, 2), dtype=np.int32)
            grids = np.zeros(3, dtype=np.int32)
            sched_kernel(from_dlpack(out), from_dlpack(grids), ntm, ntn, ts.RasterOrder(raster),
                         cm, cn, ncl, mac)
            persistent_grids[str(mac)] = grids.tolist()
            if mp is None:
                mp = out[:ncl].copy()
                params = {
                    "num_groups_regular": int(out[ncl, 0]),
                    "group_size": int(out[ncl, 1]),
                    "group_size_tail_divisor": int(out[ncl + 1, 0]),
                    "num_clusters_in_group": int(out[ncl + 1, 1]),
                    "clusters_per_problem": int(out[ncl + 2, 0]),
                    "ncluster_mnl": [int(out[ncl + 2, 1]), int(out[ncl + 3, 0]), int(out[ncl + 3, 1])],
                }
            else:
                assert np.array_equal(mp, out[:ncl])
        gnp = np.zeros(3, dtype=np.int32)
        grid_np_kernel(from_dlpack(gnp), ntm, ntn, ts.RasterOrder(raster), cm, cn)
        maps[key] = mp.astype(np.int16)
        index.append({
            "key": key, "ntiles_m": ntm, "ntiles_n": ntn, "raster_order": raster,
            "cluster_m": cm, "cluster_n": cn, "group_size_arg": 8,
            "params": params,
            "grid_nonpersistent": gnp.tolist(),
            "grid_persistent": persistent_grids,
            "map_sha256": hashlib.sha256(mp.astype("<i4").tobytes()).hexdigest(),
        })
        print(f"tile map {key}: {ncl} clusters, params {params}, grid {persistent_grids}")

    np.savez_compressed(os.path.join(HERE, "tile_maps.npz"), **maps)
    with open(os.path.join(HERE, "tile_maps.json"), "w") as f:
        json.dump({"generator": "tests/golden/gen_golden.py",
                   "source": "tile_scheduler.py:50-146 (reference), group size 8 (gemm_base.py:65)",
                   "max_active_clusters": MAX_ACTIVE_CLUSTERS,
                   "configs": index}, f, indent=1)


if __name__ == "__main__":
    main()
