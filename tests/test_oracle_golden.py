"""Pin the CPU oracle to golden vectors produced by the reference's own code.

The goldens (tests/golden/) come from executing the reference's fast_math.py and
tile_scheduler.py under CuTe-DSL (tests/golden/gen_golden.py).  If these tests pass, the oracle
used by every other test is the reference's arithmetic, bit for bit.
"""
import hashlib

import numpy as np

from oracle import fast_math_ref, tile_scheduler_ref as ts


def test_fastdivmod_params_match_reference(golden_fdm):
    assert len(golden_fdm) >= 90
    for case in golden_fdm:
        f = fast_math_ref.FastDivmod.create(case["divisor"])
        assert f.multiplier == case["multiplier"], case["divisor"]
        assert f.shift_right == case["shift_right"], case["divisor"]


def test_fastdivmod_divmod_match_reference(golden_fdm):
    n = 0
    for case in golden_fdm:
        f = fast_math_ref.FastDivmod.create(case["divisor"])
        for x, q, r in zip(case["dividends"], case["quotients"], case["remainders"]):
            assert f.divmod(x) == (q, r), (case["divisor"], x)
            assert (q, r) == divmod(x, case["divisor"])  # the reference is exact on this range
            n += 1
    assert n > 3000


def test_known_answer_table():
    # Values the reference's FastDivmod.create returned when it was executed on the host
    # (fast_math.py:56-76), written out as a known-answer table.
    table = {1: (0x80000000, 0xFFFFFFFF), 2: (0x80000000, 0), 7: (2454267027, 2),
             8: (0x80000000, 2), 12: (2863311531, 3), 64: (0x80000000, 5), 1000: (2199023256, 9)}
    for d, (mult, shift) in table.items():
        f = fast_math_ref.FastDivmod.create(d)
        assert (f.multiplier, f.shift_right) == (mult, shift)


def test_scheduler_params_match_reference(golden_maps):
    index, _ = golden_maps
    assert len(index["configs"]) >= 30
    for cfg in index["configs"]:
        p = ts.params_create((cfg["ntiles_m"], cfg["ntiles_n"], 1), cfg["raster_order"],
                             cfg["group_size_arg"], (cfg["cluster_m"], cfg["cluster_n"], 1), True)
        g = cfg["params"]
        assert p.num_groups_regular == g["num_groups_regular"], cfg["key"]
        assert p.dm_group_size.divisor == g["group_size"], cfg["key"]
        assert p.dm_group_size_tail.divisor == g["group_size_tail_divisor"], cfg["key"]
        assert p.dm_num_clusters_in_group.divisor == g["num_clusters_in_group"], cfg["key"]
        assert p.dm_clusters_per_problem.divisor == g["clusters_per_problem"], cfg["key"]
        assert list(p.ncluster_mnl) == g["ncluster_mnl"], cfg["key"]


def test_scheduler_map_matches_reference(golden_maps):
    index, maps = golden_maps
    for cfg in index["configs"]:
        p = ts.params_create((cfg["ntiles_m"], cfg["ntiles_n"], 1), cfg["raster_order"],
                             cfg["group_size_arg"], (cfg["cluster_m"], cfg["cluster_n"], 1), True)
        ours = np.array(ts.cluster_map(p), dtype=np.int32)
        ref = maps[cfg["key"]]
        assert ours.shape == ref.shape, cfg["key"]
        assert np.array_equal(ours, ref), cfg["key"]
        assert hashlib.sha256(ours.astype("<i4").tobytes()).hexdigest() == cfg["map_sha256"]


def test_scheduler_map_is_a_permutation(golden_maps):
    # Every cluster of the problem is visited exactly once.
    index, maps = golden_maps
    for cfg in index["configs"]:
        ncm, ncn = cfg["params"]["ncluster_mnl"][:2]
        m = maps[cfg["key"]]
        seen = set(map(tuple, m.tolist()))
        assert len(seen) == ncm * ncn == len(m), cfg["key"]
        assert all(0 <= a < ncm and 0 <= b < ncn for a, b in seen), cfg["key"]


def test_grid_shapes_match_reference(golden_maps):
    index, _ = golden_maps
    for cfg in index["configs"]:
        args = ((cfg["ntiles_m"], cfg["ntiles_n"], 1), cfg["raster_order"], cfg["group_size_arg"],
                (cfg["cluster_m"], cfg["cluster_n"], 1))
        p = ts.params_create(*args, True)
        for mac, grid in cfg["grid_persistent"].items():
            assert list(ts.get_grid_shape(p, int(mac))) == grid, (cfg["key"], mac)
        pn = ts.params_create(*args, False)
        assert list(ts.get_grid_shape(pn, 1)) == cfg["grid_nonpersistent"], cfg["key"]


def test_schedule_covers_every_tile_once():
    # Persistent and non-persistent launches visit each (pid_m, pid_n) of the cluster grid once.
    for persistent in (True, False):
        for cluster in ((1, 1, 1), (2, 1, 1), (1, 2, 1), (2, 2, 1)):
            p = ts.params_create((13, 7, 1), ts.ALONG_N, 8, cluster, persistent)
            grid = ts.get_grid_shape(p, 11)
            sched = ts.schedule(p, grid)
            tiles = [t for seq in sched.values() for t in seq]
            assert len(tiles) == len(set(tiles))
            ncm, ncn = p.ncluster_mnl[:2]
            assert len(tiles) == ncm * cluster[0] * ncn * cluster[1]


def test_oracle_activations_match_torch():
    """The fused-epilogue oracle's activation formulas equal torch's published ones."""
    import torch
    import torch.nn.functional as F
    from oracle import gemm_ref
    y = torch.linspace(-30, 30, 100001, dtype=torch.float64)
    assert torch.allclose(gemm_ref.activation("silu", y), F.silu(y), rtol=1e-12, atol=1e-12)
    assert torch.allclose(gemm_ref.activation("gelu", y), F.gelu(y), rtol=1e-12, atol=1e-12)
    assert torch.allclose(gemm_ref.activation("gelu_tanh", y), F.gelu(y, approximate="tanh"),
                          rtol=1e-12, atol=1e-12)
    assert torch.equal(gemm_ref.activation("relu", y), F.relu(y))
