"""C ABI library checks that need no GPU: it loads, exports every symbol of include/cpgemm.h,
and its host-side scheduler / FastDivmod code (the same headers the kernels compile) matches the
golden vectors taken from the reference."""
import ctypes
import os
import re

import numpy as np
import pytest

from conftest import ROOT
from cutedsl_pingpong_gemm_b200 import _lib
from cutedsl_pingpong_gemm_b200.fast_math import FastDivmod
from cutedsl_pingpong_gemm_b200.tile_scheduler import (RasterOrder, SimpleTileScheduler,
                                                        SimpleTileSchedulerArguments)


def declared_functions():
    with open(os.path.join(ROOT, "include", "cpgemm.h")) as f:
        text = f.read()
    text = re.sub(r"/\*.*?\*/", "", text, flags=re.S)
    return sorted(set(re.findall(r"\b(cpg_[a-z0-9_]+)\s*\(", text)))


def test_library_exports_every_declared_symbol(lib):
    names = declared_functions()
    assert len(names) >= 15
    for name in names:
        assert hasattr(lib, name), name
    # The ctypes binding covers exactly the declared functions.
    assert sorted(_lib.SIGNATURES) == names


def test_abi_version_and_strerror(lib):
    assert lib.cpg_abi_version() == _lib.ABI_VERSION
    for code in range(-10, 1):
        assert lib.cpg_strerror(code)
    assert lib.cpg_strerror(-999) == b"unknown error"


def test_fastdivmod_host_matches_reference(lib, golden_fdm):
    for case in golden_fdm:
        f = FastDivmod.create(case["divisor"])
        assert (f.multiplier, f.shift_right) == (case["multiplier"], case["shift_right"])
        for x, q, r in list(zip(case["dividends"], case["quotients"], case["remainders"]))[:12]:
            assert f.divmod(x) == (q, r)


def test_fastdivmod_rejects_bad_divisor(lib):
    with pytest.raises(_lib.CpgError) as e:
        FastDivmod.create(0)
    assert e.value.code == _lib.CPG_ERR_INVALID_SHAPE


def _params(cfg, persistent=True):
    args = SimpleTileSchedulerArguments((cfg["ntiles_m"], cfg["ntiles_n"], 1),
                                        RasterOrder(cfg["raster_order"]), cfg["group_size_arg"],
                                        (cfg["cluster_m"], cfg["cluster_n"], 1), persistent)
    return SimpleTileScheduler.to_underlying_arguments(args)


def test_host_scheduler_matches_reference(lib, golden_maps):
    index, maps = golden_maps
    for cfg in index["configs"]:
        p = _params(cfg)
        g = cfg["params"]
        assert p.num_groups_regular == g["num_groups_regular"]
        assert p.dm_group_size.divisor == g["group_size"]
        assert p.dm_group_size_tail.divisor == g["group_size_tail_divisor"]
        assert p.dm_num_clusters_in_group.divisor == g["num_clusters_in_group"]
        assert list(p.ncluster_mnl) == g["ncluster_mnl"]
        ours = SimpleTileScheduler.cluster_map(p)
        assert np.array_equal(ours, maps[cfg["key"]]), cfg["key"]
        for mac, grid in cfg["grid_persistent"].items():
            assert list(SimpleTileScheduler.get_grid_shape(p, int(mac))) == grid
        pn = _params(cfg, persistent=False)
        assert list(SimpleTileScheduler.get_grid_shape(pn, 1)) == cfg["grid_nonpersistent"]


def test_host_schedule_matches_oracle_schedule(lib):
    from oracle import tile_scheduler_ref as ts
    for persistent in (True, False):
        for cluster in ((1, 1, 1), (2, 1, 1), (2, 2, 1)):
            args = SimpleTileSchedulerArguments((9, 17, 1), RasterOrder.AlongN, 8, cluster, persistent)
            p = SimpleTileScheduler.to_underlying_arguments(args)
            grid = SimpleTileScheduler.get_grid_shape(p, 5)
            ours = SimpleTileScheduler.schedule(p, grid)
            po = ts.params_create((9, 17, 1), ts.ALONG_N, 8, cluster, persistent)
            assert ours == ts.schedule(po, ts.get_grid_shape(po, 5))


def test_map_cta_coords_single_id_matches_reference(lib, golden_maps):
    """The O(1) single-id map equals the reference-executed map at every id of every config."""
    index, maps = golden_maps
    for cfg in index["configs"][:12]:
        p = _params(cfg)
        want = maps[cfg["key"]]
        for cid in range(want.shape[0]):
            assert SimpleTileScheduler._map_cta_coords(p, cid) == tuple(want[cid]), (cfg["key"], cid)


@pytest.mark.parametrize("persistent", [True, False])
@pytest.mark.parametrize("cluster", [(1, 1, 1), (2, 1, 1), (1, 2, 1)])
def test_schedule_with_batches_covers_every_tile_once(lib, persistent, cluster):
    """L = 3 batches: every (pid_m, pid_n, l) of the problem appears exactly once, and batch 0
    holds the single-batch schedule's tiles."""
    ntm, ntn, nl = 6, 10, 3
    args = SimpleTileSchedulerArguments((ntm, ntn, nl), RasterOrder.AlongN, 8, cluster, persistent)
    p = SimpleTileScheduler.to_underlying_arguments(args)
    grid = SimpleTileScheduler.get_grid_shape(p, 7)
    tiles = [t for seq in SimpleTileScheduler.schedule(p, grid).values() for t in seq]
    assert sorted(tiles) == sorted((m, n, l) for m in range(ntm) for n in range(ntn)
                                   for l in range(nl))
    one = SimpleTileScheduler.to_underlying_arguments(
        SimpleTileSchedulerArguments((ntm, ntn, 1), RasterOrder.AlongN, 8, cluster, persistent))
    single = {t for seq in SimpleTileScheduler.schedule(
        one, SimpleTileScheduler.get_grid_shape(one, 7)).values() for t in seq}
    assert {t[:2] for t in tiles if t[2] == 0} == single


def test_sched_params_reject_cluster_k(lib):
    args = SimpleTileSchedulerArguments((4, 4, 1), RasterOrder.AlongN, 8, (1, 1, 2), True)
    with pytest.raises(_lib.CpgError) as e:
        SimpleTileScheduler.to_underlying_arguments(args)
    assert e.value.code == _lib.CPG_ERR_INVALID_CONFIG


def test_gemm_create_without_device_fails_cleanly(lib):
    """On a machine without a GPU the plan call returns an error code instead of crashing."""
    import torch
    if torch.cuda.is_available():
        pytest.skip("has a GPU")
    cfg = _lib.GemmConfigC(128, 256, 128, 32, 1, 1, 1, 2, 1, 4, 2, 1, 0, 1, 0, 8)
    prob = _lib.GemmProblemC(256, 256, 256, 256, 256, 256, 0, 0)
    h = ctypes.c_void_p()
    rc = lib.cpg_gemm_create(ctypes.byref(cfg), ctypes.byref(prob), 0, ctypes.byref(h))
    assert rc in (_lib.CPG_ERR_NO_DEVICE, _lib.CPG_ERR_CUDA)
    assert not h.value


def _header_struct_fields(name):
    """Field names, in order, of `typedef struct name { ... } name;` in include/cpgemm.h."""
    import re
    text = open(os.path.join(ROOT, "include", "cpgemm.h")).read()
    body = text[text.index(f"typedef struct {name} {{"):]
    body = body[body.index("{") + 1:body.index(f"}} {name};")]
    body = re.sub(r"/\*.*?\*/", "", body, flags=re.S)
    fields = []
    for decl in body.split(";"):
        decl = decl.strip()
        if not decl:
            continue
        names = decl.split(None, 1)[1] if not decl.startswith("const ") else decl.split(None, 2)[2]
        for part in names.split(","):
            fields.append(part.strip().lstrip("*").strip())
    return fields


@pytest.mark.parametrize("c_name,py_struct", [("cpg_gemm_config", "GemmConfigC"),
                                              ("cpg_gemm_problem", "GemmProblemC"),
                                              ("cpg_epilogue", "EpilogueC")])
def test_ctypes_structs_match_header(c_name, py_struct):
    struct = getattr(_lib, py_struct)
    assert [f[0] for f in struct._fields_] == _header_struct_fields(c_name)


def test_sched_rs_arrivals_match_the_counting_rule():
    """The peer reduce-scatter's arrival count (no GPU): every CTA tile of the schedule -- the row
    tiles of all clusters, a pair's tile past M included -- makes one arrival per epilogue warp
    (4, or 8 for 512-wide tiles) on the rank owning its first row; rows past M count for the last
    rank."""
    import ctypes
    from cutedsl_pingpong_gemm_b200 import _lib
    from cutedsl_pingpong_gemm_b200.sharding import peer_row_starts
    lib = _lib.load()
    for m, n, tile_n, cluster, world in ((600, 1000, 256, (2, 1), 2), (2048, 2048, 256, (2, 1), 8),
                                          (129, 64, 128, (1, 2), 3), (640, 512, 512, (1, 1), 4)):
        ntm, ntn = -(-m // 128), -(-n // tile_n)
        sp = _lib.SchedParamsC()
        assert lib.cpg_sched_params_create(ntm, ntn, 1, 1, 8, cluster[0], cluster[1], 1, 1,
                                           ctypes.byref(sp)) == 0
        rs = _lib.ReduceScatterC()
        rs.ranks = world
        starts = peer_row_starts(m, world)
        for q in range(world + 1):
            rs.row_start[q] = starts[q]
        out = (ctypes.c_uint32 * world)()
        assert lib.cpg_sched_rs_arrivals(ctypes.byref(sp), tile_n, ctypes.byref(rs), out) == 0
        warps = 8 if tile_n == 512 else 4
        want = [0] * world
        cta_rows = sp.ncluster_m * cluster[0]
        cta_cols = sp.ncluster_n * cluster[1]
        for i in range(cta_rows):
            owner = next((q for q in range(world) if i * 128 < starts[q + 1]), world - 1)
            want[owner] += warps * cta_cols
        assert list(out) == want, (m, n, cluster, world, list(out), want)
        assert sum(out) == warps * cta_rows * cta_cols


@pytest.mark.parametrize("tile_n,cluster,raster,dynamic,dtype,k,want", [
    # AlongN, 256 x 512 pair tiles: 512 rows of B per cluster column.
    (512, (2, 1), 1, 1, "bf16", 8192, 4),      # 8 MiB per column
    (512, (2, 1), 1, 1, "e4m3", 8192, 8),      # 4 MiB: the reference's 8
    (512, (2, 1), 1, 1, "bf16", 16384, 2),
    (512, (2, 1), 1, 1, "bf16", 131072, 1),    # one column is over 32 MiB: at least 1
    (512, (2, 1), 1, 1, "bf16", 320, 8),
    (512, (2, 1), 1, 1, "bf16", 0, 8),
    (512, (2, 1), 1, 0, "bf16", 131072, 8),    # static schedule: the configured size
    (256, (1, 2), 1, 1, "bf16", 8192, 4),      # cluster_n 2: 512 rows of B per column
    (256, (1, 1), 1, 1, "bf16", 8192 + 1, 7),  # 256 rows over 129 k-blocks: just over 4 MiB
    (256, (2, 1), 0, 1, "bf16", 8192, 8),      # AlongM: 256 rows of A per cluster row
    (256, (1, 1), 0, 1, "bf16", 65536, 2),     # 128 rows of A over 1024 k-blocks: 16 MiB
])
def test_plan_group_size_rule(lib, tile_n, cluster, raster, dynamic, dtype, k, want):
    cfg = _lib.GemmConfigC(128, tile_n, 128, 32, cluster[0], cluster[1], 1, 1, 1, 3, 2, raster,
                           0, 1, 0, 8, dynamic)
    code = {"bf16": _lib.CPG_DTYPE_BF16, "e4m3": _lib.CPG_DTYPE_E4M3}[dtype]
    out = ctypes.c_int32()
    assert lib.cpg_sched_plan_group_size(ctypes.byref(cfg), k, code, ctypes.byref(out)) == 0
    assert out.value == want


def test_plan_group_size_rejects_bad_arguments(lib):
    cfg = _lib.GemmConfigC(128, 512, 128, 32, 2, 1, 1, 1, 1, 3, 2, 1, 0, 1, 0, 8, 1)
    out = ctypes.c_int32()
    assert lib.cpg_sched_plan_group_size(ctypes.byref(cfg), -1, _lib.CPG_DTYPE_BF16,
                                         ctypes.byref(out)) == _lib.CPG_ERR_INVALID_SHAPE
    assert lib.cpg_sched_plan_group_size(ctypes.byref(cfg), 64, _lib.CPG_DTYPE_F32,
                                         ctypes.byref(out)) == _lib.CPG_ERR_DTYPE
    assert lib.cpg_sched_plan_group_size(None, 64, _lib.CPG_DTYPE_BF16,
                                         ctypes.byref(out)) == _lib.CPG_ERR_NULL
    bad = _lib.GemmConfigC(128, 512, 128, 32, 2, 1, 1, 1, 1, 3, 2, 1, 0, 1, 0, 0, 1)  # group 0
    assert lib.cpg_sched_plan_group_size(ctypes.byref(bad), 64, _lib.CPG_DTYPE_BF16,
                                         ctypes.byref(out)) == _lib.CPG_ERR_INVALID_CONFIG


def test_entry_points_reject_bad_arguments_before_touching_the_gpu(lib):
    """Every entry point validates its arguments first and returns a CPG_ERR_* code with a
    message; none of these calls reaches the CUDA runtime."""
    null = None
    f32, bf16 = _lib.CPG_DTYPE_F32, _lib.CPG_DTYPE_BF16
    cases = [
        # quantiser: extents, dtype, scales, block shapes
        (lambda: lib.cpg_quantize_e4m3(null, bf16, -1, 8, 8, null, 8, null, 0, 0, null),
         _lib.CPG_ERR_INVALID_SHAPE, "extents"),
        (lambda: lib.cpg_quantize_e4m3(null, bf16, 4, 16, 8, null, 16, null, 0, 0, null),
         _lib.CPG_ERR_INVALID_SHAPE, "extents"),
        (lambda: lib.cpg_quantize_e4m3(null, _lib.CPG_DTYPE_E4M3, 4, 8, 8, null, 8, null, 0, 0,
                                       null), _lib.CPG_ERR_DTYPE, "BF16 or FP32"),
        (lambda: lib.cpg_quantize_e4m3(null, bf16, 4, 8, 8, null, 8, null, 0, 0, null),
         _lib.CPG_ERR_NULL, "scales"),
        # cast: extents and NULL buffers
        (lambda: lib.cpg_cast_f32_bf16(null, 4, 8, 4, null, 8, null, null),
         _lib.CPG_ERR_INVALID_SHAPE, "extents"),
        (lambda: lib.cpg_cast_f32_bf16(null, 4, 8, 8, null, 8, null, null),
         _lib.CPG_ERR_NULL, "non-NULL"),
        # peer buffers and the peer finish
        (lambda: lib.cpg_peer_alloc(0, ctypes.byref(ctypes.c_void_p()),
                                    ctypes.byref(_lib.IpcHandleC())),
         _lib.CPG_ERR_INVALID_SHAPE, "positive"),
        (lambda: lib.cpg_peer_open(null, ctypes.byref(ctypes.c_void_p())),
         _lib.CPG_ERR_NULL, "NULL"),
        (lambda: lib.cpg_peer_finish(null, 8, null, 0, 4, 6, null, 8, null, null, 100, null),
         _lib.CPG_ERR_ALIGNMENT, "multiples of 4"),
        (lambda: lib.cpg_peer_finish(null, 8, null, 0, 4, 8, null, 8, null, null, 100, null),
         _lib.CPG_ERR_NULL, "count and status"),
        # plans
        (lambda: lib.cpg_gemm_run(null, null, null, null, null, null), _lib.CPG_ERR_NULL, "NULL"),
        (lambda: lib.cpg_gemm_run_grouped(null, null, null, null, null, null, null),
         _lib.CPG_ERR_NULL, "NULL"),
        (lambda: lib.cpg_gemm_status(null, ctypes.byref(ctypes.c_int32())), _lib.CPG_ERR_NULL,
         "non-NULL"),
        (lambda: lib.cpg_gemm_splitk_static(null, null, null, null, null, null, null),
         _lib.CPG_ERR_NULL, "non-NULL"),
        (lambda: lib.cpg_sched_cluster_map(null, null, 4), _lib.CPG_ERR_NULL, "NULL"),
    ]
    for i, (call, code, words) in enumerate(cases):
        assert call() == code, i
        assert words in lib.cpg_last_error_message().decode(), (i, lib.cpg_last_error_message())
    # Destroying or closing nothing is not an error.
    assert lib.cpg_gemm_destroy(null) == _lib.CPG_OK
    assert lib.cpg_peer_close(null) == _lib.CPG_OK and lib.cpg_peer_free(null) == _lib.CPG_OK


def test_static_splitk_rejects_huge_extents_without_overflow(lib):
    """M = N = 2^31 - 1 would need about 2^64 bytes of FP32 scratch: a size check that multiplies
    first wraps past 2^63 and lets the call through.  The entry point must reject it with
    CPG_ERR_INVALID_SHAPE before any CUDA call (none is possible here: no GPU)."""
    big = (1 << 31) - 1
    cfg = _lib.GemmConfigC(128, 256, 128, 32, 1, 1, 1, 1, 1, 4, 2, 1, 0, 1, 0, 8)
    for m, n in ((big, big), (big, 4), (2, big), (4097, 1024)):
        ldd = (n + 7) // 8 * 8
        prob = _lib.GemmProblemC(m, n, 64, 64, 64, ldd, _lib.CPG_DTYPE_BF16, _lib.CPG_DTYPE_BF16,
                                 _lib.CPG_SCALE_TENSOR, 2)
        rc = lib.cpg_gemm_splitk_static(ctypes.byref(cfg), ctypes.byref(prob), None, None, None,
                                        None, None)
        assert rc == _lib.CPG_ERR_INVALID_SHAPE, (m, n, rc)
        assert "static scratch" in lib.cpg_last_error_message().decode(), (m, n)


def test_product_code_never_imports_the_oracle():
    """The oracle is the checker only: the package imports nothing from it, and bench.py reaches
    it only from its CPU-baseline / reference-arm functions."""
    import ast
    pkg = os.path.join(ROOT, "cutedsl_pingpong_gemm_b200")
    for name in sorted(os.listdir(pkg)):
        if name.endswith(".py"):
            with open(os.path.join(pkg, name)) as f:
                tree = ast.parse(f.read())
            for node in ast.walk(tree):
                if isinstance(node, ast.ImportFrom):
                    assert not (node.module or "").startswith("oracle"), name
                elif isinstance(node, ast.Import):
                    assert not any(a.name.startswith("oracle") for a in node.names), name
    with open(os.path.join(ROOT, "bench.py")) as f:
        tree = ast.parse(f.read())
    users = set()
    for fn in ast.walk(tree):
        if isinstance(fn, ast.FunctionDef):
            for node in ast.walk(fn):
                if isinstance(node, ast.ImportFrom) and (node.module or "").startswith("oracle"):
                    users.add(fn.name)
    assert users == {"cpu_matmul_rate", "run_reference"}, users
