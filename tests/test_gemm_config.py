"""Constructor surface of GemmSM90: same arguments, defaults and asserts as gemm_base.py:50-122,
and the C ABI's copy of the same checks (cpg_config_validate)."""
import inspect

import pytest

from cutedsl_pingpong_gemm_b200 import GemmSM90, GemmSM100, RasterOrder, _lib


def test_signature_matches_reference():
    sig = inspect.signature(GemmSM90.__init__)
    positional = [k for k, v in sig.parameters.items()
                  if v.kind == inspect.Parameter.POSITIONAL_OR_KEYWORD][1:]
    assert positional == ["tile_shape_mn", "epi_tile_mn", "cluster_shape_mnk", "atom_layout_mn",
                          "ab_stage", "epi_stage", "raster_order", "reuse_ab", "is_persistent",
                          "gemm_n_prologue"]
    # Additions of this build are keyword-only, with defaults that keep the reference behaviour.
    extra = {k: v for k, v in sig.parameters.items() if v.kind == inspect.Parameter.KEYWORD_ONLY}
    assert extra.keys() == {"dynamic_scheduler"} and extra["dynamic_scheduler"].default is False
    d = {k: v.default for k, v in sig.parameters.items()}
    assert d["ab_stage"] == 2 and d["epi_stage"] == 2
    assert d["raster_order"] == RasterOrder.AlongN
    assert d["reuse_ab"] is True and d["is_persistent"] is False and d["gemm_n_prologue"] == 0
    assert GemmSM100 is GemmSM90


def test_harness_config_attributes():
    # The reference harness configuration (gemm_base.py:598-604).
    g = GemmSM90(tile_shape_mn=(128, 256), epi_tile_mn=(128, 32), cluster_shape_mnk=(2, 1, 1),
                 atom_layout_mn=(2, 1), ab_stage=3, reuse_ab=False, is_persistent=True)
    assert g.cta_tile_shape_mnk == (128, 256, 64)
    assert g.atom_layout_mnk == (2, 1, 1)
    assert g.mma_warpgroups == 2
    assert g.scheduler_group_size == 8
    assert g.mcast_ctas_a == 1 and g.mcast_ctas_b == 2
    assert not g.is_a_mcast and not g.is_b_mcast  # no TMA multicast on sm_100a
    g.validate()


BAD = [
    # (kwargs, message fragment) -- each is an assert of gemm_base.py
    (dict(atom_layout_mn=(4, 1)), None),                                   # :72
    (dict(atom_layout_mn=(1, 3)), None),                                   # :72
    (dict(tile_shape_mn=(192, 256), atom_layout_mn=(2, 1)), None),         # :73 (192 % 128)
    (dict(tile_shape_mn=(128, 96), atom_layout_mn=(1, 2)), None),          # :74 (96 % 64)
    (dict(atom_layout_mn=(2, 2)), None),                                   # :87 (4 warpgroups)
    (dict(atom_layout_mn=(1, 2), epi_tile_mn=(128, 32)), "epi tile n"),    # :113
    (dict(reuse_ab=True, is_persistent=True), "reuse AB"),                 # :122
]


@pytest.mark.parametrize("kwargs,msg", BAD)
def test_reference_asserts(kwargs, msg):
    base = dict(tile_shape_mn=(128, 256), epi_tile_mn=(128, 32), cluster_shape_mnk=(1, 1, 1),
                atom_layout_mn=(1, 1), reuse_ab=False, is_persistent=False)
    base.update(kwargs)
    with pytest.raises(AssertionError) as e:
        GemmSM90(**base)
    if msg:
        assert msg in str(e.value)


@pytest.mark.parametrize("kwargs", [k for k, _ in BAD])
def test_capi_validate_matches_python_asserts(lib, kwargs):
    base = dict(tile_m=128, tile_n=256, epi_tile_m=128, epi_tile_n=32, cluster_m=1, cluster_n=1,
                cluster_k=1, atom_m=1, atom_n=1, ab_stage=4, epi_stage=2, raster_order=1,
                reuse_ab=0, is_persistent=0, gemm_n_prologue=0, group_size=8)
    if "atom_layout_mn" in kwargs:
        base["atom_m"], base["atom_n"] = kwargs["atom_layout_mn"]
    if "tile_shape_mn" in kwargs:
        base["tile_m"], base["tile_n"] = kwargs["tile_shape_mn"]
    if "epi_tile_mn" in kwargs:
        base["epi_tile_m"], base["epi_tile_n"] = kwargs["epi_tile_mn"]
    if "reuse_ab" in kwargs:
        base["reuse_ab"] = int(kwargs["reuse_ab"])
    if "is_persistent" in kwargs:
        base["is_persistent"] = int(kwargs["is_persistent"])
    import ctypes
    cfg = _lib.GemmConfigC(**base)
    assert lib.cpg_config_validate(ctypes.byref(cfg)) == _lib.CPG_ERR_INVALID_CONFIG


def test_capi_validate_accepts_harness_config(lib):
    import ctypes
    cfg = _lib.GemmConfigC(128, 256, 128, 32, 2, 1, 1, 2, 1, 3, 2, 1, 0, 1, 0, 8)
    assert lib.cpg_config_validate(ctypes.byref(cfg)) == _lib.CPG_OK
    cfg.cluster_k = 2  # tile_scheduler.py:51
    assert lib.cpg_config_validate(ctypes.byref(cfg)) == _lib.CPG_ERR_INVALID_CONFIG


def test_wave_split_k_choices():
    """K ranges that fill whole waves of resident clusters (the automatic in-GPU split)."""
    from cutedsl_pingpong_gemm_b200.gemm_base import wave_split_k
    # 2048 x 2048 in 256 x 256 pair tiles (64 clusters of 74), K = 65536: 8 ranges fill 512 of
    # 518 cluster slots; a quarter of the columns (16 clusters) takes 9.
    assert wave_split_k(64, 1024, 74, min_fill=0.85) == 8
    assert wave_split_k(16, 1024, 74, min_fill=0.85) == 9
    # Decode-like M = 128, N = K = 8192 (64 tiles of 148 slots, 128 k-blocks): no split fills a
    # wave well enough with >= 32 k-blocks per range, so the caller falls back to Stream-K.
    assert wave_split_k(64, 128, 148) is None
    for clusters, kblocks, slots in ((64, 1024, 74), (16, 1024, 74), (10, 4096, 148)):
        s = wave_split_k(clusters, kblocks, slots, min_fill=0.85)
        units = clusters * s
        assert kblocks // s >= 32
        assert units / (-(-units // slots) * slots) >= 0.85
    assert wave_split_k(4, 40, 148) is None  # too few k-blocks to split


def test_capi_validate_dynamic_scheduler(lib):
    """dynamic_scheduler is 0 or 1 and excludes reuse_ab (several tiles per CTA); the Python
    constructor asserts the same."""
    import ctypes
    cfg = _lib.GemmConfigC(128, 256, 128, 32, 2, 1, 1, 1, 1, 4, 2, 1, 0, 1, 0, 8, 1)
    assert lib.cpg_config_validate(ctypes.byref(cfg)) == _lib.CPG_OK
    cfg.dynamic_scheduler = 2
    assert lib.cpg_config_validate(ctypes.byref(cfg)) == _lib.CPG_ERR_INVALID_CONFIG
    cfg.dynamic_scheduler = 1
    cfg.reuse_ab, cfg.is_persistent = 1, 0
    assert lib.cpg_config_validate(ctypes.byref(cfg)) == _lib.CPG_ERR_INVALID_CONFIG
    with pytest.raises(AssertionError):
        GemmSM90(tile_shape_mn=(128, 256), epi_tile_mn=(128, 32), cluster_shape_mnk=(1, 1, 1),
                 atom_layout_mn=(1, 1), reuse_ab=True, is_persistent=False,
                 dynamic_scheduler=True)
    g = GemmSM90(tile_shape_mn=(128, 256), epi_tile_mn=(128, 32), cluster_shape_mnk=(2, 1, 1),
                 atom_layout_mn=(1, 1), reuse_ab=False, is_persistent=False,
                 dynamic_scheduler=True)
    assert g._config_c().dynamic_scheduler == 1
    g.validate()


def test_auto_split_k_avoids_stream_k_when_dynamic(monkeypatch):
    """Stream-K partitions the k-blocks statically, so the automatic split of a dynamic-schedule
    GEMM picks K ranges instead (M = 256, N = K = 8192 would take Stream-K); one batch of at
    most 128 rows takes the small-M kernel under either schedule."""
    from cutedsl_pingpong_gemm_b200.gemm_base import CompiledGemm
    for dyn, want_stream in ((False, True), (True, False)):
        g = GemmSM90(tile_shape_mn=(128, 128), epi_tile_mn=(128, 32), cluster_shape_mnk=(1, 1, 1),
                     atom_layout_mn=(1, 1), ab_stage=6, reuse_ab=False, is_persistent=True,
                     dynamic_scheduler=dyn)
        g._max_active_clusters = 148  # B200: one CTA per SM (no GPU here)
        c = CompiledGemm.__new__(CompiledGemm)
        c.gemm = g
        s = c.auto_split_k(256, 8192, 8192)
        assert (s == _lib.CPG_SPLIT_K_STREAM) == want_stream, (dyn, s)
        assert s != 0
        assert c.auto_split_k(128, 8192, 8192) == _lib.CPG_SPLIT_K_DECODE
        assert c.auto_split_k(128, 8192, 8192, batches=2) != _lib.CPG_SPLIT_K_DECODE


def test_release_drops_cached_plans_and_workspaces():
    from cutedsl_pingpong_gemm_b200.gemm_base import CompiledGemm
    gemm = GemmSM90(tile_shape_mn=(128, 256), epi_tile_mn=(128, 32), cluster_shape_mnk=(2, 1, 1),
                    atom_layout_mn=(1, 1), ab_stage=4, reuse_ab=False, is_persistent=True)
    gemm.release()  # nothing compiled yet: no-op
    compiled = CompiledGemm(gemm)
    gemm._compiled = compiled
    compiled._plans["plan"] = object()
    compiled._workspaces["workspace"] = object()
    gemm.release()
    assert compiled._plans == {} and compiled._workspaces == {}
