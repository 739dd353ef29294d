"""GPU parity tests: the sm_100a kernels through the public API / C ABI against the CPU oracle.

Tolerance (BF16 output, fp32 accumulate), from the project spec and restated in oracle/gemm_ref.py:
  * relative Frobenius error <= 1e-2
  * element-wise |D - R| <= 2^-8 |R| + K * 2^-23 * (|A| @ |B|^T)
Tile order: the (pid_m, pid_n) sequence each CTA of the real kernel executed (device trace) must
equal the oracle's restatement of the reference scheduler, bit for bit.
"""
import numpy as np
import pytest
import torch

from cutedsl_pingpong_gemm_b200 import GemmSM90, RasterOrder, SimpleTileScheduler, compile as cpg_compile
from cutedsl_pingpong_gemm_b200 import _lib
from cutedsl_pingpong_gemm_b200.fast_math import FastDivmod
from oracle import gemm_ref
from oracle import tile_scheduler_ref as ts

pytestmark = pytest.mark.gpu


def make_gemm(tile_n=256, cluster=(1, 1, 1), persistent=True, stages=4, raster=RasterOrder.AlongN,
              reuse_ab=False, epi_stage=2):
    return GemmSM90(tile_shape_mn=(128, tile_n), epi_tile_mn=(128, 32), cluster_shape_mnk=cluster,
                    atom_layout_mn=(1, 1), ab_stage=stages, epi_stage=epi_stage, raster_order=raster,
                    reuse_ab=reuse_ab, is_persistent=persistent)


def run_and_check(m, n, k, gemm, seed=0, a_scale=1.0, b_scale=1.0, bias=False, alpha=1.0):
    a, b, bb = gemm_ref.make_inputs(m, n, k, seed=seed, a_scale=a_scale, b_scale=b_scale,
                                    with_bias=bias)
    da, db = a.cuda(), b.cuda()
    dbias = bb.cuda() if bb is not None else None
    d = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    gemm(da, db, d, None, bias=dbias, alpha=alpha)
    torch.cuda.synchronize()
    res = gemm_ref.check(d.cpu(), a, b, bias=bb, alpha=alpha)
    assert res["ok"], (m, n, k, res)
    return res


# ---------------------------------------------------------------- shared device code
def test_fastdivmod_device_matches_reference(golden_fdm):
    for case in golden_fdm:
        f = FastDivmod.create(case["divisor"])
        x = torch.tensor(case["dividends"], dtype=torch.int32, device="cuda")
        q, r = f.divmod_device(x)
        assert q.cpu().tolist() == case["quotients"], case["divisor"]
        assert r.cpu().tolist() == case["remainders"], case["divisor"]


def test_fastdivmod_device_exhaustive_sample():
    # Dense sweep of dividends below 2^31 for a few awkward divisors, against Python's //.
    x = torch.arange(0, 1 << 24, dtype=torch.int64)
    x = (x * 127 + 11) % (1 << 31)
    xs = x.to(torch.int32).cuda()
    for d in (3, 7, 37, 1000, 14336, 65537, 123456789, (1 << 31) - 1):
        q, r = FastDivmod.create(d).divmod_device(xs)
        assert torch.equal(q.cpu().to(torch.int64), x // d), d
        assert torch.equal(r.cpu().to(torch.int64), x % d), d


def test_scheduler_device_map_matches_reference(golden_maps):
    from cutedsl_pingpong_gemm_b200.tile_scheduler import SimpleTileSchedulerArguments
    index, maps = golden_maps
    for cfg in index["configs"]:
        args = SimpleTileSchedulerArguments((cfg["ntiles_m"], cfg["ntiles_n"], 1),
                                            RasterOrder(cfg["raster_order"]), 8,
                                            (cfg["cluster_m"], cfg["cluster_n"], 1), True)
        p = SimpleTileScheduler.to_underlying_arguments(args)
        dev = SimpleTileScheduler.cluster_map_device(p).cpu().numpy()
        assert np.array_equal(dev, maps[cfg["key"]]), cfg["key"]


# ---------------------------------------------------------------- tile order of the real kernel
def traced_schedule(gemm, m, n, k):
    """Run the GEMM with the device tile trace on; return (kernel schedule, oracle schedule)."""
    a, b, _ = gemm_ref.make_inputs(m, n, k, seed=1)
    da, db = a.cuda(), b.cuda()
    d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    compiled = cpg_compile(gemm, da, db, d, None)
    plan = compiled.plan_for(da, db, d)
    info = plan.launch_info()
    grid = info["grid"]
    p = plan.sched_params()
    total = p.ncluster_mnl[0] * p.ncluster_mnl[1]
    per_cta = -(-total // grid[2]) if p.is_persistent else 1
    nctas = grid[0] * grid[1] * grid[2]
    trace = torch.full((nctas * per_cta * 2,), -1, dtype=torch.int32, device="cuda")
    plan.set_trace(trace, per_cta)
    compiled(da, db, d, None)
    torch.cuda.synchronize()
    plan.set_trace(None, 0)
    t = trace.cpu().numpy().reshape(nctas, per_cta, 2)
    got = {}
    for z in range(grid[2]):
        for y in range(grid[1]):
            for x in range(grid[0]):
                c = x + grid[0] * (y + grid[1] * z)
                got[(x, y, z)] = [tuple(map(int, e)) for e in t[c] if e[0] >= 0]
    po = ts.params_create((-(-m // 128), -(-n // gemm.cta_tile_shape_mnk[1]), 1),
                          int(gemm.raster_order), 8, gemm.cluster_shape_mnk, gemm.is_persistent)
    want = ts.schedule(po, grid)
    res = gemm_ref.check(d.cpu(), a, b)
    assert res["ok"], res
    return got, want


@pytest.mark.parametrize("cluster", [(1, 1, 1), (2, 1, 1)])
@pytest.mark.parametrize("persistent", [True, False])
def test_tile_order_1024_matches_reference(cluster, persistent):
    """1024^3, 128x256 tiles, swizzle 8; the kernel's own tile sequence."""
    gemm = make_gemm(256, cluster, persistent)
    got, want = traced_schedule(gemm, 1024, 1024, 1024)
    assert got == want


@pytest.mark.parametrize("cluster,raster", [((1, 1, 1), RasterOrder.AlongM), ((2, 2, 1), RasterOrder.AlongN),
                                            ((1, 2, 1), RasterOrder.AlongM)])
def test_tile_order_ragged_matches_reference(cluster, raster):
    gemm = make_gemm(128, cluster, True, raster=raster)
    got, want = traced_schedule(gemm, 128 * 13 - 5, 128 * 9 + 8, 192)
    assert got == want


# ---------------------------------------------------------------- numerics
def test_gemm_1024_baseline_config():
    """M=N=K=1024, N(0,1) inputs, seed 0."""
    for cluster in ((1, 1, 1), (2, 1, 1)):
        res = run_and_check(1024, 1024, 1024, make_gemm(256, cluster))
        assert res["frob"] < 5e-3


SHAPES = [
    (128, 256, 64),       # one tile, one k-block
    (256, 512, 1024),
    (200, 136, 72),       # ragged everywhere, K tail inside one k-block
    (1, 8, 8),            # smallest legal problem
    (16, 8192, 512),      # decode-like M
    (384, 384, 1000),     # odd tile counts for CTA pairs, K tail
    (1000, 264, 4104),
    (129, 1032, 136),
]


@pytest.mark.parametrize("tile_n", [64, 128, 256])
@pytest.mark.parametrize("cluster", [(1, 1, 1), (2, 1, 1)])
@pytest.mark.parametrize("shape", SHAPES)
def test_gemm_shapes(shape, cluster, tile_n):
    m, n, k = shape
    run_and_check(m, n, k, make_gemm(tile_n, cluster), seed=hash(shape) % 1000)


@pytest.mark.parametrize("persistent,reuse_ab", [(False, True), (False, False)])
@pytest.mark.parametrize("cluster", [(1, 1, 1), (2, 1, 1), (2, 2, 1)])
def test_non_persistent(persistent, reuse_ab, cluster):
    gemm = make_gemm(256, cluster, persistent=persistent, reuse_ab=reuse_ab, stages=3)
    run_and_check(640, 1536, 320, gemm)


@pytest.mark.parametrize("stages,epi_stage", [(1, 1), (2, 2), (3, 1), (4, 4), (5, 2)])
def test_pipeline_depths(stages, epi_stage):
    gemm = make_gemm(128, (1, 1, 1), stages=stages, epi_stage=epi_stage)
    run_and_check(512, 512, 1024, gemm)


@pytest.mark.parametrize("cluster", [(1, 1, 1), (2, 1, 1)])
def test_bias_and_alpha(cluster):
    run_and_check(384, 1000, 512, make_gemm(256, cluster), bias=True)
    run_and_check(384, 1000, 512, make_gemm(128, cluster), bias=True, alpha=0.5)
    run_and_check(300, 264, 128, make_gemm(64, cluster), alpha=-2.0)


def test_empty_and_k0():
    gemm = make_gemm(256)
    for m, n in ((0, 64), (64, 0), (0, 0)):
        a = torch.empty(m, 64, dtype=torch.bfloat16, device="cuda")
        b = torch.empty(n, 64, dtype=torch.bfloat16, device="cuda")
        d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
        gemm(a, b, d)
    # K = 0: D = bias (or zeros)
    a = torch.empty(64, 0, dtype=torch.bfloat16, device="cuda")
    b = torch.empty(48, 0, dtype=torch.bfloat16, device="cuda")
    d = torch.full((64, 48), 7.0, dtype=torch.bfloat16, device="cuda")
    gemm(a, b, d)
    torch.cuda.synchronize()
    assert torch.count_nonzero(d).item() == 0
    bias = torch.randn(48, device="cuda").to(torch.bfloat16)
    gemm(a, b, d, bias=bias)
    torch.cuda.synchronize()
    assert torch.equal(d, bias.expand(64, 48))


def test_strided_operands():
    """Row strides larger than the row (views into wider buffers)."""
    m, n, k = 300, 200, 256
    a_full, b_full, _ = gemm_ref.make_inputs(m, n, k + 64, seed=3)
    a, b = a_full[:, 16:16 + k], b_full[:, 8:8 + k]
    d_full = torch.zeros(m, n + 40, dtype=torch.bfloat16, device="cuda")
    d = d_full[:, :n]
    gemm = make_gemm(128)
    gemm(a_full.cuda()[:, 16:16 + k], b_full.cuda()[:, 8:8 + k], d)
    torch.cuda.synchronize()
    res = gemm_ref.check(d.cpu(), a, b)
    assert res["ok"], res
    assert torch.count_nonzero(d_full[:, n:]).item() == 0  # nothing written outside D


def test_errors_are_reported():
    gemm = make_gemm(256)
    a = torch.randn(64, 60, device="cuda").to(torch.bfloat16)  # K = 60: row stride not 16 B
    b = torch.randn(64, 60, device="cuda").to(torch.bfloat16)
    d = torch.empty(64, 64, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.CpgError) as e:
        gemm(a, b, d)
    assert e.value.code == _lib.CPG_ERR_ALIGNMENT
    with pytest.raises(AssertionError):
        gemm(a.float(), b.float(), d.float())
    big = GemmSM90((128, 256), (128, 32), (1, 1, 1), (1, 1), ab_stage=12, reuse_ab=False,
                   is_persistent=True)
    a = torch.randn(64, 64, device="cuda").to(torch.bfloat16)
    with pytest.raises(_lib.CpgError) as e:
        big(a, a, torch.empty(64, 64, dtype=torch.bfloat16, device="cuda"))
    assert e.value.code == _lib.CPG_ERR_SMEM


def test_status_word_clear_after_runs():
    gemm = make_gemm(256, (2, 1, 1))
    a, b, _ = gemm_ref.make_inputs(512, 512, 512)
    da, db = a.cuda(), b.cuda()
    d = torch.empty(512, 512, dtype=torch.bfloat16, device="cuda")
    compiled = cpg_compile(gemm, da, db, d)
    for _ in range(3):
        compiled(da, db, d)
    assert compiled.plan_for(da, db, d).status() == 0


# ---------------------------------------------------------------- full-size configurations
def _full_size_check(m, n, k, gemm, a_scale, b_scale, bias=False, nrows=256, seed=0):
    a, b, bb = gemm_ref.make_inputs(m, n, k, seed=seed, a_scale=a_scale, b_scale=b_scale,
                                    with_bias=bias)
    da, db = a.cuda(), b.cuda()
    dbias = bb.cuda() if bb is not None else None
    d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    gemm(da, db, d, None, bias=dbias)
    torch.cuda.synchronize()
    dc = d.cpu()
    # (1) sampled rows against the fp32 oracle, element-wise and Frobenius
    g = torch.Generator().manual_seed(123)
    rows = torch.randperm(m, generator=g)[:nrows].sort().values
    res = gemm_ref.check(dc[rows], a, b, bias=bb, rows=rows)
    assert res["ok"], res
    # (2) column and row checksums over the whole output (ABFT), fp64
    ref_col = gemm_ref.column_checksum(a, b, bb)
    ref_row = gemm_ref.row_checksum(a, b, bb)
    d64 = dc.double()
    col_bound = gemm_ref.checksum_bound(d64.abs().sum(0),
                                        torch.matmul(b.double().abs(), a.double().abs().sum(0)), k, m)
    row_bound = gemm_ref.checksum_bound(d64.abs().sum(1),
                                        torch.matmul(a.double().abs(), b.double().abs().sum(0)), k, n)
    assert bool(((d64.sum(0) - ref_col).abs() <= col_bound).all())
    assert bool(((d64.sum(1) - ref_row).abs() <= row_bound).all())
    assert not bool(torch.isnan(d64).any())
    return res


@pytest.mark.slow
@pytest.mark.parametrize("cluster", [(1, 1, 1), (2, 1, 1)])
def test_full_8192_cubed(cluster):
    """8192^3, N(0,1)/sqrt(K)."""
    k = 8192
    _full_size_check(8192, 8192, k, make_gemm(256, cluster, stages=4 if cluster[0] == 1 else 6),
                     1.0, 1.0 / k ** 0.5)


@pytest.mark.slow
def test_full_llm_ffn_up_with_bias():
    """BASELINE config 3 (one GPU, one M shard of 2048 rows): N=28672, K=8192, bias."""
    _full_size_check(2048, 28672, 8192, make_gemm(256, (2, 1, 1), stages=6), 1.0, 0.02, bias=True)


# ---------------------------------------------------------------- FP8 E4M3 (per-tensor scales)
@pytest.mark.parametrize("tile_n", [128, 256])
@pytest.mark.parametrize("cluster", [(1, 1, 1), (2, 1, 1)])
@pytest.mark.parametrize("shape", [(256, 512, 512), (300, 264, 1000 + 8), (1024, 1024, 1024)])
def test_fp8_per_tensor(shape, cluster, tile_n):
    """BASELINE config 4 (per-tensor variant) at parity-test sizes; tolerance rel-Frobenius 3e-2
    and the element-wise bound, against the fp32 product of the dequantised E4M3 operands."""
    m, n, k = shape
    qa, sa, qb, sb = gemm_ref.make_fp8_inputs(m, n, k, seed=m + n + k)
    d = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    gemm = make_gemm(tile_n, cluster)
    gemm(qa.cuda(), qb.cuda(), d, None, scale_a=sa.reshape(1).cuda(), scale_b=sb.reshape(1).cuda())
    torch.cuda.synchronize()
    res = gemm_ref.check_fp8(d.cpu(), qa, sa, qb, sb)
    assert res["ok"], res
    assert res["frob"] < 1e-2


# ---------------------------------------------------------------- FP32 output (split-K partials)
@pytest.mark.parametrize("cluster", [(1, 1, 1), (2, 1, 1)])
@pytest.mark.parametrize("tile_n", [64, 256])
def test_fp32_output(cluster, tile_n):
    m, n, k = 384, 520, 768
    a, b, _ = gemm_ref.make_inputs(m, n, k, seed=11)
    d = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    gemm = make_gemm(tile_n, cluster)
    gemm(a.cuda(), b.cuda(), d)
    torch.cuda.synchronize()
    r = gemm_ref.reference(a, b)
    s = gemm_ref.abs_product(a, b)
    # fp32 output: no output rounding term, only the accumulation bound.
    assert bool(((d.cpu() - r).abs() <= k * gemm_ref.ACC_SLACK_PER_K * s + 1e-6).all())


# ---------------------------------------------------------------- FP8 E4M3 (block scales)
def _block_gemm(tile_n, cluster):
    # Deepest ring that fits 227 KiB next to 8 promotion warps' epilogue staging.
    stages, epi = {(128, 1): (5, 2), (128, 2): (8, 1), (256, 1): (4, 1),
                   (256, 2): (6, 1)}[(tile_n, cluster[0])]
    return make_gemm(tile_n, cluster, stages=stages, epi_stage=epi)


@pytest.mark.parametrize("cluster", [(1, 1, 1), (2, 1, 1)])
@pytest.mark.parametrize("tile_n", [128, 256])
@pytest.mark.parametrize("shape", [(128, 128, 128), (256, 384, 1024), (300, 264, 1000 + 8),
                                   (1024, 1024, 2048), (136, 392, 272)])
def test_fp8_block_scaled(shape, tile_n, cluster):
    """BASELINE config 4 (block variant): A scaled per 1x128, B per 128x128, against the fp32
    product of the block-dequantised operands.  N = 264 and 392 leave 256-wide edge tiles whose
    right half lies past the last scale block of B."""
    m, n, k = shape
    g = torch.Generator().manual_seed(m * 7 + n + k)
    a = torch.randn(m, k, generator=g) * torch.rand(m, 1, generator=g) * 4
    b = torch.randn(n, k, generator=g) * torch.rand(n, 1, generator=g) * 4
    qa, sa = gemm_ref.quantize_e4m3_blocks(a, (1, 128))
    qb, sb = gemm_ref.quantize_e4m3_blocks(b, (128, 128))
    bias = (torch.randn(n, generator=g) * 4).to(torch.bfloat16) if n % 2 == 0 else None
    d = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    gemm = _block_gemm(tile_n, cluster)
    gemm(qa.cuda(), qb.cuda(), d, None, scale_a=sa.cuda(), scale_b=sb.cuda(),
         bias=None if bias is None else bias.cuda())
    torch.cuda.synchronize()
    da = gemm_ref.dequantize_blocks(qa, sa, (1, 128))
    db = gemm_ref.dequantize_blocks(qb, sb, (128, 128))
    res = gemm_ref.check(d.cpu(), da, db, bias=bias, frob_tol=gemm_ref.FROB_TOL_FP8)
    assert res["ok"], res
    assert res["frob"] < 1e-2


@pytest.mark.parametrize("tile_n", [128, 256])
def test_fp8_block_scaled_many_tiles_per_cta(tile_n):
    """Persistent CTAs with several tiles each (partial-buffer phases wrap many times)."""
    m, n, k = 2048, 2048, 512
    g = torch.Generator().manual_seed(5)
    a = torch.randn(m, k, generator=g)
    b = torch.randn(n, k, generator=g)
    qa, sa = gemm_ref.quantize_e4m3_blocks(a, (1, 128))
    qb, sb = gemm_ref.quantize_e4m3_blocks(b, (128, 128))
    d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    gemm = _block_gemm(tile_n, (2, 1, 1))
    gemm(qa.cuda(), qb.cuda(), d, None, scale_a=sa.cuda(), scale_b=sb.cuda())
    torch.cuda.synchronize()
    rows = torch.arange(0, m, 7)
    res = gemm_ref.check(d.cpu()[rows], gemm_ref.dequantize_blocks(qa, sa, (1, 128)),
                         gemm_ref.dequantize_blocks(qb, sb, (128, 128)), rows=rows,
                         frob_tol=gemm_ref.FROB_TOL_FP8)
    assert res["ok"], res


def test_many_tiles_per_cta_bf16():
    """Persistent CTAs with many tiles (both TMEM accumulators reused many times)."""
    for cluster in ((1, 1, 1), (2, 1, 1)):
        run_and_check(2048, 4096, 256, make_gemm(128, cluster, stages=6))


# ---------------------------------------------------------------- split-K inside one GPU (L dim)
@pytest.mark.parametrize("cluster", [(1, 1, 1), (2, 1, 1)])
@pytest.mark.parametrize("split_k,persistent", [(2, True), (3, True), (7, True), (4, False)])
def test_split_k_fp32(split_k, persistent, cluster):
    """K cut into split_k ranges scheduled as the L dimension, partial sums added into FP32 D."""
    m, n, k = 256, 640, 64 * 21 + 8
    a, b, bias = gemm_ref.make_inputs(m, n, k, seed=split_k, with_bias=True)
    d = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    gemm = make_gemm(128, cluster, persistent=persistent)
    gemm(a.cuda(), b.cuda(), d, None, bias=bias.cuda(), split_k=split_k)
    torch.cuda.synchronize()
    r = gemm_ref.reference(a, b, bias)
    s = gemm_ref.abs_product(a, b)
    bound = k * gemm_ref.ACC_SLACK_PER_K * s + 2.0 ** -23 * bias.float().abs() + 1e-6
    assert bool(((d.cpu() - r).abs() <= bound).all())


def test_split_k_small_m_then_cast():
    """Decode-like M: split-K partial sums in FP32, then the BF16 cast kernel (with bias)."""
    from cutedsl_pingpong_gemm_b200.quant import cast_f32_bf16
    m, n, k = 64, 8192, 8192
    a, b, bias = gemm_ref.make_inputs(m, n, k, seed=9, b_scale=k ** -0.5, with_bias=True)
    d32 = torch.empty(m, n, dtype=torch.float32, device="cuda")
    gemm = make_gemm(64, (1, 1, 1), stages=8)
    gemm(a.cuda(), b.cuda(), d32, None, split_k=4)
    out = cast_f32_bf16(d32, bias.cuda())
    torch.cuda.synchronize()
    res = gemm_ref.check(out.cpu(), a, b, bias=bias)
    assert res["ok"], res


# ---------------------------------------------------------------- 512-wide tiles (two MMAs per k-step)
@pytest.mark.parametrize("cluster,stages", [((2, 1, 1), 3), ((1, 1, 1), 2), ((2, 2, 1), 3)])
@pytest.mark.parametrize("shape", [(256, 512, 128), (640, 1536, 1000), (1000, 1032, 4104),
                                   (2048, 4096, 512)])
def test_tile_n_512(shape, cluster, stages):
    m, n, k = shape
    run_and_check(m, n, k, make_gemm(512, cluster, stages=stages), seed=m + n)


def test_tile_n_512_fp8_and_bias():
    m, n, k = 1024, 2048, 1024
    qa, sa, qb, sb = gemm_ref.make_fp8_inputs(m, n, k, seed=3)
    d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    make_gemm(512, (2, 1, 1), stages=3)(qa.cuda(), qb.cuda(), d, None, scale_a=sa.reshape(1).cuda(),
                              scale_b=sb.reshape(1).cuda())
    torch.cuda.synchronize()
    assert gemm_ref.check_fp8(d.cpu(), qa, sa, qb, sb)["ok"]
    run_and_check(384, 1536, 512, make_gemm(512, (2, 1, 1), stages=3), bias=True)


def test_tile_order_512_matches_reference():
    got, want = traced_schedule(make_gemm(512, (2, 1, 1), stages=3), 128 * 9, 512 * 5 + 64, 128)
    assert got == want


@pytest.mark.parametrize("m", [16, 64, 128])
def test_small_m_auto_split_bf16(m):
    """BASELINE config 5 (decode-like M at N = K = 8192): the automatic choice (the small-M
    kernel), then the same through explicit K ranges (FP32 workspace, rounded into the BF16
    output with the bias)."""
    n, k = 8192, 8192
    a, b, bias = gemm_ref.make_inputs(m, n, k, seed=m, b_scale=k ** -0.5, with_bias=True)
    gemm = make_gemm(256, (1, 1, 1))
    d = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    compiled = cpg_compile(gemm, a.cuda(), b.cuda(), d)
    assert compiled.auto_split_k(m, n, k) == _lib.CPG_SPLIT_K_DECODE  # the small-M kernel
    compiled(a.cuda(), b.cuda(), d, None, bias=bias.cuda(), split_k=0)
    torch.cuda.synchronize()
    assert gemm_ref.check(d.cpu(), a, b, bias=bias)["ok"]
    # The same through explicit K ranges (the kernel's L dimension).
    compiled(a.cuda(), b.cuda(), d, None, bias=bias.cuda(), split_k=7)
    torch.cuda.synchronize()
    res = gemm_ref.check(d.cpu(), a, b, bias=bias)
    assert res["ok"], res


# ---------------------------------------------------------------- Stream-K
@pytest.mark.parametrize("cluster", [(1, 1, 1), (2, 1, 1)])
@pytest.mark.parametrize("shape", [(128, 8192, 8192), (64, 1024, 4096 + 64), (300, 520, 1000 + 8),
                                   (1024, 1024, 1024)])
def test_stream_k_fp32(shape, cluster):
    """Stream-K: persistent clusters split the (tile, k-block) space evenly; partial tiles add
    into FP32 D (element-wise accumulation bound only: no BF16 rounding)."""
    m, n, k = shape
    a, b, bias = gemm_ref.make_inputs(m, n, k, seed=k, b_scale=k ** -0.5, with_bias=True)
    d = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    gemm = make_gemm(256, cluster, stages=4 if cluster[0] == 1 else 6)
    gemm(a.cuda(), b.cuda(), d, None, bias=bias.cuda(), split_k=-1)
    torch.cuda.synchronize()
    r = gemm_ref.reference(a, b, bias)
    s = gemm_ref.abs_product(a, b)
    bound = k * gemm_ref.ACC_SLACK_PER_K * s + 2.0 ** -22 * bias.float().abs() + 1e-6
    assert bool(((d.cpu() - r).abs() <= bound).all())


def test_stream_k_bf16_through_api():
    m, n, k = 16, 8192, 8192
    a, b, bias = gemm_ref.make_inputs(m, n, k, seed=1, b_scale=k ** -0.5, with_bias=True)
    d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    compiled = cpg_compile(make_gemm(256, (1, 1, 1)), a.cuda(), b.cuda(), d)
    for _ in range(2):  # the workspace is reused: the second call must clear it again
        compiled(a.cuda(), b.cuda(), d, None, bias=bias.cuda(), split_k=-1)
    torch.cuda.synchronize()
    assert gemm_ref.check(d.cpu(), a, b, bias=bias)["ok"]


def test_plans_of_one_kernel_keep_their_shared_memory():
    """Plans of different shapes share one kernel function.  A plan with fewer stages created
    after one with more must not lower the function's shared-memory limit below the first plan's
    need (its launches would fail with an invalid argument)."""
    m, n, k = 512, 1024, 1024
    big = make_gemm(tile_n=256, cluster=(1, 1, 1), stages=4)
    small = make_gemm(tile_n=256, cluster=(1, 1, 1), stages=2)
    run_and_check(m, n, k, big, seed=31)
    run_and_check(m, n, k, small, seed=32)
    run_and_check(m, n, k, big, seed=33)
