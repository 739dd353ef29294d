"""Dynamic scheduling (cluster launch control) on the GPU, through the public API / C ABI.

The reference has only the static schedule (tile_scheduler.py:94-183); the dynamic mode keeps its
linear-id -> tile map (map_cta_coords) but lets running clusters take over clusters of the grid
that have not started.  Checked here: the numerics against the fp32 CPU oracle (relative
Frobenius <= 1e-2 and the element-wise bound of oracle.gemm_ref.check), that the device trace
covers every tile exactly once with tiles of the reference map, that each cluster starts with its
own tile, and that clusters were in fact taken over (fewer CTAs ran tiles than the grid holds).
"""
import pytest
import torch

from cutedsl_pingpong_gemm_b200 import GemmSM90, RasterOrder, _lib, compile as cpg_compile
from cutedsl_pingpong_gemm_b200.quant import quantize_e4m3
from oracle import gemm_ref
from oracle import tile_scheduler_ref as ts

pytestmark = pytest.mark.gpu


def make_gemm(tile_n=256, cluster=(1, 1, 1), stages=4, raster=RasterOrder.AlongN,
              persistent=True):
    return GemmSM90(tile_shape_mn=(128, tile_n), epi_tile_mn=(128, 32), cluster_shape_mnk=cluster,
                    atom_layout_mn=(1, 1), ab_stage=stages, epi_stage=2, raster_order=raster,
                    reuse_ab=False, is_persistent=persistent, dynamic_scheduler=True)


CONFIGS = [(128, (1, 1, 1)), (256, (2, 1, 1)), (512, (2, 1, 1)), (128, (1, 2, 1)),
           (256, (2, 2, 1))]


@pytest.mark.parametrize("tile_n,cluster", CONFIGS)
def test_dynamic_tiles_once_and_numerics(tile_n, cluster):
    m, n, k = 128 * 24 - 40, 4096 + 72, 320
    gemm = make_gemm(tile_n, cluster, stages=3 if tile_n == 512 else 4)
    a, b, _ = gemm_ref.make_inputs(m, n, k, seed=71, b_scale=k ** -0.5)
    da, db = a.cuda(), b.cuda()
    d = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    compiled = cpg_compile(gemm, da, db, d, None)
    plan = compiled.plan_for(da, db, d)
    grid = plan.launch_info()["grid"]
    cm, cn = cluster[0], cluster[1]
    ntm, ntn = -(-m // 128), -(-n // tile_n)
    # The plan's group size (the dynamic schedule may lower the reference's 8 for long K).
    group = plan.sched_params().dm_group_size.divisor
    p = ts.params_create((ntm, ntn, 1), int(gemm.raster_order), group, cluster, True)
    nclusters = grid[0] // cm
    assert grid[1] == cn and grid[2] == 1
    nctas = grid[0] * grid[1]
    per_cta = nclusters
    trace = torch.full((nctas * per_cta * 2,), -1, dtype=torch.int32, device="cuda")
    plan.set_trace(trace, per_cta)
    compiled(da, db, d, None)
    torch.cuda.synchronize()
    plan.set_trace(None, 0)
    assert plan.status() == 0
    res = gemm_ref.check(d.cpu(), a, b)
    assert res["ok"], res
    t = trace.cpu().numpy().reshape(grid[1], grid[0], per_cta, 2)
    seen = []
    ran = 0
    for y in range(grid[1]):
        for x in range(grid[0]):
            tiles = [tuple(map(int, e)) for e in t[y, x] if e[0] >= 0]
            if not tiles:
                continue
            ran += 1
            # A cluster starts with its own tile: cluster id x // cm through the reference map.
            cmc, cnc = ts.map_cta_coords(p, x // cm)
            assert tiles[0] == (cmc * cm + x % cm, cnc * cn + y), (x, y, tiles[0])
            seen.extend(tiles)
    want = sorted((cmc * cm + i, cnc * cn + j) for cmc, cnc in ts.cluster_map(p)
                  for i in range(cm) for j in range(cn))
    assert sorted(seen) == want
    assert ran < nctas, "no cluster was taken over"


def test_dynamic_matches_static_bitwise():
    """Same tiles, same k order: the dynamic and the static schedule give identical bytes."""
    m, n, k = 2048, 3072, 1024
    a, b, bias = gemm_ref.make_inputs(m, n, k, seed=72, b_scale=k ** -0.5, with_bias=True)
    da, db, dbias = a.cuda(), b.cuda(), bias.cuda()
    outs = []
    for dyn in (False, True):
        gemm = GemmSM90(tile_shape_mn=(128, 512), epi_tile_mn=(128, 32),
                        cluster_shape_mnk=(2, 1, 1), atom_layout_mn=(1, 1), ab_stage=3,
                        epi_stage=2, raster_order=RasterOrder.AlongN, reuse_ab=False,
                        is_persistent=True, dynamic_scheduler=dyn)
        d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
        gemm(da, db, d, None, bias=dbias, activation="gelu")
        outs.append(d)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
    res = gemm_ref.check_epilogue(outs[1].cpu(), a, b, bias=bias, act="gelu")
    assert res["ok"], res


def test_dynamic_batched_split_k_fp32():
    l, m, n, k = 3, 256, 512, 2048
    g = torch.Generator().manual_seed(73)
    a = torch.randn(l, m, k, generator=g).to(torch.bfloat16)
    b = (torch.randn(l, n, k, generator=g) * k ** -0.5).to(torch.bfloat16)
    d = torch.empty(l, m, n, dtype=torch.float32, device="cuda")
    make_gemm(128, (1, 1, 1), stages=6)(a.cuda(), b.cuda(), d, None, split_k=4)
    torch.cuda.synchronize()
    for i in range(l):
        r = gemm_ref.reference(a[i], b[i])
        s = gemm_ref.abs_product(a[i], b[i])
        assert bool(((d[i].cpu() - r).abs() <= k * gemm_ref.ACC_SLACK_PER_K * s + 1e-6).all()), i


def test_dynamic_grouped_skips_empty_clusters():
    """The grid holds the grouped GEMM's tile bound; clusters past the real tiles end at once and
    cancelled ones are skipped."""
    sizes = [0, 300, 17, 640, 0, 129, 1000]
    n, k = 520, 256
    g = torch.Generator().manual_seed(74)
    t = sum(sizes)
    a = torch.randn(t, k, generator=g).to(torch.bfloat16)
    b = (torch.randn(len(sizes), n, k, generator=g) * k ** -0.5).to(torch.bfloat16)
    off = [0]
    for s in sizes:
        off.append(off[-1] + s)
    d = torch.empty(t, n, dtype=torch.bfloat16, device="cuda")
    gemm = make_gemm(256, (2, 1, 1))
    gemm.grouped(a.cuda(), b.cuda(), d, torch.tensor(off, dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    for gi in range(len(sizes)):
        s, e = off[gi], off[gi + 1]
        if e > s:
            res = gemm_ref.check(d[s:e].cpu(), a[s:e], b[gi])
            assert res["ok"], (gi, res)


def test_dynamic_fp8_per_tensor():
    m, n, k = 1024, 2048, 1024
    g = torch.Generator().manual_seed(75)
    qa, sa = quantize_e4m3(torch.randn(m, k, generator=g).cuda())
    qb, sb = quantize_e4m3(torch.randn(n, k, generator=g).cuda())
    d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    make_gemm(512, (2, 1, 1), stages=3)(qa, qb, d, None, scale_a=sa, scale_b=sb)
    torch.cuda.synchronize()
    res = gemm_ref.check(d.cpu(), qa.cpu().float() * sa.cpu(), qb.cpu().float() * sb.cpu(),
                         frob_tol=gemm_ref.FROB_TOL_FP8)
    assert res["ok"], res


def test_dynamic_repeated_launches_and_side_stream():
    """Back-to-back launches, one of them beside a kernel on another stream that holds SMs."""
    m, n, k = 4096, 4096, 2048
    a, b, _ = gemm_ref.make_inputs(m, n, k, seed=76, b_scale=k ** -0.5)
    da, db = a.cuda(), b.cuda()
    gemm = make_gemm(512, (2, 1, 1), stages=3)
    ref = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    gemm(da, db, ref, None)
    side = torch.cuda.Stream()
    x = torch.randn(8192, 8192, device="cuda")
    for i in range(4):
        d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
        if i == 2:
            with torch.cuda.stream(side):
                x @ x
        gemm(da, db, d, None)
        torch.cuda.synchronize()
        assert torch.equal(d, ref), i
    res = gemm_ref.check(ref.cpu(), a, b)
    assert res["ok"], res


def test_dynamic_rejections():
    m, n, k = 256, 256, 256
    a, b, _ = gemm_ref.make_inputs(m, n, k, seed=77)
    a, b = a.cuda(), b.cuda()
    d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(AssertionError):  # reuse_ab needs one tile per CTA
        GemmSM90(tile_shape_mn=(128, 256), epi_tile_mn=(128, 32), cluster_shape_mnk=(1, 1, 1),
                 atom_layout_mn=(1, 1), reuse_ab=True, is_persistent=False,
                 dynamic_scheduler=True)
    with pytest.raises(_lib.CpgError):  # Stream-K partitions the k-blocks statically
        make_gemm(256)(a, b, d, None, split_k=-1)


@pytest.mark.parametrize("tile_n,cluster,stages,epi", [(128, (1, 1, 1), 5, 2),
                                                       (256, (2, 1, 1), 6, 1)])
def test_dynamic_fp8_block_scales(tile_n, cluster, stages, epi):
    """The block-scaled FP8 kernel under the dynamic schedule: identical bytes to the static one
    and within the FP8 tolerance of the dequantised oracle."""
    m, n, k = 2048 + 128, 3072 - 64, 1024
    g = torch.Generator().manual_seed(78)
    qa, sa = quantize_e4m3(torch.randn(m, k, generator=g).cuda(), (1, 128))
    qb, sb = quantize_e4m3(torch.randn(n, k, generator=g).cuda(), (128, 128))
    outs = []
    for dyn in (False, True):
        gemm = GemmSM90(tile_shape_mn=(128, tile_n), epi_tile_mn=(128, 32),
                        cluster_shape_mnk=cluster, atom_layout_mn=(1, 1), ab_stage=stages,
                        epi_stage=epi, raster_order=RasterOrder.AlongN, reuse_ab=False,
                        is_persistent=True, dynamic_scheduler=dyn)
        d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
        gemm(qa, qb, d, None, scale_a=sa, scale_b=sb)
        outs.append(d)
    torch.cuda.synchronize()
    assert torch.equal(outs[0], outs[1])
    da = gemm_ref.dequantize_blocks(qa.cpu(), sa.cpu(), (1, 128))
    db = gemm_ref.dequantize_blocks(qb.cpu(), sb.cpu(), (128, 128))
    res = gemm_ref.check(outs[1].cpu(), da, db, frob_tol=gemm_ref.FROB_TOL_FP8)
    assert res["ok"], res


def test_dynamic_in_cuda_graph():
    """A dynamic-schedule GEMM captured into a CUDA graph and replayed: each replay cancels
    clusters of its own launch."""
    m, n, k = 1024, 4096, 1024
    a, b, _ = gemm_ref.make_inputs(m, n, k, seed=79, b_scale=k ** -0.5)
    da, db = a.cuda(), b.cuda()
    d = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
    gemm = make_gemm(256, (2, 1, 1))
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        gemm(da, db, d, None)  # plan and tensor maps built before capture
    torch.cuda.synchronize()
    ref = d.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        gemm(da, db, d, None)
    for _ in range(3):
        d.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(d, ref)
    res = gemm_ref.check(ref.cpu(), a, b)
    assert res["ok"], res


@pytest.mark.parametrize("dtype,k,dynamic,want", [
    (torch.bfloat16, 8192, True, 4),         # B panel of a cluster column: 512 x 8192 x 2 = 8 MiB
    (torch.float8_e4m3fn, 8192, True, 8),    # 4 MiB per column: the reference's 8
    (torch.bfloat16, 16384, True, 2),
    (torch.bfloat16, 8192, False, 8),        # static schedule: always the reference's 8
    (torch.bfloat16, 320, True, 8),
])
def test_dynamic_group_size_keeps_the_panel_in_l2(dtype, k, dynamic, want):
    """The dynamic schedule lowers the group size until the B rows of a group's cluster columns
    over one K range take at most 32 MiB (256 x 512 pair tiles: 512 rows of B per column)."""
    m, n = 256, 512 * 12
    gemm = GemmSM90(tile_shape_mn=(128, 512), epi_tile_mn=(128, 32), cluster_shape_mnk=(2, 1, 1),
                    atom_layout_mn=(1, 1), ab_stage=3, reuse_ab=False, is_persistent=True,
                    dynamic_scheduler=dynamic)
    a = torch.empty(m, k, dtype=dtype, device="cuda")
    b = torch.empty(n, k, dtype=dtype, device="cuda")
    d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    plan = cpg_compile(gemm, a, b, d, None).plan_for(a, b, d)
    assert plan.sched_params().dm_group_size.divisor == want
