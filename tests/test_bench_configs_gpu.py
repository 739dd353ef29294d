"""Parity at full size on the exact configurations bench.py times.

Each test builds the GEMM with the bench's constructor arguments and schedule for its workload and
checks the whole output against the fp32/fp64 CPU oracle of the same seeded inputs:

* sampled rows element-wise: |D - R| <= 2^-8 |R| + K 2^-23 (|A| |B|^T) (+ bias rounding), and the
  relative Frobenius error of those rows <= 1e-2 (BF16) / 3e-2 (FP8 E4M3, against the product of
  the dequantised operands);
* fp64 column and row sums of all of D against (1^T A) B^T and A (B^T 1) (O(MK + NK) work), so no
  tile of D goes unchecked.

Workloads (bench.py --workload): bf16_8192 (256 x 512 pair tiles, 3 stages, cluster launch
control, raster group 4 at K = 8192 -- its tile order is pinned here against the reference map
with that group size), llm (16384 x 28672 x 8192 + bias), fp8 and fp8_block (16384 x 8192 x 8192),
tallk on one GPU (2048 x 2048 x 131072 through the in-GPU split), and ref_harness (the reference's
own benchmark, 65536 x 4096 x 8192 with its constructor arguments, gemm_base.py:578-609).
"""
import pytest
import torch

from cutedsl_pingpong_gemm_b200 import GemmSM90, RasterOrder, compile as cpg_compile
from cutedsl_pingpong_gemm_b200.quant import quantize_e4m3
from oracle import gemm_ref
from oracle import tile_scheduler_ref as ts

pytestmark = [pytest.mark.gpu, pytest.mark.slow]


def bench_gemm(tile_n=512, stages=3, dynamic=True, atom=(1, 1), epi_stage=2):
    """The bench's operator for the dense workloads (bench.py run_cpg)."""
    return GemmSM90(tile_shape_mn=(128, tile_n), epi_tile_mn=(128, 32), cluster_shape_mnk=(2, 1, 1),
                    atom_layout_mn=atom, ab_stage=stages, epi_stage=epi_stage,
                    raster_order=RasterOrder.AlongN, reuse_ab=False, is_persistent=True,
                    dynamic_scheduler=dynamic)


def check_whole(d, a, b, bias=None, frob_tol=gemm_ref.FROB_TOL_BF16, nrows=256, seed=123):
    """Sampled rows element-wise + fp64 column / row checksums of all of D (CPU tensors)."""
    m, k = a.shape
    n = d.shape[1]
    g = torch.Generator().manual_seed(seed)
    rows = torch.randperm(m, generator=g)[:nrows].sort().values
    res = gemm_ref.check(d[rows], a, b, bias=bias, rows=rows, frob_tol=frob_tol)
    assert res["ok"], res
    d64 = d.double()
    assert not bool(torch.isnan(d64).any())
    col_bound = gemm_ref.checksum_bound(d64.abs().sum(0),
                                        torch.mv(b.double().abs(), a.double().abs().sum(0)), k, m)
    row_bound = gemm_ref.checksum_bound(d64.abs().sum(1),
                                        torch.mv(a.double().abs(), b.double().abs().sum(0)), k, n)
    col_err = (d64.sum(0) - gemm_ref.column_checksum(a, b, bias)).abs()
    row_err = (d64.sum(1) - gemm_ref.row_checksum(a, b, bias)).abs()
    assert bool((col_err <= col_bound).all()), float((col_err / col_bound).max())
    assert bool((row_err <= row_bound).all()), float((row_err / row_bound).max())
    return res


def test_bench_bf16_8192_config_and_its_tile_order():
    """bench.py --workload bf16_8192 at full size: the numerics, and every tile once in the
    order of the reference scheduler with the plan's group size (4: a group's B panel of
    4 x 512 rows x 8192 x 2 bytes = 32 MiB stays in L2), each cluster starting on its own tile."""
    m = n = k = 8192
    a, b, _ = gemm_ref.make_inputs(m, n, k, seed=0, b_scale=k ** -0.5)
    da, db = a.cuda(), b.cuda()
    d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    gemm = bench_gemm()
    compiled = cpg_compile(gemm, da, db, d, None)
    plan = compiled.plan_for(da, db, d)
    group = plan.sched_params().dm_group_size.divisor
    assert group == 4
    grid = plan.launch_info()["grid"]
    ntm, ntn = m // 128, n // 512
    nclusters = grid[0] // 2
    assert nclusters == ntm // 2 * ntn and grid[1] == 1
    trace = torch.full((grid[0] * nclusters * 2,), -1, dtype=torch.int32, device="cuda")
    plan.set_trace(trace, nclusters)
    compiled(da, db, d, None)
    torch.cuda.synchronize()
    plan.set_trace(None, 0)
    assert plan.status() == 0
    p = ts.params_create((ntm, ntn, 1), ts.ALONG_N, 4, (2, 1, 1), True)
    t = trace.cpu().numpy().reshape(grid[0], nclusters, 2)
    seen = []
    for x in range(grid[0]):
        tiles = [tuple(map(int, e)) for e in t[x] if e[0] >= 0]
        if tiles:
            cmc, cnc = ts.map_cta_coords(p, x // 2)
            assert tiles[0] == (cmc * 2 + x % 2, cnc), (x, tiles[0])
            seen.extend(tiles)
    want = sorted((cmc * 2 + i, cnc) for cmc, cnc in ts.cluster_map(p) for i in range(2))
    assert sorted(seen) == want
    check_whole(d.cpu(), a, b)


def test_bench_llm_config_with_bias():
    """bench.py --workload llm on one GPU: 16384 x 28672 x 8192, A ~ N(0,1), B ~ N(0, 0.02),
    BF16 bias, the 512-wide pair kernel under cluster launch control."""
    m, n, k = 16384, 28672, 8192
    a, b, bias = gemm_ref.make_inputs(m, n, k, seed=0, b_scale=0.02, with_bias=True)
    d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    gemm = bench_gemm()
    gemm(a.cuda(), b.cuda(), d, None, bias=bias.cuda())
    torch.cuda.synchronize()
    check_whole(d.cpu(), a, b, bias=bias)


@pytest.mark.parametrize("scales", ["tensor", "block"])
def test_bench_fp8_configs(scales):
    """bench.py --workload fp8 / fp8_block: E4M3 16384 x 8192 x 8192, A and B ~ N(0,1)
    quantised on the GPU (s = amax / 448 per tensor, or per 1 x 128 of A and 128 x 128 of B), then
    the bench's kernel: the 512-wide pair kernel under cluster launch control (per tensor) or
    the block-scaled kernel with 256-wide pair tiles, 6 stages, the static schedule (block)."""
    m, n, k = 16384, 8192, 8192
    g = torch.Generator().manual_seed(0)
    a = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    b = torch.randn(n, k, generator=g).to(torch.bfloat16).cuda()
    d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    if scales == "tensor":
        qa, sa = quantize_e4m3(a)
        qb, sb = quantize_e4m3(b)
        gemm = bench_gemm()
    else:
        qa, sa = quantize_e4m3(a, (1, 128))
        qb, sb = quantize_e4m3(b, (128, 128))
        gemm = bench_gemm(tile_n=256, stages=6, dynamic=False, epi_stage=1)
    del a, b
    gemm(qa, qb, d, None, scale_a=sa, scale_b=sb)
    torch.cuda.synchronize()
    if scales == "tensor":
        a_deq = qa.cpu().float() * sa.cpu()
        b_deq = qb.cpu().float() * sb.cpu()
    else:
        a_deq = gemm_ref.dequantize_blocks(qa.cpu(), sa.cpu(), (1, 128))
        b_deq = gemm_ref.dequantize_blocks(qb.cpu(), sb.cpu(), (128, 128))
    res = check_whole(d.cpu(), a_deq, b_deq, frob_tol=gemm_ref.FROB_TOL_FP8)
    assert res["frob"] < 1e-2


def test_bench_tallk_config_on_one_gpu():
    """bench.py --workload tallk at one GPU: 2048 x 2048 x 131072, the K range split inside the GPU
    (auto_split_k) into FP32 partials summed by TMA reduce-add, then the BF16 cast; 256-wide pair
    tiles, 6 stages, cluster launch control.  Small enough to check every element."""
    from cutedsl_pingpong_gemm_b200.sharding import SplitKGemm
    m, n, k = 2048, 2048, 131072
    a, b, _ = gemm_ref.make_inputs(m, n, k, seed=0, b_scale=k ** -0.5)
    gemm = bench_gemm(tile_n=256, stages=6)
    sk = SplitKGemm.on_gpu(gemm, 1, 0, local_split_k=0)
    out = sk(a.cuda(), b.cuda(), m, n)
    torch.cuda.synchronize()
    gemm_ref.set_threads()
    res = gemm_ref.check(out.cpu(), a, b)
    assert res["ok"], res


def test_reference_harness_config():
    """The reference's own benchmark: 65536 x 4096 x 8192 BF16, A and B ~ N(0,1), with its
    constructor arguments (tile (128, 256), epi (128, 32), cluster (2, 1, 1), atom (2, 1),
    ab_stage=3, reuse_ab=False, is_persistent=True; gemm_base.py:578-609)."""
    m, n, k = 65536, 4096, 8192
    a, b, _ = gemm_ref.make_inputs(m, n, k, seed=0)
    gemm = GemmSM90(tile_shape_mn=(128, 256), epi_tile_mn=(128, 32), cluster_shape_mnk=(2, 1, 1),
                    atom_layout_mn=(2, 1), ab_stage=3, reuse_ab=False, is_persistent=True)
    da, db = a.cuda(), b.cuda()
    d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    compiled = cpg_compile(gemm, da, db, d, None)
    compiled(da, db, d, None)
    torch.cuda.synchronize()
    check_whole(d.cpu(), a, b)
