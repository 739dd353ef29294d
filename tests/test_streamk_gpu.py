"""Stream-K with in-kernel fixup on the GPU against the fp32 CPU oracle.

split_k = -2 (CPG_SPLIT_K_HYBRID): all full waves but the last are computed whole and the rest of
the tiles' k-blocks are shared evenly by the resident clusters; split_k = -1 with a BF16 D: every
tile is shared.  A tile split between clusters is finished in the kernel by its last contributor
from an FP32 workspace, which it clears for the next launch (checked by repeating launches).
Tolerance as for the other GEMM tests: relative Frobenius <= 1e-2 (BF16) and the element-wise
bound 2^-8 |R| + K 2^-23 |A||B|^T.
"""
import pytest
import torch

from cutedsl_pingpong_gemm_b200 import GemmSM90, RasterOrder, _lib, compile as cpg_compile
from oracle import gemm_ref

pytestmark = pytest.mark.gpu


def make_gemm(tile_n, cluster, stages):
    return GemmSM90(tile_shape_mn=(128, tile_n), epi_tile_mn=(128, 32), cluster_shape_mnk=cluster,
                    atom_layout_mn=(1, 1), ab_stage=stages, epi_stage=2,
                    raster_order=RasterOrder.AlongN, reuse_ab=False, is_persistent=True)


CASES = [
    # (tile_n, cluster, stages, m, n, k): tiles vs resident clusters (148 single CTAs, 74 pairs)
    (128, (1, 1, 1), 6, 2560, 2560, 1024),   # 400 tiles: 148 whole, 252 shared
    (256, (1, 1, 1), 4, 1280, 2816, 640),    # 110 tiles < 148: all shared
    (512, (2, 1, 1), 3, 4096, 5120, 512),    # 160 pair tiles: 74 whole, 86 shared
    (256, (2, 1, 1), 6, 2304, 4352, 768),    # 153 pair tiles, ragged N
    (128, (1, 1, 1), 6, 1024, 4736, 256),    # 296 tiles = 2 full waves: nothing shared
]


@pytest.mark.parametrize("case", CASES)
def test_hybrid_bf16_bias_repeated(case):
    tile_n, cluster, stages, m, n, k = case
    a, b, bias = gemm_ref.make_inputs(m, n, k, seed=m + n, b_scale=k ** -0.5, with_bias=True)
    gemm = make_gemm(tile_n, cluster, stages)
    d = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    for it in range(3):  # the workspace and counts must be back to zero after every launch
        gemm(a.cuda(), b.cuda(), d, None, bias=bias.cuda(), alpha=0.75, split_k=-2)
        torch.cuda.synchronize()
        res = gemm_ref.check(d.cpu(), a, b, bias=bias, alpha=0.75)
        assert res["ok"], (it, res)
    assert gemm._compiled.plan_for(a.cuda(), b.cuda(), d, 0, -2).status() == 0


@pytest.mark.parametrize("cluster", [(1, 1, 1), (2, 1, 1)])
def test_hybrid_fp32_output(cluster):
    m, n, k = 2304, 3328, 512
    a, b, bias = gemm_ref.make_inputs(m, n, k, seed=3, b_scale=k ** -0.5, with_bias=True)
    gemm = make_gemm(256, cluster, 4 if cluster[0] == 1 else 6)
    d = torch.full((m, n), float("nan"), dtype=torch.float32, device="cuda")
    gemm(a.cuda(), b.cuda(), d, None, bias=bias.cuda(), split_k=-2)
    torch.cuda.synchronize()
    r = gemm_ref.reference(a, b, bias)
    s = gemm_ref.abs_product(a, b)
    bound = k * gemm_ref.ACC_SLACK_PER_K * s + 2.0 ** -22 * bias.float().abs() + 1e-6
    assert bool(((d.cpu() - r).abs() <= bound).all())


def test_stream_k_bf16_in_kernel_fixup_and_auto_choice():
    """Stream-K into BF16 D through the C ABI plan (the kernel finishes split tiles itself; no
    workspace of the caller, no cast kernel), and the automatic choices."""
    m, n, k = 128, 4096, 4096
    a, b, bias = gemm_ref.make_inputs(m, n, k, seed=9, b_scale=k ** -0.5, with_bias=True)
    gemm = make_gemm(128, (1, 1, 1), 6)
    da, db = a.cuda(), b.cuda()
    d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    compiled = cpg_compile(gemm, da, db, d)
    plan = compiled.plan_for(da, db, d, 0, -1)
    for _ in range(2):
        plan.run(da, db, d, None, bias=bias.cuda())
    torch.cuda.synchronize()
    res = gemm_ref.check(d.cpu(), a, b, bias=bias)
    assert res["ok"], res
    assert plan.status() == 0
    pair = make_gemm(512, (2, 1, 1), 3)
    big = cpg_compile(pair, torch.empty(256, 64, dtype=torch.bfloat16, device="cuda"),
                      torch.empty(512, 64, dtype=torch.bfloat16, device="cuda"),
                      torch.empty(256, 512, dtype=torch.bfloat16, device="cuda"))
    # A partial last wave keeps whole tiles (the hybrid is an explicit choice).
    assert big.auto_split_k(2048, 28672, 8192) == 1
    assert big.auto_split_k(8192, 8192, 8192) == 1


def test_fused_epilogue_rejects_stream_k():
    m, n, k = 256, 512, 256
    a, b, _ = gemm_ref.make_inputs(m, n, k, seed=4)
    d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.CpgError):
        make_gemm(256, (1, 1, 1), 4)(a.cuda(), b.cuda(), d, None, activation="silu", split_k=-2)


def test_split_k_bf16_on_two_streams():
    """The same split-K shape launched on two streams at once: each stream adds its partial sums
    into its own FP32 workspace, so neither output sees the other's sums."""
    m, n, k = 256, 2048, 4096
    gemm = make_gemm(256, (2, 1, 1), 6)
    inputs = [gemm_ref.make_inputs(m, n, k, seed=90 + i, b_scale=k ** -0.5) for i in range(2)]
    dev = [(a.cuda(), b.cuda()) for a, b, _ in inputs]
    outs = [torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda") for _ in range(2)]
    streams = [torch.cuda.Stream(), torch.cuda.Stream()]
    torch.cuda.synchronize()
    for it in range(3):
        for (da, db), d, s in zip(dev, outs, streams):
            with torch.cuda.stream(s):
                gemm(da, db, d, None, split_k=4)
        torch.cuda.synchronize()
        for (a, b, _), d in zip(inputs, outs):
            res = gemm_ref.check(d.cpu(), a, b)
            assert res["ok"], (it, res)
    assert len(gemm._compiled._workspaces) == 2
    gemm.release()
    assert not gemm._compiled._workspaces and not gemm._compiled._plans
    gemm(dev[0][0], dev[0][1], outs[0], None, split_k=4)  # plans again after release
    torch.cuda.synchronize()
    res = gemm_ref.check(outs[0].cpu(), inputs[0][0], inputs[0][1])
    assert res["ok"], res
