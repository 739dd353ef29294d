"""Grouped GEMM (ragged groups, MoE-style) on the GPU against the fp32 CPU oracle, group by group.

The reference has no grouped form (its kernel fixes the L mode at one, gemm_base.py:221); the
spec is cpgemm.h's cpg_gemm_run_grouped: for every group g, D[r] = epilogue(A[r] . B[g]^T) for
group_offsets[g] <= r < group_offsets[g + 1], rows outside every group untouched.  Tolerance as
for the 2-D tests (relative Frobenius <= 1e-2, element-wise 2^-8 |R| + K 2^-23 |A||B|^T).
"""
import pytest
import torch

from cutedsl_pingpong_gemm_b200 import GemmSM90, RasterOrder, _lib
from cutedsl_pingpong_gemm_b200.quant import quantize_e4m3
from oracle import gemm_ref

pytestmark = pytest.mark.gpu


def make_gemm(tile_n=256, cluster=(1, 1, 1), stages=4):
    return GemmSM90(tile_shape_mn=(128, tile_n), epi_tile_mn=(128, 32), cluster_shape_mnk=cluster,
                    atom_layout_mn=(1, 1), ab_stage=stages, epi_stage=2,
                    raster_order=RasterOrder.AlongN, reuse_ab=False, is_persistent=True)


def offsets_of(sizes, start=0):
    off = [start]
    for s in sizes:
        off.append(off[-1] + s)
    return off


def grouped_inputs(sizes, n, k, seed, start=0, tail=0, b_rows=None):
    g = torch.Generator().manual_seed(seed)
    t = start + sum(sizes) + tail
    a = torch.randn(t, k, generator=g).to(torch.bfloat16)
    b = (torch.randn(len(sizes), b_rows or n, k, generator=g) * k ** -0.5).to(torch.bfloat16)
    return a, b, offsets_of(sizes, start)


def check_groups(d, a, b, off, checker=gemm_ref.check, **kw):
    for gi in range(len(off) - 1):
        s, e = off[gi], off[gi + 1]
        if e > s:
            res = checker(d[s:e].cpu(), a[s:e], b[gi], **kw)
            assert res["ok"], (gi, s, e, res)


SIZES = [0, 37, 128, 300, 1, 0, 513, 256, 90]


@pytest.mark.parametrize("tile_n,cluster", [(128, (1, 1, 1)), (256, (2, 1, 1)),
                                            (512, (2, 1, 1))])
def test_grouped_ragged(tile_n, cluster):
    n, k = 392, 320
    a, b, off = grouped_inputs(SIZES, n, k, seed=61, start=16, tail=40)
    t = a.shape[0]
    d = torch.full((t, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    gemm = make_gemm(tile_n, cluster, stages=3 if tile_n == 512 else 4)
    gemm.grouped(a.cuda(), b.cuda(), d, torch.tensor(off, dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    check_groups(d, a, b, off)
    # Rows before the first and after the last group are not written.
    assert torch.isnan(d[:off[0]].float()).all() and torch.isnan(d[off[-1]:].float()).all()


def test_grouped_many_groups_and_repeat():
    """Many small groups (the prefix kernel's runs of several groups per thread) and a second
    launch with different offsets on the same plan."""
    g = torch.Generator().manual_seed(62)
    sizes = torch.randint(0, 60, (1500,), generator=g).tolist()
    n, k = 256, 128
    a, b, off = grouped_inputs(sizes, n, k, seed=63)
    d = torch.empty(a.shape[0], n, dtype=torch.bfloat16, device="cuda")
    gemm = make_gemm(256, (1, 1, 1))
    gemm.grouped(a.cuda(), b.cuda(), d, torch.tensor(off, dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    check_groups(d, a, b, off)
    sizes2 = sizes[::-1]
    off2 = offsets_of(sizes2)
    gemm.grouped(a.cuda(), b.cuda(), d, torch.tensor(off2, dtype=torch.int32, device="cuda"))
    torch.cuda.synchronize()
    check_groups(d, a, b, off2)


def test_grouped_fused_epilogue_fp32_and_gated():
    sizes = [200, 0, 129, 384]
    n, k = 264, 256
    a, b, off = grouped_inputs(sizes, n, k, seed=64)
    g = torch.Generator().manual_seed(65)
    bias = torch.randn(n, generator=g).to(torch.bfloat16)
    offs = torch.tensor(off, dtype=torch.int32, device="cuda")
    d = torch.empty(a.shape[0], n, dtype=torch.bfloat16, device="cuda")
    make_gemm(256, (2, 1, 1)).grouped(a.cuda(), b.cuda(), d, offs, bias=bias.cuda(),
                                      activation="silu", alpha=0.5)
    torch.cuda.synchronize()
    for gi in range(len(sizes)):
        s, e = off[gi], off[gi + 1]
        if e > s:
            res = gemm_ref.check_epilogue(d[s:e].cpu(), a[s:e], b[gi], bias=bias, alpha=0.5,
                                          act="silu")
            assert res["ok"], (gi, res)
    d32 = torch.empty(a.shape[0], n, dtype=torch.float32, device="cuda")
    make_gemm(128, (1, 1, 1)).grouped(a.cuda(), b.cuda(), d32, offs)
    torch.cuda.synchronize()
    for gi in range(len(sizes)):
        s, e = off[gi], off[gi + 1]
        if e > s:
            r = gemm_ref.reference(a[s:e], b[gi])
            sabs = gemm_ref.abs_product(a[s:e], b[gi])
            assert bool(((d32[s:e].cpu() - r).abs() <= k * gemm_ref.ACC_SLACK_PER_K * sabs
                         + 1e-6).all()), gi
    ag, bg, offg = grouped_inputs(sizes, n, k, seed=66, b_rows=2 * n)
    dg = torch.empty(ag.shape[0], n, dtype=torch.bfloat16, device="cuda")
    make_gemm(512, (2, 1, 1), stages=3).grouped(
        ag.cuda(), bg.cuda(), dg, torch.tensor(offg, dtype=torch.int32, device="cuda"),
        activation="silu", gated=True)
    torch.cuda.synchronize()
    for gi in range(len(sizes)):
        s, e = offg[gi], offg[gi + 1]
        if e > s:
            res = gemm_ref.check_gated(dg[s:e].cpu(), ag[s:e], bg[gi], act="silu")
            assert res["ok"], (gi, res)


def test_grouped_fp8_per_tensor():
    sizes = [300, 17, 640]
    n, k = 512, 512
    g = torch.Generator().manual_seed(67)
    a = torch.randn(sum(sizes), k, generator=g)
    b = torch.randn(len(sizes) * n, k, generator=g)
    qa, sa = quantize_e4m3(a.cuda())
    qb, sb = quantize_e4m3(b.cuda())
    off = offsets_of(sizes)
    d = torch.empty(sum(sizes), n, dtype=torch.bfloat16, device="cuda")
    make_gemm(512, (2, 1, 1), stages=3).grouped(
        qa, qb.view(len(sizes), n, k), d, torch.tensor(off, dtype=torch.int32, device="cuda"),
        scale_a=sa, scale_b=sb)
    torch.cuda.synchronize()
    da = qa.cpu().float() * sa.cpu()
    db = (qb.cpu().float() * sb.cpu()).view(len(sizes), n, k)
    check_groups(d, da, db, off, frob_tol=gemm_ref.FROB_TOL_FP8)


def test_grouped_bad_offsets_report_status():
    """Offsets that decrease or pass T empty their groups and set the plan's status (0x200);
    the kernel reads nothing out of range for them."""
    n, k = 256, 128
    a, b, _ = grouped_inputs([256, 256], n, k, seed=68)
    d = torch.zeros(512, n, dtype=torch.bfloat16, device="cuda")
    gemm = make_gemm(256, (1, 1, 1))
    bad = torch.tensor([0, 300, 200], dtype=torch.int32, device="cuda")
    gemm.grouped(a.cuda(), b.cuda(), d, bad)
    torch.cuda.synchronize()
    plan = gemm._compiled._grouped_plan(a.cuda(), b.cuda(), d, False)
    with pytest.raises(_lib.CpgError):
        plan.status()
    # The plan stays usable with valid offsets afterwards.
    good = torch.tensor([0, 256, 512], dtype=torch.int32, device="cuda")
    gemm.grouped(a.cuda(), b.cuda(), d, good)
    torch.cuda.synchronize()
    assert plan.status() == 0
    check_groups(d, a, b, [0, 256, 512])


def test_grouped_rejections():
    n, k = 256, 128
    a, b, off = grouped_inputs([128, 128], n, k, seed=69)
    offs = torch.tensor(off, dtype=torch.int32, device="cuda")
    d = torch.empty(256, n, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.CpgError):  # offsets of the wrong length
        make_gemm().grouped(a.cuda(), b.cuda(), d, offs[:2])
    with pytest.raises(_lib.CpgError):  # int64 offsets
        make_gemm().grouped(a.cuda(), b.cuda(), d, offs.long())
    nonpersist = GemmSM90(tile_shape_mn=(128, 256), epi_tile_mn=(128, 32),
                          cluster_shape_mnk=(1, 1, 1), atom_layout_mn=(1, 1), ab_stage=4,
                          epi_stage=2, raster_order=RasterOrder.AlongN, reuse_ab=False,
                          is_persistent=False)
    with pytest.raises(_lib.CpgError):  # needs a persistent kernel
        nonpersist.grouped(a.cuda(), b.cuda(), d, offs)
