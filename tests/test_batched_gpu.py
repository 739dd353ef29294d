"""Batched GEMM (the L mode) on the GPU against the fp32 CPU oracle, batch by batch.

The reference's tensors are (M, K, L) but its kernel fixes L at one (gemm_base.py:221,
tile_scheduler.py:96); here the scheduler's L index runs over batches (x split-K ranges) and
every batch must match its own 2-D product.  Tolerance as for the 2-D tests: relative
Frobenius error <= 1e-2 and |D - R| <= 2^-8 |R| + K 2^-23 |A||B|^T per element.
"""
import pytest
import torch

from cutedsl_pingpong_gemm_b200 import GemmSM90, RasterOrder, _lib
from cutedsl_pingpong_gemm_b200.quant import quantize_e4m3
from oracle import gemm_ref

pytestmark = pytest.mark.gpu


def make_gemm(tile_n=256, cluster=(1, 1, 1), stages=4, persistent=True):
    return GemmSM90(tile_shape_mn=(128, tile_n), epi_tile_mn=(128, 32), cluster_shape_mnk=cluster,
                    atom_layout_mn=(1, 1), ab_stage=stages, epi_stage=2,
                    raster_order=RasterOrder.AlongN, reuse_ab=False, is_persistent=persistent)


def batched_inputs(l, m, n, k, seed, b_rows=None):
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(l, m, k, generator=g).to(torch.bfloat16)
    b = (torch.randn(l, b_rows or n, k, generator=g) * k ** -0.5).to(torch.bfloat16)
    return a, b


def check_batches(d, a, b, **kw):
    for i in range(a.shape[0]):
        res = gemm_ref.check(d[i].cpu(), a[i], b[i], **kw)
        assert res["ok"], (i, res)


@pytest.mark.parametrize("tile_n,cluster", [(128, (1, 1, 1)), (256, (2, 1, 1)),
                                            (512, (2, 1, 1))])
@pytest.mark.parametrize("persistent", [True, False])
def test_batched_contiguous(tile_n, cluster, persistent):
    l, m, n, k = 3, 300, 392, 320
    a, b = batched_inputs(l, m, n, k, seed=41)
    d = torch.full((l, m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    gemm = make_gemm(tile_n, cluster, stages=3 if tile_n == 512 else 4, persistent=persistent)
    gemm(a.cuda(), b.cuda(), d, None)
    torch.cuda.synchronize()
    check_batches(d, a, b)


def test_batched_strided_views_and_bias():
    """Batches that are slices of larger buffers (batch strides > rows * row stride)."""
    l, m, n, k = 4, 200, 264, 136
    g = torch.Generator().manual_seed(42)
    a_big = torch.randn(l, m + 56, k + 64, generator=g).to(torch.bfloat16)
    b_big = (torch.randn(l, n + 8, k + 64, generator=g) * 0.1).to(torch.bfloat16)
    bias = torch.randn(n, generator=g).to(torch.bfloat16)
    a, b = a_big[:, :m, :k], b_big[:, :n, :k]
    d_big = torch.full((l, m + 8, n + 8), float("nan"), dtype=torch.bfloat16, device="cuda")
    d = d_big[:, :m, :n]
    gemm = make_gemm(128, (2, 1, 1))
    gemm(a_big.cuda()[:, :m, :k], b_big.cuda()[:, :n, :k], d, None, bias=bias.cuda(), alpha=0.5)
    torch.cuda.synchronize()
    check_batches(d, a, b, bias=bias, alpha=0.5)
    assert torch.isnan(d_big[:, m:, :].float()).all() and torch.isnan(d_big[:, :, n:].float()).all()


@pytest.mark.parametrize("split_k", [3, -1])
def test_batched_split_k_fp32_and_bf16(split_k):
    """Split-K / Stream-K: the L index carries batch x K range."""
    l, m, n, k = 3, 128, 256, 2048
    a, b = batched_inputs(l, m, n, k, seed=43)
    gemm = make_gemm(128, (1, 1, 1), stages=6)
    d32 = torch.empty(l, m, n, dtype=torch.float32, device="cuda")
    gemm(a.cuda(), b.cuda(), d32, None, split_k=split_k)
    torch.cuda.synchronize()
    for i in range(l):
        r = gemm_ref.reference(a[i], b[i])
        s = gemm_ref.abs_product(a[i], b[i])
        assert bool(((d32[i].cpu() - r).abs() <= k * gemm_ref.ACC_SLACK_PER_K * s + 1e-6).all()), i
    d16 = torch.empty(l, m, n, dtype=torch.bfloat16, device="cuda")
    gemm(a.cuda(), b.cuda(), d16, None, split_k=split_k)
    torch.cuda.synchronize()
    check_batches(d16, a, b)


def test_batched_small_m_auto_stream_k():
    l, m, n, k = 4, 64, 1024, 4096
    a, b = batched_inputs(l, m, n, k, seed=44)
    d = torch.empty(l, m, n, dtype=torch.bfloat16, device="cuda")
    gemm = make_gemm(128, (1, 1, 1), stages=6)
    gemm(a.cuda(), b.cuda(), d, None, split_k=0)
    torch.cuda.synchronize()
    check_batches(d, a, b)


def test_batched_fused_epilogue_and_gated():
    l, m, n, k = 2, 256, 384, 512
    a, b = batched_inputs(l, m, n, k, seed=45)
    g = torch.Generator().manual_seed(46)
    c = torch.randn(l, m, n, generator=g).to(torch.bfloat16)
    bias = torch.randn(n, generator=g).to(torch.bfloat16)
    d = torch.empty(l, m, n, dtype=torch.bfloat16, device="cuda")
    gemm = make_gemm(256, (2, 1, 1))
    gemm(a.cuda(), b.cuda(), d, None, bias=bias.cuda(), source=c.cuda(), beta=0.25,
         activation="gelu_tanh")
    torch.cuda.synchronize()
    for i in range(l):
        res = gemm_ref.check_epilogue(d[i].cpu(), a[i], b[i], bias=bias, beta=0.25, c=c[i],
                                      act="gelu_tanh")
        assert res["ok"], (i, res)
    ab, bb = batched_inputs(l, m, n, k, seed=47, b_rows=2 * n)
    dg = torch.empty(l, m, n, dtype=torch.bfloat16, device="cuda")
    make_gemm(512, (2, 1, 1), stages=3)(ab.cuda(), bb.cuda(), dg, None, gated=True,
                                        activation="silu")
    torch.cuda.synchronize()
    for i in range(l):
        res = gemm_ref.check_gated(dg[i].cpu(), ab[i], bb[i], act="silu")
        assert res["ok"], (i, res)


def test_batched_fp8_per_tensor():
    l, m, n, k = 2, 384, 512, 1024
    g = torch.Generator().manual_seed(48)
    a = torch.randn(l, m, k, generator=g)
    b = torch.randn(l, n, k, generator=g)
    qa, sa = quantize_e4m3(a.reshape(l * m, k).cuda())
    qb, sb = quantize_e4m3(b.reshape(l * n, k).cuda())
    d = torch.empty(l, m, n, dtype=torch.bfloat16, device="cuda")
    make_gemm(512, (2, 1, 1), stages=3)(qa.view(l, m, k), qb.view(l, n, k), d, None,
                                        scale_a=sa, scale_b=sb)
    torch.cuda.synchronize()
    da = (qa.cpu().float() * sa.cpu()).view(l, m, k)
    db = (qb.cpu().float() * sb.cpu()).view(l, n, k)
    for i in range(l):
        res = gemm_ref.check(d[i].cpu(), da[i], db[i], frob_tol=gemm_ref.FROB_TOL_FP8)
        assert res["ok"], (i, res)


def test_batched_single_and_empty():
    m, n, k = 256, 256, 256
    a, b = batched_inputs(1, m, n, k, seed=49)
    d3 = torch.empty(1, m, n, dtype=torch.bfloat16, device="cuda")
    d2 = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    gemm = make_gemm(256, (1, 1, 1))
    gemm(a.cuda(), b.cuda(), d3, None)
    gemm(a[0].cuda(), b[0].cuda(), d2, None)
    torch.cuda.synchronize()
    assert torch.equal(d3[0], d2)
    e = torch.empty(0, m, n, dtype=torch.bfloat16, device="cuda")
    gemm(torch.empty(0, m, k, dtype=torch.bfloat16, device="cuda"),
         torch.empty(0, n, k, dtype=torch.bfloat16, device="cuda"), e, None)


def test_batched_rejections():
    l, m, n, k = 2, 256, 256, 256
    a, b = batched_inputs(l, m, n, k, seed=50)
    a, b = a.cuda(), b.cuda()
    d = torch.empty(l, m, n, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.CpgError):  # batch counts differ
        make_gemm()(a, b[:1], d[:1], None)
    with pytest.raises(_lib.CpgError):  # mixed 2-D / 3-D
        make_gemm()(a[0], b, d, None)
    with pytest.raises(_lib.CpgError):  # D batches overlap
        over = torch.empty(m * n + n, dtype=torch.bfloat16, device="cuda").as_strided(
            (l, m, n), (n, n, 1))
        make_gemm()(a, b, over, None)
    qa, sa = quantize_e4m3(a.reshape(l * m, k), (1, 128))
    qb, sb = quantize_e4m3(b.reshape(l * n, k), (128, 128))
    with pytest.raises(_lib.CpgError):  # batched block-scaled FP8 is not implemented
        make_gemm(128, (1, 1, 1))(qa.view(l, m, k), qb.view(l, n, k), d, None, scale_a=sa,
                                  scale_b=sb)
