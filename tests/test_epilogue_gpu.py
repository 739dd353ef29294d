"""Fused epilogue on the GPU through the public API / C ABI, against the fp32 CPU oracle.

D = act(alpha * A . B^T + bias + beta * C) and the gated form D = act(alpha A Wg^T) * alpha A Wu^T
with B = [Wg; Wu].  The reference kernel has no epilogue options (gemm_base.py:133); the spec is
that of cpgemm.h.  Tolerance: relative Frobenius error <= 1e-2 (BF16 D) and the element-wise bound
of oracle.gemm_ref.check_epilogue / check_gated: BF16 rounding of D (2^-8 relative), the fp32
accumulation bound K * 2^-23 * |A| |B|^T through the activation's slope (<= 1.13), and 2^-18
relative for the device's exp / erf / tanh.
"""
import pytest
import torch

from cutedsl_pingpong_gemm_b200 import GemmSM90, RasterOrder, _lib
from cutedsl_pingpong_gemm_b200.quant import quantize_e4m3
from oracle import gemm_ref

pytestmark = pytest.mark.gpu

ACTS = ["relu", "silu", "gelu", "gelu_tanh"]


def make_gemm(tile_n, cluster, stages=4):
    return GemmSM90(tile_shape_mn=(128, tile_n), epi_tile_mn=(128, 32), cluster_shape_mnk=cluster,
                    atom_layout_mn=(1, 1), ab_stage=stages, epi_stage=2,
                    raster_order=RasterOrder.AlongN, reuse_ab=False, is_persistent=True)


CONFIGS = [(64, (1, 1, 1)), (256, (1, 1, 1)), (128, (2, 1, 1)), (512, (2, 1, 1))]


@pytest.mark.parametrize("act", ACTS)
@pytest.mark.parametrize("tile_n,cluster", CONFIGS)
def test_activation_with_bias(act, tile_n, cluster):
    m, n, k = 384, 1000, 520
    a, b, bias = gemm_ref.make_inputs(m, n, k, seed=21, b_scale=k ** -0.5, with_bias=True)
    d = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    gemm = make_gemm(tile_n, cluster, stages=3 if tile_n == 512 else 4)
    gemm(a.cuda(), b.cuda(), d, None, bias=bias.cuda(), alpha=1.5, activation=act)
    torch.cuda.synchronize()
    res = gemm_ref.check_epilogue(d.cpu(), a, b, bias=bias, alpha=1.5, act=act)
    assert res["ok"], res


@pytest.mark.parametrize("tile_n,cluster", CONFIGS)
@pytest.mark.parametrize("out_dtype", [torch.bfloat16, torch.float32])
def test_source_beta(tile_n, cluster, out_dtype):
    """D = alpha A B^T + bias + beta C with C a separate tensor of D's type."""
    m, n, k = 300, 392, 264
    a, b, bias = gemm_ref.make_inputs(m, n, k, seed=22, with_bias=True)
    g = torch.Generator().manual_seed(23)
    c = (torch.randn(m, n, generator=g) * 8).to(out_dtype)
    d = torch.full((m, n), float("nan"), dtype=out_dtype, device="cuda")
    gemm = make_gemm(tile_n, cluster, stages=3 if tile_n == 512 else 4)
    gemm(a.cuda(), b.cuda(), d, None, bias=bias.cuda(), source=c.cuda(), beta=-0.75)
    torch.cuda.synchronize()
    rounding = gemm_ref.BF16_REL if out_dtype == torch.bfloat16 else 2.0 ** -24
    res = gemm_ref.check_epilogue(d.cpu(), a, b, bias=bias, beta=-0.75, c=c,
                                  out_rounding=rounding)
    assert res["ok"], res


@pytest.mark.parametrize("cluster", [(1, 1, 1), (2, 1, 1)])
def test_source_in_place_residual(cluster):
    """D <- D + A B^T (C is D itself), then an activation on top of a strided C view."""
    m, n, k = 512, 768, 1024
    a, b, _ = gemm_ref.make_inputs(m, n, k, seed=24, b_scale=k ** -0.5)
    g = torch.Generator().manual_seed(25)
    c0 = torch.randn(m, n, generator=g).to(torch.bfloat16)
    d = c0.cuda()
    gemm = make_gemm(256, cluster)
    gemm(a.cuda(), b.cuda(), d, None, source=d, beta=1.0)
    torch.cuda.synchronize()
    res = gemm_ref.check_epilogue(d.cpu(), a, b, c=c0)
    assert res["ok"], res
    # C as a column slice of a wider buffer (row stride 1024 elements), GELU on the sum.
    wide = torch.randn(m, 1024, generator=g).to(torch.bfloat16)
    cv = wide.cuda()[:, 128:128 + n]
    out = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    gemm(a.cuda(), b.cuda(), out, None, source=cv, beta=0.5, activation="gelu")
    torch.cuda.synchronize()
    res = gemm_ref.check_epilogue(out.cpu(), a, b, c=wide[:, 128:128 + n], beta=0.5, act="gelu")
    assert res["ok"], res


@pytest.mark.parametrize("act", ["silu", "gelu", "gelu_tanh"])
@pytest.mark.parametrize("cluster", [(1, 1, 1), (2, 1, 1)])
@pytest.mark.parametrize("shape", [(256, 256, 512), (300, 200, 264), (1024, 1536, 1024)])
def test_gated(act, cluster, shape):
    """SwiGLU / GeGLU: B = [W_gate; W_up] (2N rows), D = act(A Wg^T) * (A Wu^T)."""
    m, n, k = shape
    a, b, _ = gemm_ref.make_inputs(m, 2 * n, k, seed=m + n + k, b_scale=k ** -0.5)
    d = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    gemm = make_gemm(512, cluster, stages=3 if cluster[0] == 2 else 2)
    gemm(a.cuda(), b.cuda(), d, None, activation=act, gated=True, alpha=0.9)
    torch.cuda.synchronize()
    res = gemm_ref.check_gated(d.cpu(), a, b, alpha=0.9, act=act)
    assert res["ok"], res


def test_gated_fp8_per_tensor():
    m, n, k = 512, 640, 1024
    g = torch.Generator().manual_seed(31)
    a = torch.randn(m, k, generator=g)
    b = torch.randn(2 * n, k, generator=g) * k ** -0.5
    qa, sa = quantize_e4m3(a.cuda())
    qb, sb = quantize_e4m3(b.cuda())
    d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    gemm = make_gemm(512, (2, 1, 1), stages=3)
    gemm(qa, qb, d, None, scale_a=sa, scale_b=sb, activation="silu", gated=True)
    torch.cuda.synchronize()
    da = qa.cpu().float() * sa.cpu()
    db = qb.cpu().float() * sb.cpu()
    res = gemm_ref.check_gated(d.cpu(), da, db, act="silu", frob_tol=gemm_ref.FROB_TOL_FP8)
    assert res["ok"], res


def test_fused_epilogue_rejections():
    m, n, k = 256, 256, 256
    a, b, bias = gemm_ref.make_inputs(m, 2 * n, k, seed=5, with_bias=True)
    a, b, bias = a.cuda(), b.cuda(), bias.cuda()
    d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.CpgError):  # gated needs 512-wide tiles
        make_gemm(256, (1, 1, 1))(a, b, d, None, gated=True, activation="silu")
    with pytest.raises(_lib.CpgError):  # gated takes no bias
        make_gemm(512, (1, 1, 1), stages=2)(a, b, d, None, gated=True, bias=bias[:n])
    with pytest.raises(_lib.CpgError):  # unknown activation
        make_gemm(256, (1, 1, 1))(a, b[:n], d, None, activation="tanh")
    d32 = torch.empty(m, n, dtype=torch.float32, device="cuda")
    with pytest.raises(_lib.CpgError):  # activations need the whole K in one pass
        make_gemm(256, (1, 1, 1))(a, b[:n], d32, None, activation="relu", split_k=2)
    odd = torch.empty(m, n + 1, dtype=torch.bfloat16, device="cuda")[:, :n]
    with pytest.raises(_lib.CpgError):  # C rows not 16-byte aligned
        make_gemm(256, (1, 1, 1))(a, b[:n], d, None, source=odd)


@pytest.mark.parametrize("act", ["relu", "gelu"])
def test_fp8_per_tensor_with_bias_and_activation(act):
    m, n, k = 384, 768, 512
    g = torch.Generator().manual_seed(33)
    a = torch.randn(m, k, generator=g)
    b = torch.randn(n, k, generator=g) * k ** -0.5
    bias = torch.randn(n, generator=g).to(torch.bfloat16)
    qa, sa = quantize_e4m3(a.cuda())
    qb, sb = quantize_e4m3(b.cuda())
    d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    make_gemm(512, (2, 1, 1), stages=3)(qa, qb, d, None, scale_a=sa, scale_b=sb,
                                        bias=bias.cuda(), activation=act)
    torch.cuda.synchronize()
    res = gemm_ref.check_epilogue(d.cpu(), qa.cpu().float() * sa.cpu(),
                                  qb.cpu().float() * sb.cpu(), bias=bias, act=act,
                                  frob_tol=gemm_ref.FROB_TOL_FP8)
    assert res["ok"], res
