"""The numerics checker of the GPU parity tests, checked on CPU: it must accept a correctly
rounded BF16 product and reject the mistakes a GEMM kernel can make.  Each mistake is planted in
a CPU-made output, never on the GPU.

Tolerance under test (oracle/gemm_ref.py): relative Frobenius <= 1e-2 and the element-wise bound
|D - R| <= 2^-8 |R| + K 2^-23 (|A| |B|^T) (+ 2^-24 |bias|).
"""
import torch

from oracle import gemm_ref

M, N, K = 96, 160, 320


def _inputs(with_bias=False):
    return gemm_ref.make_inputs(M, N, K, seed=5, b_scale=K ** -0.5, with_bias=with_bias)


def _bf16_product(a, b, bias=None, alpha=1.0):
    return gemm_ref.reference(a, b, bias, alpha).to(torch.bfloat16)


def test_accepts_the_rounded_product_and_its_sampled_rows():
    a, b, bias = _inputs(with_bias=True)
    d = _bf16_product(a, b, bias, alpha=0.5)
    assert gemm_ref.check(d, a, b, bias=bias, alpha=0.5)["ok"]
    rows = torch.tensor([0, 7, 95])
    assert gemm_ref.check(d[rows], a, b, bias=bias, alpha=0.5, rows=rows)["ok"]


def test_rejects_planted_mistakes():
    a, b, bias = _inputs(with_bias=True)
    good = _bf16_product(a, b, bias)
    mistakes = {
        # one k-block (64 columns of K) left out of the sum
        "missing k-block": _bf16_product(a[:, 64:], b[:, 64:], bias),
        # the bias not added, or added twice
        "no bias": _bf16_product(a, b),
        "bias twice": (gemm_ref.reference(a, b, bias) + bias.float()).to(torch.bfloat16),
        # alpha ignored
        "alpha ignored": good,
        # two rows of tiles swapped (a wrong tile map)
        "rows swapped": torch.cat([good[32:64], good[:32], good[64:]]),
        # one element off by 2 % of its magnitude plus 0.05
        "one element": good.clone().index_put_((torch.tensor([3]), torch.tensor([5])),
                                               good[3, 5] + 0.02 * good[3, 5].abs() + 0.05),
        # an FP32 partial sum truncated to BF16 before the last K range is added
        "early rounding": (gemm_ref.reference(a[:, :K // 2], b[:, :K // 2]).to(torch.bfloat16)
                           .float() * 1.01 + gemm_ref.reference(a[:, K // 2:], b[:, K // 2:])
                           + bias.float()).to(torch.bfloat16),
    }
    for name, d in mistakes.items():
        alpha = 0.5 if name == "alpha ignored" else 1.0
        res = gemm_ref.check(d, a, b, bias=bias, alpha=alpha)
        assert not res["ok"], (name, res)


def test_rejects_a_transposed_operand():
    g = torch.Generator().manual_seed(9)
    a = torch.randn(128, 128, generator=g).to(torch.bfloat16)
    b = (torch.randn(128, 128, generator=g) * 128 ** -0.5).to(torch.bfloat16)
    wrong = (a.float() @ b.float()).to(torch.bfloat16)  # A . B instead of A . B^T
    assert not gemm_ref.check(wrong, a, b)["ok"]
    assert gemm_ref.check((a.float() @ b.float().t()).to(torch.bfloat16), a, b)["ok"]


def test_checksums_match_the_full_product():
    a, b, bias = _inputs(with_bias=True)
    r = 2.0 * (a.double() @ b.double().t()) + bias.double()  # exact in fp64 for these sizes
    assert torch.allclose(gemm_ref.column_checksum(a, b, bias, alpha=2.0), r.sum(0),
                          rtol=1e-9, atol=1e-9)
    assert torch.allclose(gemm_ref.row_checksum(a, b, bias, alpha=2.0), r.sum(1),
                          rtol=1e-9, atol=1e-9)


def test_e4m3_quantisers_round_trip_within_half_an_fp8_step():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(256, 384, generator=g).to(torch.bfloat16)
    q, s = gemm_ref.quantize_e4m3_per_tensor(x)
    assert q.dtype == torch.float8_e4m3fn and s.numel() == 1
    assert float(q.float().abs().max()) == 448.0  # the amax element maps to the largest finite
    back = gemm_ref.dequantize(q, s)
    # E4M3 keeps 3 mantissa bits: the relative error of a normal value is at most 2^-4.
    normal = x.float().abs() / s > 2.0 ** -6
    rel = ((back - x.float()).abs() / x.float().abs().clamp_min(1e-30))[normal]
    assert float(rel.max()) <= 2.0 ** -4
    for block in ((1, 128), (128, 128)):
        qb, sb = gemm_ref.quantize_e4m3_blocks(x, block)
        xb = gemm_ref.dequantize_blocks(qb, sb, block)
        assert xb.shape == x.shape
        assert gemm_ref.rel_frobenius(xb, x.float()) < 3e-2
