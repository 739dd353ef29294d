"""FP8 quantiser and FP32->BF16 cast kernels against the oracle (bit-exact: the quantised bytes and
the fp32 scales must be identical, since both follow s = amax/448, q = RN-even e4m3(x / s))."""
import pytest
import torch

from cutedsl_pingpong_gemm_b200.quant import cast_f32_bf16, quantize_e4m3
from oracle import gemm_ref

pytestmark = pytest.mark.gpu


def _bits(q):
    return q.view(torch.uint8)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("shape", [(1, 16), (128, 256), (300, 1000), (1024, 4096), (7, 1001),
                                   (3, 6)])
def test_per_tensor_bit_exact(shape, dtype):
    """Whole 16-byte vectors per row take the vectorised kernels, the odd widths the element
    kernels; both must give the oracle's bytes."""
    g = torch.Generator().manual_seed(sum(shape))
    x = (torch.randn(*shape, generator=g) * 3.0).to(dtype)
    q, s = quantize_e4m3(x.cuda())
    qr, sr = gemm_ref.quantize_e4m3_per_tensor(x)
    assert s.cpu().item() == sr.item()
    assert torch.equal(_bits(q.cpu()), _bits(qr))


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_per_tensor_unaligned_view(dtype):
    """A column window whose rows start off a 16-byte boundary: element kernels."""
    g = torch.Generator().manual_seed(99)
    big = (torch.randn(64, 1040, generator=g) * 2).to(dtype)
    x = big[:, 3:1027]
    q, s = quantize_e4m3(big.cuda()[:, 3:1027])
    qr, sr = gemm_ref.quantize_e4m3_per_tensor(x)
    assert s.cpu().item() == sr.item()
    assert torch.equal(_bits(q.cpu()), _bits(qr))


@pytest.mark.parametrize("block", [(1, 128), (128, 128)])
@pytest.mark.parametrize("shape", [(1, 128), (128, 256), (300, 1000), (1000, 4104)])
def test_block_bit_exact(shape, block):
    g = torch.Generator().manual_seed(7 + sum(shape))
    x = torch.randn(*shape, generator=g) * torch.rand(shape[0], 1, generator=g) * 10
    q, s = quantize_e4m3(x.cuda(), block)
    qr, sr = gemm_ref.quantize_e4m3_blocks(x, block)
    assert torch.equal(s.cpu(), sr)
    assert torch.equal(_bits(q.cpu()), _bits(qr))


def test_zero_and_saturation():
    x = torch.zeros(64, 64)
    q, s = quantize_e4m3(x.cuda())
    assert s.item() == pytest.approx(1e-12 / 448)
    assert torch.count_nonzero(_bits(q)).item() == 0
    x = torch.tensor([[1e30, -1e30, 1.0, -448.0]])
    q, s = quantize_e4m3(x.cuda())
    assert torch.equal(_bits(q.cpu()), _bits(gemm_ref.quantize_e4m3_per_tensor(x)[0]))


def test_cast_with_bias():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(257, 520, generator=g) * 100
    bias = torch.randn(520, generator=g).to(torch.bfloat16)
    y = cast_f32_bf16(x.cuda(), bias.cuda())
    want = (x + bias.float()).to(torch.bfloat16)
    assert torch.equal(y.cpu(), want)


@pytest.mark.parametrize("shape", [(1, 1), (3, 7), (129, 1030), (64, 8192)])
def test_cast_odd_and_strided_shapes(shape):
    """Scalar path (columns not a multiple of 4) and strided views."""
    rows, cols = shape
    g = torch.Generator().manual_seed(rows * cols)
    full = torch.randn(rows, cols + 5, generator=g) * 50
    x = full[:, 1:cols + 1]
    y = cast_f32_bf16(x.cuda())
    assert torch.equal(y.cpu(), x.to(torch.bfloat16))
