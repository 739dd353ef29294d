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


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
@pytest.mark.parametrize("block", [(1, 128), (128, 128)])
@pytest.mark.parametrize("shape", [(1, 128), (128, 256), (300, 1000), (1000, 4104), (256, 4096)])
def test_block_bit_exact(shape, block, dtype):
    """Whole blocks take the vector kernels, ragged edge blocks the element form."""
    g = torch.Generator().manual_seed(7 + sum(shape))
    x = (torch.randn(*shape, generator=g) * torch.rand(shape[0], 1, generator=g) * 10).to(dtype)
    q, s = quantize_e4m3(x.cuda(), block)
    qr, sr = gemm_ref.quantize_e4m3_blocks(x, block)
    assert torch.equal(s.cpu(), sr)
    assert torch.equal(_bits(q.cpu()), _bits(qr))


@pytest.mark.parametrize("block", [(1, 128), (128, 128)])
def test_block_unaligned_view(block):
    """Rows that start off the vector boundary: the element kernels."""
    g = torch.Generator().manual_seed(98)
    big = (torch.randn(256, 1040, generator=g) * 3).to(torch.bfloat16)
    x = big[:, 1:1025]
    q, s = quantize_e4m3(big.cuda()[:, 1:1025], block)
    qr, sr = gemm_ref.quantize_e4m3_blocks(x, block)
    assert torch.equal(s.cpu(), sr)
    assert torch.equal(_bits(q.cpu()), _bits(qr))


def _near_midpoints(rows, cols, amax, ulps, seed):
    """x with amax(|x|) = `amax` in every 128-column block of every row (column 0 of the block),
    all other entries such that x / s (s = amax / 448) lies within `ulps` fp32 steps of an E4M3
    rounding midpoint: the normal-range midpoints (1 + (2k + 1) / 16) 2^e and the subnormal ones
    (2j + 1) 2^-10, with random signs."""
    import numpy as np
    rng = np.random.default_rng(seed)
    s = np.float32(amax) / np.float32(448.0)
    mids = [(1 + (2 * k + 1) / 16) * 2.0 ** e for e in range(-6, 9) for k in range(8)]
    mids = [m for m in mids if m <= 440] + [(2 * j + 1) * 2.0 ** -10 for j in range(7)]
    base = np.float32(rng.choice(mids, size=(rows, cols))) * s
    steps = rng.integers(-ulps, ulps + 1, size=(rows, cols)).astype(np.int32)
    x = (base.view(np.int32) + steps).view(np.float32)
    x = np.minimum(x, np.float32(amax) * np.float32(440 / 448))
    x *= np.where(rng.random((rows, cols)) < 0.5, np.float32(-1), np.float32(1))
    x[:, ::128] = np.float32(amax)
    return torch.from_numpy(x)


@pytest.mark.parametrize("block", [None, (1, 128), (128, 128)])
def test_near_midpoint_inputs(block):
    """The vector kernels quantise with a reciprocal multiply and fall back to the division where
    the product is within a few steps of an E4M3 rounding midpoint; inputs placed within 3 fp32
    steps of the midpoints (non-power-of-two scale), and BF16 inputs exactly on them (scale 1/8,
    ties to even), must still give the oracle's bytes."""
    cases = [_near_midpoints(256, 1024, 3.7, 3, seed=5),
             _near_midpoints(256, 1024, 56.0, 0, seed=6).to(torch.bfloat16)]
    for x in cases:
        if block is None:
            q, s = quantize_e4m3(x.cuda())
            qr, sr = gemm_ref.quantize_e4m3_per_tensor(x)
        else:
            q, s = quantize_e4m3(x.cuda(), block)
            qr, sr = gemm_ref.quantize_e4m3_blocks(x, block)
        assert torch.equal(s.cpu().reshape(sr.shape), sr)
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
