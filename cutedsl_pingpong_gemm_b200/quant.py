"""FP8 E4M3 quantisation and FP32 -> BF16 cast on the GPU (C ABI: cpg_quantize_e4m3,
cpg_cast_f32_bf16).

``quantize_e4m3(x, block=None)`` returns ``(q, scales)`` with ``s = amax(|x|) / 448`` per tensor
(``block=None``), per 1 x 128 block (``block=(1, 128)``, the A operand of block-scaled FP8
GEMM) or per 128 x 128 block (``block=(128, 128)``, the B operand), and ``q = e4m3(x / s)``.
Scale layouts are described in ``include/cpgemm.h``.
"""
from typing import Optional, Tuple

from . import _lib


def _stream(t):
    import torch
    return torch.cuda.current_stream(t.device).cuda_stream


def quantize_e4m3(x, block: Optional[Tuple[int, int]] = None):
    import torch
    if not x.is_cuda or x.dim() != 2 or x.dtype not in (torch.bfloat16, torch.float32):
        raise _lib.CpgError(_lib.CPG_ERR_DTYPE, "x must be a 2-D BF16 or FP32 CUDA tensor")
    if x.numel() and x.stride(1) != 1:
        raise _lib.CpgError(_lib.CPG_ERR_UNSUPPORTED, "x must have unit column stride")
    rows, cols = x.shape
    q = torch.empty(rows, cols, dtype=torch.float8_e4m3fn, device=x.device)
    br, bc = (0, 0) if block is None else block
    if (br, bc) == (0, 0):
        scales = torch.empty(1, dtype=torch.float32, device=x.device)
    elif (br, bc) == (1, 128):
        scales = torch.empty(-(-cols // 128), rows, dtype=torch.float32, device=x.device)
    elif (br, bc) == (128, 128):
        scales = torch.empty(-(-rows // 128), -(-cols // 128), dtype=torch.float32, device=x.device)
    else:
        raise _lib.CpgError(_lib.CPG_ERR_UNSUPPORTED, f"block {block} not supported")
    dt = _lib.CPG_DTYPE_BF16 if x.dtype == torch.bfloat16 else _lib.CPG_DTYPE_F32
    ldx = x.stride(0) if rows > 1 else cols
    lib = _lib.load()
    _lib.check(lib.cpg_quantize_e4m3(x.data_ptr() if x.numel() else None, dt, rows, cols, ldx,
                                     q.data_ptr() if q.numel() else None, cols, scales.data_ptr(),
                                     br, bc, _stream(x)), "quantize_e4m3")
    return q, scales


def cast_f32_bf16(x, bias=None, out=None, stream=None):
    """out = bf16(x + bias) for a 2-D FP32 CUDA tensor x (on ``stream``, default current)."""
    import torch
    if not x.is_cuda or x.dim() != 2 or x.dtype != torch.float32:
        raise _lib.CpgError(_lib.CPG_ERR_DTYPE, "x must be a 2-D FP32 CUDA tensor")
    rows, cols = x.shape
    if out is None:
        out = torch.empty(rows, cols, dtype=torch.bfloat16, device=x.device)
    if bias is not None and (bias.dtype != torch.bfloat16 or bias.numel() != cols):
        raise _lib.CpgError(_lib.CPG_ERR_INVALID_SHAPE, "bias must be BF16 of length cols")
    ldx = x.stride(0) if rows > 1 else cols
    ldy = out.stride(0) if rows > 1 else cols
    lib = _lib.load()
    from .gemm_base import _stream_handle
    st = _stream_handle(stream, x.device)
    _lib.check(lib.cpg_cast_f32_bf16(x.data_ptr() if x.numel() else None, rows, cols, ldx,
                                     out.data_ptr() if out.numel() else None, ldy,
                                     None if bias is None else bias.data_ptr(), st),
               "cast_f32_bf16")
    return out
