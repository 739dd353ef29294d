"""FastDivmod with the interface of the reference's ``fast_math.FastDivmod`` (fast_math.py:49-81).

``create`` precomputes the multiplier and shift on the host, ``div``/``divmod`` divide by the
fixed divisor.  The arithmetic is the shared C++ header ``csrc/fast_divmod.h``, reached through
the C ABI, which is the same code the GEMM kernels run for their tile coordinates; ``divmod_device``
runs that code on the GPU for a batch of dividends.
"""
import ctypes
from dataclasses import dataclass
from typing import Tuple

from . import _lib


@dataclass
class FastDivmod:
    divisor: int
    multiplier: int
    shift_right: int

    @staticmethod
    def create(divisor: int) -> "FastDivmod":
        """fast_math.py:56-65: p = 31 + ceil(log2(d)), multiplier = ceil(2^p / d), shift = p - 32."""
        lib = _lib.load()
        out = _lib.FastDivmodC()
        _lib.check(lib.cpg_fast_divmod_create(int(divisor), ctypes.byref(out)), "FastDivmod.create")
        return FastDivmod(out.divisor, out.multiplier, out.shift_right)

    def _c(self) -> "_lib.FastDivmodC":
        return _lib.FastDivmodC(self.divisor, self.multiplier, self.shift_right)

    def div(self, dividend: int) -> int:
        """fast_math.py:67-76: umulhi(dividend, multiplier) >> shift, or dividend when d == 1."""
        return self.divmod(dividend)[0]

    def divmod(self, dividend: int) -> Tuple[int, int]:
        """fast_math.py:78-81: (quotient, dividend - quotient * divisor)."""
        lib = _lib.load()
        q, r = ctypes.c_int32(), ctypes.c_int32()
        f = self._c()
        _lib.check(lib.cpg_fast_divmod_divmod(ctypes.byref(f), int(dividend), ctypes.byref(q),
                                              ctypes.byref(r)), "FastDivmod.divmod")
        return q.value, r.value

    def divmod_device(self, x):
        """(q, r) for a CUDA int32 tensor ``x``, computed by the device code of the kernels."""
        import torch
        if not (x.is_cuda and x.dtype == torch.int32 and x.is_contiguous()):
            raise ValueError("x must be a contiguous CUDA int32 tensor")
        q = torch.empty_like(x)
        r = torch.empty_like(x)
        lib = _lib.load()
        f = self._c()
        stream = torch.cuda.current_stream(x.device).cuda_stream
        _lib.check(lib.cpg_fast_divmod_device(ctypes.byref(f), x.data_ptr(), q.data_ptr(),
                                              r.data_ptr(), x.numel(), stream),
                   "FastDivmod.divmod_device")
        return q, r
