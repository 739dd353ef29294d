"""Pure-Python restatement of the reference's FastDivmod -- TEST ORACLE ONLY.

Follows adelmuursepp/cutedsl_pingpong_gemm ``fast_math.py``:

* ``clz``       fast_math.py:17-26  (count leading zeros of an Int32)
* ``find_log2`` fast_math.py:29-31  (ceil(log2(x)))
* ``umulhi``    fast_math.py:34-47  (``mul.hi.u32``: high 32 bits of the u32 x u32 product)
* ``FastDivmod.create`` fast_math.py:56-65, ``div`` :67-76, ``divmod`` :78-81

Integer widths are emulated exactly: Uint32 results are reduced modulo 2**32, Int32 results
are wrapped to [-2**31, 2**31).  Pinned against ``tests/golden/fast_divmod.json``.
"""

MASK32 = 0xFFFFFFFF


def _i32(x: int) -> int:
    x &= MASK32
    return x - (1 << 32) if x & 0x80000000 else x


def clz(x: int) -> int:
    """fast_math.py:17-26: index of the first set bit scanning from bit 31 down; 32 if x == 0."""
    x &= MASK32
    for i in range(32):
        if (1 << (31 - i)) & x:
            return i
    return 32


def find_log2(x: int) -> int:
    """fast_math.py:29-31: 31 - clz(x), plus one when x is not a power of two."""
    a = _i32(31 - clz(x))
    return a + (1 if (x & (x - 1)) != 0 else 0)


def umulhi(a: int, b: int) -> int:
    """fast_math.py:34-47: (a * b) >> 32 on unsigned 32-bit operands."""
    return ((a & MASK32) * (b & MASK32)) >> 32


class FastDivmod:
    """fast_math.py:49-81."""

    def __init__(self, divisor: int, multiplier: int, shift_right: int):
        self.divisor = divisor
        self.multiplier = multiplier
        self.shift_right = shift_right

    @staticmethod
    def create(divisor: int) -> "FastDivmod":
        # fast_math.py:61-65.  p = 31 + ceil(log2(d)); multiplier = ceil(2^p / d) as Uint32;
        # shift_right = p - 32 as Uint32 (wraps to 0xFFFFFFFF for d == 1, where div bypasses it).
        p = (31 + find_log2(divisor)) & MASK32
        d = divisor & MASK32
        multiplier = (((1 << p) + d - 1) // d) & MASK32
        shift_right = (p - 32) & MASK32
        return FastDivmod(divisor, multiplier, shift_right)

    def div(self, dividend: int) -> int:
        # fast_math.py:72-76
        if self.divisor == 1:
            return dividend
        return _i32(umulhi(dividend, self.multiplier) >> self.shift_right)

    def divmod(self, dividend: int):
        # fast_math.py:78-81
        q = self.div(dividend)
        return q, _i32(dividend - q * self.divisor)
