"""fp32 CPU reference for D = A @ B.T and the tolerance checks -- TEST ORACLE ONLY.

Spec followed: the reference harness computes ``ref = a @ b.t()`` on BF16 inputs and compares the
kernel's BF16 ``c`` with it (gemm_base.py:587-590, :611).  The reference kernel accumulates in fp32
(``acc_dtype = Float32``, gemm_base.py:63) and converts to BF16 in the epilogue (:336-338).  Here the
product is evaluated in fp32 (or fp64 for checksums) on the CPU from the same BF16-rounded inputs.

Tolerances (project spec, stated in the tests that use them):

* relative Frobenius error ``||D - R||_F / ||R||_F <= 1e-2`` for BF16 outputs;
* element-wise ``|D - R| <= 2^-8 |R| + K * 2^-23 * (|A| @ |B|.T)``: BF16 output rounding (half an
  ulp is at most 2^-8 relative) plus the worst-case fp32 summation error of a K-term dot product
  for both the kernel and this reference (each at most (K-1) * 2^-24 * sum|a||b|).
"""
import os

import torch

BF16_REL = 2.0 ** -8
ACC_SLACK_PER_K = 2.0 ** -23
FROB_TOL_BF16 = 1e-2
FROB_TOL_FP8 = 3e-2


def set_threads():
    n = os.cpu_count() or 1
    torch.set_num_threads(n)
    return n


def make_inputs(m, n, k, seed=0, a_scale=1.0, b_scale=1.0, with_bias=False, bias_scale=1.0):
    """Seeded BF16 inputs: torch.Generator().manual_seed(seed) on the CPU, N(0,1) times a scale."""
    g = torch.Generator().manual_seed(seed)
    a = (torch.randn(m, k, generator=g) * a_scale).to(torch.bfloat16)
    b = (torch.randn(n, k, generator=g) * b_scale).to(torch.bfloat16)
    bias = (torch.randn(n, generator=g) * bias_scale).to(torch.bfloat16) if with_bias else None
    return a, b, bias


def reference(a, b, bias=None, alpha=1.0, rows=None):
    """fp32 R = alpha * A @ B.T (+ bias) on the CPU; ``rows`` restricts to a subset of rows."""
    a32 = a.float() if rows is None else a[rows].float()
    r = torch.matmul(a32, b.float().t())
    if alpha != 1.0:
        r = r * alpha
    if bias is not None:
        r = r + bias.float()
    return r


def abs_product(a, b, rows=None):
    a32 = a.float().abs() if rows is None else a[rows].float().abs()
    return torch.matmul(a32, b.float().abs().t())


def elementwise_bound(r, s, k, alpha=1.0, bias=None):
    tol = BF16_REL * r.abs() + abs(alpha) * k * ACC_SLACK_PER_K * s
    if bias is not None:
        tol = tol + 2.0 ** -24 * bias.float().abs()
    return tol


def rel_frobenius(d, r):
    d64 = d.double()
    r64 = r.double()
    den = torch.linalg.vector_norm(r64)
    num = torch.linalg.vector_norm(d64 - r64)
    return float(num / den) if float(den) > 0 else float(num)


def check(d, a, b, bias=None, alpha=1.0, rows=None, frob_tol=FROB_TOL_BF16):
    """Compare GPU output ``d`` (CPU tensor, full or the selected rows) with the fp32 oracle.

    Returns a dict with the error figures; ``ok`` is True when both bounds hold.
    """
    k = a.shape[1]
    r = reference(a, b, bias, alpha, rows)
    s = abs_product(a, b, rows)
    dd = d.float() if rows is None or d.shape[0] == r.shape[0] else d[rows].float()
    if dd.shape != r.shape:
        raise ValueError(f"shape mismatch {tuple(dd.shape)} vs {tuple(r.shape)}")
    tol = elementwise_bound(r, s, k, alpha, bias)
    err = (dd - r).abs()
    viol = err > tol
    frob = rel_frobenius(dd, r)
    n_bad = int(viol.sum())
    worst = float((err / tol.clamp_min(1e-30)).max()) if err.numel() else 0.0
    return {"ok": n_bad == 0 and frob <= frob_tol, "n_bad": n_bad, "frob": frob,
            "worst_ratio": worst, "max_abs_err": float(err.max()) if err.numel() else 0.0}


def column_checksum(a, b, bias=None, alpha=1.0):
    """fp64 sum over rows of R: (1^T A) B^T (+ M * bias).  Cost O(MK + NK)."""
    colsum_a = a.double().sum(0)
    r = alpha * torch.matmul(b.double(), colsum_a)
    if bias is not None:
        r = r + a.shape[0] * bias.double()
    return r


def row_checksum(a, b, bias=None, alpha=1.0):
    """fp64 sum over columns of R: A (B^T 1) (+ sum(bias))."""
    rowsum_b = b.double().sum(0)
    r = alpha * torch.matmul(a.double(), rowsum_b)
    if bias is not None:
        r = r + bias.double().sum()
    return r


def checksum_bound(d_abs_sum, abs_sum_product, k, count):
    """Bound for a checksum of ``count`` BF16 outputs: rounding of each output plus accumulation."""
    return BF16_REL * d_abs_sum + k * ACC_SLACK_PER_K * abs_sum_product + 1e-6 * count


E4M3_MAX = 448.0


def quantize_e4m3_per_tensor(x):
    """Per-tensor FP8 E4M3 quantisation of the project spec: s = amax(|x|) / 448, q = e4m3(x / s).

    Returns (q as torch.float8_e4m3fn, s as a 0-d float32 tensor).  The dequantised operand is
    q.float() * s; the GEMM oracle for FP8 is the fp32 product of dequantised operands.
    """
    xf = x.float()
    amax = xf.abs().max().clamp_min(1e-12)
    s = (amax / E4M3_MAX).to(torch.float32)
    q = (xf / s).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
    return q, s


def dequantize(q, s):
    return q.float() * s


def make_fp8_inputs(m, n, k, seed=0):
    """BASELINE config 4 inputs: A, B ~ N(0,1), quantised per tensor."""
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(m, k, generator=g)
    b = torch.randn(n, k, generator=g)
    qa, sa = quantize_e4m3_per_tensor(a)
    qb, sb = quantize_e4m3_per_tensor(b)
    return qa, sa, qb, sb


def check_fp8(d, qa, sa, qb, sb, rows=None, frob_tol=FROB_TOL_FP8):
    """FP8 GEMM check against the fp32 product of the dequantised operands."""
    a = dequantize(qa, sa)
    b = dequantize(qb, sb)
    return check(d, a, b, rows=rows, frob_tol=frob_tol)


def quantize_e4m3_blocks(x, block):
    """Block FP8 quantisation (oracle): block (1,128) -> scales [ceil(K/128), M] (one per row and
    128 columns), block (128,128) -> scales [ceil(M/128), ceil(K/128)].  Same s = amax/448 rule."""
    xf = x.float()
    m, k = xf.shape
    nkb = -(-k // 128)
    pad_k = nkb * 128 - k
    if block == (1, 128):
        xp = torch.nn.functional.pad(xf, (0, pad_k)).reshape(m, nkb, 128)
        amax = xp.abs().amax(dim=2).clamp_min(1e-12)          # [m, nkb]
        s = (amax / E4M3_MAX).to(torch.float32)
        q = (xp / s.unsqueeze(2)).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
        return q.reshape(m, nkb * 128)[:, :k].contiguous(), s.t().contiguous()
    if block == (128, 128):
        nmb = -(-m // 128)
        xp = torch.nn.functional.pad(xf, (0, pad_k, 0, nmb * 128 - m)).reshape(nmb, 128, nkb, 128)
        amax = xp.abs().amax(dim=(1, 3)).clamp_min(1e-12)    # [nmb, nkb]
        s = (amax / E4M3_MAX).to(torch.float32)
        q = (xp / s[:, None, :, None]).clamp(-E4M3_MAX, E4M3_MAX).to(torch.float8_e4m3fn)
        return q.reshape(nmb * 128, nkb * 128)[:m, :k].contiguous(), s
    raise ValueError(block)


def dequantize_blocks(q, s, block):
    qf = q.float()
    m, k = qf.shape
    if block == (1, 128):
        scale = s.t().repeat_interleave(128, dim=1)[:, :k]
    else:
        scale = s.repeat_interleave(128, dim=0).repeat_interleave(128, dim=1)[:m, :k]
    return qf * scale


# ---------------------------------------------------------------- fused epilogue (spec of cpgemm.h)
# D = act(alpha * A @ B.T + bias + beta * C); gated: D = act(alpha * A @ Wg.T) * (alpha * A @ Wu.T).
# Activation formulas as documented for CPG_ACT_*; the kernel evaluates them with CUDA's expf /
# erff / tanhf family, which the ACT_REL term below covers.
ACT_SLOPE = 1.13   # max |act'(y)| over the reals for relu, silu (1.0998), gelu (1.1289), gelu_tanh
ACT_REL = 2.0 ** -18


def activation(name, y):
    if name in (None, "none"):
        return y
    if name == "relu":
        return y.clamp_min(0.0)
    if name == "silu":
        return y * torch.sigmoid(y)
    if name == "gelu":
        return 0.5 * y * (1.0 + torch.erf(y * 0.7071067811865476))
    if name == "gelu_tanh":
        return 0.5 * y * (1.0 + torch.tanh(0.7978845608028654 * (y + 0.044715 * y * y * y)))
    raise ValueError(name)


def check_epilogue(d, a, b, bias=None, alpha=1.0, beta=1.0, c=None, act=None,
                   frob_tol=FROB_TOL_BF16, out_rounding=BF16_REL):
    """Check D = act(alpha A B^T + bias + beta C) (fp32 CPU oracle, C given on the CPU)."""
    k = a.shape[1]
    pre = reference(a, b, bias, alpha)
    tol_pre = abs(alpha) * k * ACC_SLACK_PER_K * abs_product(a, b)
    if bias is not None:
        tol_pre = tol_pre + 2.0 ** -24 * bias.float().abs()
    if c is not None:
        bc = beta * c.float()
        pre = pre + bc
        tol_pre = tol_pre + 2.0 ** -23 * (bc.abs() + pre.abs())
    r = activation(act, pre)
    tol = out_rounding * r.abs() + ACT_SLOPE * tol_pre + ACT_REL * pre.abs() + 1e-6
    return _verdict(d.float(), r, tol, frob_tol)


def check_gated(d, a, b_stacked, alpha=1.0, act="silu", frob_tol=FROB_TOL_BF16):
    """Check D = act(alpha A Wg^T) * (alpha A Wu^T) for B = [Wg; Wu] (2N rows)."""
    k = a.shape[1]
    n = b_stacked.shape[0] // 2
    wg, wu = b_stacked[:n], b_stacked[n:]
    g = reference(a, wg, None, alpha)
    u = reference(a, wu, None, alpha)
    tg = abs(alpha) * k * ACC_SLACK_PER_K * abs_product(a, wg)
    tu = abs(alpha) * k * ACC_SLACK_PER_K * abs_product(a, wu)
    ag = activation(act, g)
    r = ag * u
    tol = (BF16_REL * r.abs() + ACT_SLOPE * tg * (u.abs() + tu) + ag.abs() * tu
           + ACT_REL * (g.abs() * u.abs() + r.abs()) + 1e-6)
    return _verdict(d.float(), r, tol, frob_tol)


def _verdict(dd, r, tol, frob_tol):
    if dd.shape != r.shape:
        raise ValueError(f"shape mismatch {tuple(dd.shape)} vs {tuple(r.shape)}")
    err = (dd - r).abs()
    n_bad = int((err > tol).sum())
    frob = rel_frobenius(dd, r)
    worst = float((err / tol.clamp_min(1e-30)).max()) if err.numel() else 0.0
    return {"ok": n_bad == 0 and frob <= frob_tol, "n_bad": n_bad, "frob": frob,
            "worst_ratio": worst, "max_abs_err": float(err.max()) if err.numel() else 0.0}
