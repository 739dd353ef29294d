"""The allocation-free split-K entry point (cpg_gemm_splitk_static) against the plan-based one.

Some callers of this library cannot call cudaMalloc (an embedding runtime whose device memory is
carved up in advance, or code that must not allocate while work is captured into a CUDA graph).
For them cpg_gemm_splitk_static keeps the FP32 partial-sum buffer of split-K in a static device
array compiled into the library.  This test calls it through the C ABI twice in a row (a larger
problem, then a smaller one, so the second call must not see the first call's leftover sums) and
checks each output against the existing entry point (cpg_gemm_run with split_k into an FP32 D,
then the BF16 cast), within the tolerance of the other GPU tests.  It also checks that a problem
larger than the static array is rejected with a clear error.

This file is collected last so that a run stopping at the first failure has run everything else.
"""
import ctypes

import pytest
import torch

from cutedsl_pingpong_gemm_b200 import GemmSM90, _lib
from cutedsl_pingpong_gemm_b200.quant import cast_f32_bf16
from oracle import gemm_ref

pytestmark = pytest.mark.gpu

STATIC_SCRATCH_FLOATS = (16 << 20) // 4


def _config(tile_n, cluster_m):
    return _lib.GemmConfigC(128, tile_n, 128, 32, cluster_m, 1, 1, 1, 1, 4 if cluster_m == 1 else 6,
                            2, 1, 0, 1, 0, 8)


def _static_call(lib, a, b, d, split_k, tile_n, cluster_m, bias=None, scale_a=None,
                 scale_b=None):
    m, k = a.shape
    n = b.shape[0]
    cfg = _config(tile_n, cluster_m)
    dtype_ab = _lib.CPG_DTYPE_E4M3 if a.dtype == torch.float8_e4m3fn else _lib.CPG_DTYPE_BF16
    prob = _lib.GemmProblemC(m, n, k, a.stride(0), b.stride(0), d.stride(0), dtype_ab,
                             _lib.CPG_DTYPE_BF16, _lib.CPG_SCALE_TENSOR, split_k)
    epi = _lib.EpilogueC(1.0, None if bias is None else bias.data_ptr(),
                         None if scale_a is None else scale_a.data_ptr(),
                         None if scale_b is None else scale_b.data_ptr())
    stream = torch.cuda.current_stream().cuda_stream
    return lib.cpg_gemm_splitk_static(ctypes.byref(cfg), ctypes.byref(prob), a.data_ptr(),
                                      b.data_ptr(), d.data_ptr(), ctypes.byref(epi), stream)


def _existing_path(a, b, split_k, tile_n, cluster_m, bias=None, scale_a=None, scale_b=None):
    """The plan-based entry points: cpg_gemm_run (split-K into FP32 D), then cpg_cast_f32_bf16.
    FP32 rows are padded to 16 bytes (a TMA rule) when N is not a multiple of 4."""
    m, n = a.shape[0], b.shape[0]
    gemm = GemmSM90((128, tile_n), (128, 32), (cluster_m, 1, 1), (1, 1),
                    ab_stage=4 if cluster_m == 1 else 6, reuse_ab=False, is_persistent=True)
    d32 = torch.empty(m, (n + 3) // 4 * 4, dtype=torch.float32, device="cuda")[:, :n]
    gemm(a, b, d32, None, split_k=split_k, scale_a=scale_a, scale_b=scale_b)
    return cast_f32_bf16(d32, bias)


@pytest.mark.parametrize("cluster_m", [1, 2])
def test_static_scratch_entry_point_matches_plan_path(lib, cluster_m):
    problems = [  # (m, n, k, split_k, tile_n): a larger problem first, then a smaller one
        (384, 2048, 4096 + 64, 4, 256),
        (200, 520, 1000 + 8, 3, 128),
    ]
    for i, (m, n, k, split_k, tile_n) in enumerate(problems):
        a, b, bias = gemm_ref.make_inputs(m, n, k, seed=40 + i, b_scale=k ** -0.5, with_bias=True)
        da, db, dbias = a.cuda(), b.cuda(), bias.cuda()
        d_static = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
        rc = _static_call(lib, da, db, d_static, split_k, tile_n, cluster_m, dbias)
        assert rc == _lib.CPG_OK, lib.cpg_last_error_message()
        d_plan = _existing_path(da, db, split_k, tile_n, cluster_m, dbias)
        torch.cuda.synchronize()
        got, want = d_static.cpu(), d_plan.cpu()
        # Both must meet the GPU tests' tolerance against the fp32 oracle ...
        for out in (got, want):
            res = gemm_ref.check(out, a, b, bias=bias)
            assert res["ok"], (i, res)
        # ... and agree with each other within twice that element-wise bound (the two runs add
        # the same partial sums, possibly in another order).
        r = gemm_ref.reference(a, b, bias)
        s = gemm_ref.abs_product(a, b)
        bound = 2 * gemm_ref.elementwise_bound(r, s, k, bias=bias)
        assert bool(((got.float() - want.float()).abs() <= bound).all()), i
        assert gemm_ref.rel_frobenius(got, want.float()) <= gemm_ref.FROB_TOL_BF16


def test_static_scratch_rejects_oversized_problem(lib):
    m, n, k = 1024, 8192, 128  # M * N = 8 Mi floats > the 4 Mi the static array holds
    assert m * n > STATIC_SCRATCH_FLOATS
    a = torch.zeros(m, k, dtype=torch.bfloat16, device="cuda")
    b = torch.zeros(n, k, dtype=torch.bfloat16, device="cuda")
    d = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
    rc = _static_call(lib, a, b, d, 2, 256, 1)
    assert rc == _lib.CPG_ERR_INVALID_SHAPE
    msg = lib.cpg_last_error_message().decode()
    assert "static scratch" in msg and str(m * n * 4) in msg


def test_static_scratch_padded_rows_fp8_and_unsplit_after_split(lib):
    """Cases beyond the BF16 pair above, each against the plan path in the same way: N not a
    multiple of 4 (the scratch rows are padded to 16 bytes, D has its own wider row stride), FP8
    E4M3 operands with per-tensor scales, and split_k = 1 (no scratch: the GEMM stores D's FP32
    sums straight into the array, no clearing) right after a split call left sums there."""
    from cutedsl_pingpong_gemm_b200.quant import quantize_e4m3
    cases = [  # (m, n, k, split_k, tile_n, cluster_m, fp8)
        (256, 517, 2048, 3, 128, 1, False),
        (320, 1024, 4096, 4, 256, 2, True),
        (320, 1024, 1024, 1, 256, 2, False),
        (130, 517, 640, 1, 128, 1, True),
    ]
    for i, (m, n, k, split_k, tile_n, cluster_m, fp8) in enumerate(cases):
        a, b, bias = gemm_ref.make_inputs(m, n, k, seed=60 + i, b_scale=k ** -0.5, with_bias=True)
        da, db, dbias = a.cuda(), b.cuda(), bias.cuda()
        sa = sb = None
        if fp8:
            da, sa = quantize_e4m3(da)
            db, sb = quantize_e4m3(db)
            a = da.cpu().float() * sa.cpu()  # the dequantised operands are the oracle's inputs
            b = db.cpu().float() * sb.cpu()
        ldd = (n + 7) // 8 * 8 + 8  # a row stride wider than N
        d_static = torch.full((m, ldd), float("nan"), dtype=torch.bfloat16, device="cuda")[:, :n]
        rc = _static_call(lib, da, db, d_static, split_k, tile_n, cluster_m, dbias, sa, sb)
        assert rc == _lib.CPG_OK, lib.cpg_last_error_message()
        d_plan = _existing_path(da, db, split_k, tile_n, cluster_m, dbias, sa, sb)
        torch.cuda.synchronize()
        got, want = d_static.cpu(), d_plan.cpu()
        frob = gemm_ref.FROB_TOL_FP8 if fp8 else gemm_ref.FROB_TOL_BF16
        for out in (got, want):
            res = gemm_ref.check(out, a, b, bias=bias, frob_tol=frob)
            assert res["ok"], (i, res)
        r = gemm_ref.reference(a, b, bias)
        s = gemm_ref.abs_product(a, b)
        bound = 2 * gemm_ref.elementwise_bound(r, s, k, bias=bias)
        assert bool(((got.float() - want.float()).abs() <= bound).all()), i
