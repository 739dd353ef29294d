"""The small-M kernel (split_k = CPG_SPLIT_K_DECODE) on the GPU, through the public API / C ABI.

BASELINE config 5 (decode-like M in {16, 64, 128} at N = K = 8192) and ragged shapes around it:
a CTA computes D^T for 128 rows of B, the K range of a tile is split over a cluster of 1, 2 or 4
CTAs (or CTA pairs, one cta_group::2 MMA per k-step for 256 rows) and the partial sums are added
in distributed shared memory.  Checked against the fp32 CPU
oracle with the tolerance of the other GPU tests (relative Frobenius <= 1e-2 for BF16 output,
3e-2 for FP8 E4M3 operands, and the element-wise bound |D - R| <= 2^-8 |R| + K 2^-23 (|A| |B|^T)),
for every cluster size the plan can pick, M not a multiple of 16, ragged N and K, FP32 output,
bias, alpha, K = 0, CUDA-graph replay, chains of calls each reading the previous one's output
(programmatic dependent launch), and the rejection of what the kernel does not do.
"""
import pytest
import torch

from cutedsl_pingpong_gemm_b200 import GemmSM90, _lib, compile as cpg_compile
from cutedsl_pingpong_gemm_b200.quant import quantize_e4m3
from oracle import gemm_ref

pytestmark = pytest.mark.gpu

DECODE = _lib.CPG_SPLIT_K_DECODE


def make_gemm():
    return GemmSM90(tile_shape_mn=(128, 128), epi_tile_mn=(128, 32), cluster_shape_mnk=(1, 1, 1),
                    atom_layout_mn=(1, 1), ab_stage=4, reuse_ab=False, is_persistent=True)


def run(m, n, k, seed, bias=True, alpha=1.0, out_dtype=torch.bfloat16):
    a, b, bb = gemm_ref.make_inputs(m, n, k, seed=seed, b_scale=max(k, 1) ** -0.5,
                                    with_bias=bias)
    da, db = a.cuda(), b.cuda()
    d = torch.full((m, n), float("nan"), dtype=out_dtype, device="cuda")
    compiled = cpg_compile(make_gemm(), da, db, d)
    compiled(da, db, d, None, bias=None if bb is None else bb.cuda(), alpha=alpha, split_k=DECODE)
    torch.cuda.synchronize()
    plan = compiled.plan_for(da, db, d, 0, DECODE)
    assert plan.status() == 0
    return d.cpu(), a, b, bb, plan


@pytest.mark.parametrize("m", [16, 64, 128])
def test_baseline_small_m_configs(m):
    """BASELINE config 5 exactly: M x 8192 x 8192, N(0,1)/sqrt(K) entries, BF16 out with bias.
    64 tiles of 128 rows of B, each on 2 CTAs (K split in two): a cluster of 2."""
    d, a, b, bb, plan = run(m, 8192, 8192, seed=m)
    res = gemm_ref.check(d, a, b, bias=bb)
    assert res["ok"], res
    info = plan.launch_info()
    assert info["grid"][:2] == (2, 64) and info["cluster"][0] == 2


@pytest.mark.parametrize("m,n,k,cluster,tiles", [
    (1, 520, 4096 + 64, 4, 5),       # 5 tiles of 128 rows: 4 CTAs per cluster
    (17, 520, 128, 2, 5),            # 2 k-blocks: at most 2 CTAs
    (33, 128 * 3 + 8, 64, 1, 4),     # one k-block: no split
    (100, 16384, 1000 + 8, 1, 128),  # 128 tiles: no room for a second CTA per tile
    (128, 9472, 3000 + 40, 2, 74),   # 74 tiles x 2 CTAs fill the 148 SMs
    (5, 4096, 130 * 64, 4, 32),      # 32 tiles x 4
    (64, 1000, 1000 + 8, 4, 8),      # ragged N: the last tile has 104 rows
    (80, 2056, 640, 4, 17),          # 10 k-blocks over 4 CTAs: 3, 3, 3, 1; last tile 8 rows
])
def test_ragged_shapes_and_cluster_sizes(m, n, k, cluster, tiles):
    d, a, b, bb, plan = run(m, n, k, seed=m + n + k)
    res = gemm_ref.check(d, a, b, bias=bb)
    assert res["ok"], (m, n, k, res)
    info = plan.launch_info()
    assert info["cluster"][0] == cluster and info["grid"][1] == tiles


@pytest.mark.parametrize("m,n,k,env,cluster", [
    (16, 8192, 8192, {"CPG_DECODE_PAIR": "1"}, 4),      # 32 pair tiles x 2 pairs
    (100, 1000, 2048, {"CPG_DECODE_PAIR": "1"}, 8),     # 4 pair tiles x 4 pairs, ragged N
    (128, 4096, 4096 + 64, {"CPG_DECODE_PAIR": "1", "CPG_DECODE_ROTATE": "0"}, 8),
    (64, 2056, 640, {"CPG_DECODE_ROTATE": "0", "CPG_DECODE_SPIN": "0"}, 4),
    (48, 4096, 4096, {"CPG_DECODE_PDL": "0"}, 4),         # launched without the dependency
    (128, 8192, 8192, {"CPG_DECODE_STASYNC": "1"}, 2),    # partial sums by per-thread st.async
    (5, 4096, 8320, {"CPG_DECODE_STASYNC": "1"}, 4),      # the same into 3 peers
])
def test_other_variants(monkeypatch, m, n, k, env, cluster):
    """The CTA-pair form (256-row tiles, one cta_group::2 MMA per k-step for both CTAs of a pair),
    every tile walking its K range from the start, sleeping pipeline waits, the launch without
    the programmatic dependency and the partial sums sent by per-thread st.async: the same
    checks."""
    for key, value in env.items():
        monkeypatch.setenv(key, value)
    d, a, b, bb, plan = run(m, n, k, seed=m + k)
    res = gemm_ref.check(d, a, b, bias=bb)
    assert res["ok"], (m, n, k, env, res)
    assert plan.launch_info()["cluster"][0] == cluster


def test_fp32_output_and_alpha():
    m, n, k = 48, 2048 + 128, 4096
    d, a, b, _, _ = run(m, n, k, seed=3, bias=False, alpha=0.5, out_dtype=torch.float32)
    r = gemm_ref.reference(a, b, alpha=0.5)
    s = gemm_ref.abs_product(a, b)
    assert bool(((d - r).abs() <= 0.5 * k * gemm_ref.ACC_SLACK_PER_K * s + 1e-6).all())


@pytest.mark.parametrize("m", [16, 128])
def test_fp8_per_tensor_scales(m):
    n, k = 4096, 8192
    g = torch.Generator().manual_seed(m)
    a = torch.randn(m, k, generator=g).to(torch.bfloat16).cuda()
    b = torch.randn(n, k, generator=g).to(torch.bfloat16).cuda()
    qa, sa = quantize_e4m3(a)
    qb, sb = quantize_e4m3(b)
    d = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    make_gemm()(qa, qb, d, None, scale_a=sa, scale_b=sb, split_k=DECODE)
    torch.cuda.synchronize()
    res = gemm_ref.check(d.cpu(), qa.cpu().float() * sa.cpu(), qb.cpu().float() * sb.cpu(),
                         frob_tol=gemm_ref.FROB_TOL_FP8)
    assert res["ok"], res


def test_k_zero_gives_bias():
    m, n = 7, 256
    bias = torch.randn(n).to(torch.bfloat16).cuda()
    a = torch.empty(m, 0, dtype=torch.bfloat16, device="cuda")
    b = torch.empty(n, 0, dtype=torch.bfloat16, device="cuda")
    d = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    make_gemm()(a, b, d, None, bias=bias, split_k=DECODE)
    torch.cuda.synchronize()
    assert torch.equal(d, bias.expand(m, n))


def test_repeated_calls_and_graph_replay_are_bitwise_stable():
    """No state survives a call (no workspace): eager calls and replays of a captured call give
    identical bytes."""
    m, n, k = 64, 8192, 8192
    a, b, bias = gemm_ref.make_inputs(m, n, k, seed=11, b_scale=k ** -0.5, with_bias=True)
    da, db, dbias = a.cuda(), b.cuda(), bias.cuda()
    d = torch.empty(m, n, dtype=torch.bfloat16, device="cuda")
    compiled = cpg_compile(make_gemm(), da, db, d)
    compiled(da, db, d, None, bias=dbias, split_k=DECODE)
    torch.cuda.synchronize()
    ref = d.clone()
    assert gemm_ref.check(ref.cpu(), a, b, bias=bias)["ok"]
    compiled(da, db, d, None, bias=dbias, split_k=DECODE)
    torch.cuda.synchronize()
    assert torch.equal(d, ref)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        compiled(da, db, d, s, bias=dbias, split_k=DECODE)
    for _ in range(3):
        d.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(d, ref)


@pytest.mark.parametrize("graph", [False, True])
def test_chained_calls_wait_for_their_producer(graph):
    """Each call is a programmatic dependent of the previous kernel on the stream: it may start
    (barriers, TMEM, an L2 prefetch of B) while that kernel runs, but must read A only after it
    has completed.  A chain D1 = A B1^T, D2 = D1 B2^T, D3 = D2 B3^T on one stream, D1 and D2
    poisoned with NaN just before, checked link by link against the oracle on the GPU's own
    inputs; eagerly and replayed from one CUDA graph."""
    m = 16
    dims = [4096, 4096, 2048, 1024]  # K of the first link, then each link's N
    g = torch.Generator().manual_seed(21)
    a = torch.randn(m, dims[0], generator=g).to(torch.bfloat16)
    bs = [(torch.randn(dims[i + 1], dims[i], generator=g) * dims[i] ** -0.5).to(torch.bfloat16)
          for i in range(3)]
    da, dbs = a.cuda(), [b.cuda() for b in bs]
    ds = [torch.empty(m, dims[i + 1], dtype=torch.bfloat16, device="cuda") for i in range(3)]
    compiled = [cpg_compile(make_gemm(), da if i == 0 else ds[i - 1], dbs[i], ds[i])
                for i in range(3)]
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())

    def chain():
        with torch.cuda.stream(s):
            for d in ds:
                d.fill_(float("nan"))
            for i in range(3):
                compiled[i](da if i == 0 else ds[i - 1], dbs[i], ds[i], s, split_k=DECODE)

    if graph:
        chain()  # plans and tensor maps before capture
        torch.cuda.synchronize()
        cg = torch.cuda.CUDAGraph()
        with torch.cuda.graph(cg, stream=s):
            chain()
        for _ in range(3):
            cg.replay()
    else:
        for _ in range(3):
            chain()
    torch.cuda.synchronize()
    inputs = [a] + [d.cpu() for d in ds[:2]]
    for i in range(3):
        res = gemm_ref.check(ds[i].cpu(), inputs[i], bs[i])
        assert res["ok"], (i, res)


def test_rejects_what_the_kernel_does_not_do():
    m, n, k = 200, 512, 256
    a = torch.zeros(m, k, dtype=torch.bfloat16, device="cuda")
    b = torch.zeros(n, k, dtype=torch.bfloat16, device="cuda")
    d = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
    with pytest.raises(_lib.CpgError) as e:  # M > 128
        make_gemm()(a, b, d, None, split_k=DECODE)
    assert e.value.code == _lib.CPG_ERR_INVALID_SHAPE
    with pytest.raises(_lib.CpgError) as e:  # fused activation
        make_gemm()(a[:64], b, d[:64], None, split_k=DECODE, activation="relu")
    assert e.value.code == _lib.CPG_ERR_UNSUPPORTED
