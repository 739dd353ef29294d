"""Split-K reduce-scatter through the GEMM epilogue (cpg_gemm_run_reduce_scatter +
cpg_peer_finish) on one GPU: the ranks are emulated in one process, their GEMMs launched one
after another on one stream and the finishes after all of them, so no kernel waits for work that
has not been launched before it.  The cross-process form (CUDA IPC, NVLink) is tested in
test_multi_gpu.py.

Tolerance: relative Frobenius <= 1e-2 and the element-wise bound of oracle.gemm_ref.check (the
split partial sums are FP32, added in any order, then rounded once to BF16).
"""
import ctypes

import pytest
import torch

from cutedsl_pingpong_gemm_b200 import GemmSM90, RasterOrder, _lib
from cutedsl_pingpong_gemm_b200.gemm_base import _Plan
from cutedsl_pingpong_gemm_b200.sharding import k_ranges, peer_row_starts
from oracle import gemm_ref

pytestmark = pytest.mark.gpu


def make_gemm(tile_n, cluster, dynamic):
    return GemmSM90(tile_shape_mn=(128, tile_n), epi_tile_mn=(128, 32), cluster_shape_mnk=cluster,
                    atom_layout_mn=(1, 1), ab_stage=3 if tile_n == 512 else 4, epi_stage=2,
                    raster_order=RasterOrder.AlongN, reuse_ab=False, is_persistent=True,
                    dynamic_scheduler=dynamic)


class Emulated:
    """`world` ranks in one process: buffers, counters, one plan per rank's K range."""

    def __init__(self, gemm, m, n, k, world, split, a, b):
        self.lib = _lib.load()
        self.m, self.n, self.world = m, n, world
        self.starts = peer_row_starts(m, world)
        self.bufs = [torch.zeros(max(self.starts[q + 1] - self.starts[q], 1), n,
                                 dtype=torch.float32, device="cuda") for q in range(world)]
        self.counts = torch.zeros(world * 16, dtype=torch.int32, device="cuda")
        self.status = torch.zeros(1, dtype=torch.int32, device="cuda")
        self.parts = []
        for r, (ks, ke) in enumerate(k_ranges(k, world)):
            ar = a[:, ks:ke].contiguous().cuda()
            br = b[:, ks:ke].contiguous().cuda()
            plan = _Plan(gemm, m, n, ke - ks, max(ke - ks, 8), max(ke - ks, 8), n, 0,
                         _lib.CPG_DTYPE_BF16, _lib.CPG_DTYPE_F32, 0, split)
            rs = _lib.ReduceScatterC()
            rs.ranks, rs.rank, rs.ld = world, r, n
            for q in range(world + 1):
                rs.row_start[q] = self.starts[q]
            for q in range(world):
                rs.dst[q] = self.bufs[q].data_ptr()
                rs.count[q] = self.counts.data_ptr() + 64 * q
            self.parts.append((ar, br, plan, rs))
        self.expected = [0] * world
        for _, _, plan, rs in self.parts:
            arr = (ctypes.c_uint32 * world)()
            _lib.check(self.lib.cpg_gemm_rs_arrivals(plan.handle, ctypes.byref(rs), arr))
            for q in range(world):
                self.expected[q] += arr[q]
        self.calls = 0

    def gemms(self):
        epi = _lib.EpilogueC(1.0, None, None, None, 0.0, 0, None, 0, 0)
        st = torch.cuda.current_stream().cuda_stream
        for ar, br, plan, rs in self.parts:
            _lib.check(self.lib.cpg_gemm_run_reduce_scatter(
                plan.handle, ar.data_ptr(), br.data_ptr(), ctypes.byref(rs), ctypes.byref(epi),
                st), "run_reduce_scatter")
        self.calls += 1

    def finish(self, q, out, bias=None, extra=0, timeout_ms=2000):
        st = torch.cuda.current_stream().cuda_stream
        rows = self.starts[q + 1] - self.starts[q]
        target = (self.calls * self.expected[q] + extra) & 0xFFFFFFFF
        _lib.check(self.lib.cpg_peer_finish(
            self.bufs[q].data_ptr(), self.n, self.counts.data_ptr() + 64 * q, target, rows,
            self.n, out.data_ptr(), self.n, None if bias is None else bias.data_ptr(),
            self.status.data_ptr(), timeout_ms, st), "peer_finish")


@pytest.mark.parametrize("tile_n,cluster,dynamic,world,split", [
    (256, (2, 1, 1), False, 2, 2), (256, (2, 1, 1), True, 3, 1), (128, (1, 1, 1), True, 2, 3),
    (512, (2, 1, 1), False, 4, 1)])
def test_reduce_scatter_rounds(tile_n, cluster, dynamic, world, split):
    m, n, k = 128 * 5 - 40, 1000, 2048
    a, b, bias = gemm_ref.make_inputs(m, n, k, seed=91 + world, b_scale=k ** -0.5, with_bias=True)
    em = Emulated(make_gemm(tile_n, cluster, dynamic), m, n, k, world, split, a, b)
    dbias = bias.cuda()
    for _ in range(2):  # the second round checks the running count and the cleared buffers
        em.gemms()
        outs = []
        for q in range(world):
            rows = em.starts[q + 1] - em.starts[q]
            out = torch.full((max(rows, 1), n), float("nan"), dtype=torch.bfloat16, device="cuda")
            em.finish(q, out, dbias)
            outs.append(out)
        torch.cuda.synchronize()
        assert int(em.status.item()) == 0
        for q in range(world):
            s, e = em.starts[q], em.starts[q + 1]
            if e > s:
                res = gemm_ref.check(outs[q][: e - s].cpu(), a[s:e], b, bias=bias)
                assert res["ok"], (q, res)
            assert int(torch.count_nonzero(em.bufs[q]).item()) == 0


@pytest.mark.parametrize("m,n,k,dynamic,split,rounds", [
    (512, 768, 8192, False, 2, 3),              # 4 row tiles over 8 ranks: ranks 4-7 own no rows
    (128 * 17 - 40, 1000, 6144, True, 0, 2)])   # ragged M, bias, the automatic in-GPU split
def test_reduce_scatter_eight_ranks(m, n, k, dynamic, split, rounds):
    """The peer reduce-scatter shapes of the 8-process test in test_multi_gpu.py (its GEMM
    arguments, K split over 8 ranks, each rank's K range split again inside the GPU), with the 8
    ranks emulated on one GPU: the arrival counts of every owner, ranks without rows, the
    running count over repeated calls and the cleared buffers."""
    from types import SimpleNamespace
    from cutedsl_pingpong_gemm_b200.gemm_base import CompiledGemm
    from cutedsl_pingpong_gemm_b200.sharding import PeerSplitK
    world = 8
    gemm = GemmSM90((128, 256), (128, 32), (2, 1, 1), (1, 1), ab_stage=6, reuse_ab=False,
                    is_persistent=True, dynamic_scheduler=dynamic)
    if split == 0:
        ks, ke = k_ranges(k, world)[0]
        split = PeerSplitK._split(SimpleNamespace(gemm=gemm, local_split_k=0), CompiledGemm(gemm),
                                  m, n, ke - ks)
    a, b, bias = gemm_ref.make_inputs(m, n, k, seed=7, b_scale=k ** -0.5, with_bias=dynamic)
    em = Emulated(gemm, m, n, k, world, split, a, b)
    dbias = bias.cuda() if bias is not None else None
    for _ in range(rounds):
        em.gemms()
        outs = []
        for q in range(world):
            rows = em.starts[q + 1] - em.starts[q]
            out = torch.full((max(rows, 1), n), float("nan"), dtype=torch.bfloat16, device="cuda")
            em.finish(q, out, dbias)
            outs.append(out)
        torch.cuda.synchronize()
        assert int(em.status.item()) == 0
        for q in range(world):
            s, e = em.starts[q], em.starts[q + 1]
            if e > s:
                res = gemm_ref.check(outs[q][: e - s].cpu(), a[s:e], b, bias=bias)
                assert res["ok"], (q, split, res)
            assert int(torch.count_nonzero(em.bufs[q]).item()) == 0


def test_finish_times_out_when_arrivals_are_missing():
    """A finish whose target is never reached gives up after its limit with a status code and
    writes nothing; the context stays usable."""
    m, n, k = 256, 256, 512
    a, b, _ = gemm_ref.make_inputs(m, n, k, seed=95)
    em = Emulated(make_gemm(256, (1, 1, 1), False), m, n, k, 1, 1, a, b)
    em.gemms()
    out = torch.full((m, n), float("nan"), dtype=torch.bfloat16, device="cuda")
    em.finish(0, out, extra=1, timeout_ms=200)  # one arrival more than any rank makes
    torch.cuda.synchronize()
    assert int(em.status.item()) == 0x100 | 10
    assert bool(torch.isnan(out.float()).all())
    # The same buffers finish correctly once the target matches.
    em.status.zero_()
    em.finish(0, out)
    torch.cuda.synchronize()
    assert int(em.status.item()) == 0
    res = gemm_ref.check(out.cpu(), a, b)
    assert res["ok"], res


def test_reduce_scatter_rejections():
    m, n, k = 256, 258, 512
    gemm = make_gemm(256, (1, 1, 1), False)
    lib = _lib.load()
    plan = _Plan(gemm, m, n, k, k, k, 260, 0, _lib.CPG_DTYPE_BF16, _lib.CPG_DTYPE_F32, 0, 1)
    rs = _lib.ReduceScatterC()
    buf = torch.zeros(m, 260, dtype=torch.float32, device="cuda")
    cnt = torch.zeros(16, dtype=torch.int32, device="cuda")
    rs.ranks, rs.rank, rs.ld = 1, 0, 260
    rs.row_start[0], rs.row_start[1] = 0, m
    rs.dst[0], rs.count[0] = buf.data_ptr(), cnt.data_ptr()
    arr = (ctypes.c_uint32 * 1)()
    assert lib.cpg_gemm_rs_arrivals(plan.handle, ctypes.byref(rs), arr) == _lib.CPG_ERR_ALIGNMENT
    plan16 = _Plan(gemm, m, 256, k, k, k, 256, 0, _lib.CPG_DTYPE_BF16, _lib.CPG_DTYPE_BF16, 0, 1)
    rs.ld = 256
    assert lib.cpg_gemm_rs_arrivals(plan16.handle, ctypes.byref(rs), arr) == \
        _lib.CPG_ERR_UNSUPPORTED  # BF16 output
    plan32 = _Plan(gemm, m, 256, k, k, k, 256, 0, _lib.CPG_DTYPE_BF16, _lib.CPG_DTYPE_F32, 0, 1)
    rs.row_start[1] = m - 1
    assert lib.cpg_gemm_rs_arrivals(plan32.handle, ctypes.byref(rs), arr) == \
        _lib.CPG_ERR_INVALID_SHAPE  # rows must run to M
    rs.row_start[1] = m
    rs.ranks = 9
    assert lib.cpg_gemm_rs_arrivals(plan32.handle, ctypes.byref(rs), arr) == \
        _lib.CPG_ERR_INVALID_CONFIG
