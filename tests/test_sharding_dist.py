"""Multi-rank host logic on CPU ranks (gloo, world size 2): the M-shard and split-K
decompositions reproduce the full product computed by the oracle."""
import os
import socket

import pytest
import torch
import torch.distributed as dist
import torch.multiprocessing as mp

from cutedsl_pingpong_gemm_b200.sharding import (MShardedGemm, SplitKGemm, k_ranges,
                                                  peer_row_starts, reduce_scatter_rows, row_range)


def test_row_range_partitions():
    for m in (0, 1, 127, 128, 129, 1000, 16384, 16384 + 5):
        for world in (1, 2, 3, 4, 8):
            ranges = [row_range(m, world, r) for r in range(world)]
            covered = [i for s, e in ranges for i in range(s, e)] if m < 5000 else None
            if covered is not None:
                assert covered == list(range(m))
            assert ranges[0][0] == 0 and ranges[-1][1] == m
            for (s0, e0), (s1, e1) in zip(ranges, ranges[1:]):
                assert e0 == s1 and s0 <= e0
            for s, _ in ranges:
                assert s % 128 == 0 or s == m
    # The LLM shape splits into equal 2048-row shards on 8 GPUs.
    assert [row_range(16384, 8, r) for r in range(8)] == [(2048 * r, 2048 * (r + 1)) for r in range(8)]


def test_peer_row_starts():
    """Row blocks of the peer reduce-scatter: contiguous, from 0 to M, interior boundaries on
    128-row tiles (or at M for ranks left without rows), as cpg_gemm_run_reduce_scatter
    requires."""
    for m in (1, 129, 600, 2048, 16384 + 40):
        for world in (1, 2, 3, 8):
            st = peer_row_starts(m, world)
            assert len(st) == world + 1 and st[0] == 0 and st[-1] == m
            assert all(a <= b for a, b in zip(st, st[1:]))
            assert all(x % 128 == 0 or x == m for x in st[1:-1])
            assert [(st[q], st[q + 1]) for q in range(world)] == \
                [row_range(m, world, q) for q in range(world)]


def test_k_ranges_aligned():
    for k in (64, 1000, 8192, 131072):
        for parts in (1, 2, 8):
            rs = k_ranges(k, parts)
            assert rs[0][0] == 0 and rs[-1][1] == k
            assert all(s % 64 == 0 or s == k for s, _ in rs)
    assert k_ranges(131072, 8) == [(16384 * p, 16384 * (p + 1)) for p in range(8)]


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def _worker(rank, world, port, q):
    os.environ["MASTER_ADDR"] = "127.0.0.1"
    os.environ["MASTER_PORT"] = str(port)
    dist.init_process_group("gloo", rank=rank, world_size=world)
    try:
        from oracle import gemm_ref
        torch.manual_seed(0)
        m, n, k = 300, 96, 4 * 64 + 8
        a, b, bias = gemm_ref.make_inputs(m, n, k, seed=5, with_bias=True)
        full = gemm_ref.reference(a, b, bias)

        # M-shard: each rank computes its rows with the oracle standing in for the GPU GEMM.
        calls = []

        class FakeGemm:
            def __call__(self, a_s, b_, d_s, stream=None, *, bias=None, alpha=1.0):
                calls.append(a_s.shape[0])
                d_s.copy_(gemm_ref.reference(a_s, b_, bias, alpha))

        sh = MShardedGemm(FakeGemm(), world, rank)
        s, e = sh.rows(m)
        d_s = torch.empty(e - s, n)
        sh(a[s:e], b, d_s, bias=bias)
        sizes = [row_range(m, world, r)[1] - row_range(m, world, r)[0] for r in range(world)]
        per = max(sizes)
        padded = torch.zeros(per, n)
        padded[: e - s] = d_s
        gathered = [torch.empty(per, n) for _ in range(world)]
        dist.all_gather(gathered, padded)
        got = torch.cat([g[:sz] for g, sz in zip(gathered, sizes)])
        assert torch.equal(got, full)
        assert calls == [e - s]

        # Split-K: partial over this rank's K range, reduce-scatter rows.
        def partial(a_k, b_k):
            return torch.matmul(a_k.double(), b_k.double().t())

        sk = SplitKGemm(world, rank, partial)
        ks, ke = sk.k_range(k)
        rows = sk(a[:, ks:ke], b[:, ks:ke], m, n)
        s, e = row_range(m, world, rank)
        want = torch.matmul(a.double(), b.double().t())[s:e]
        assert torch.allclose(rows, want, rtol=1e-12, atol=1e-9)

        # Chunked split-K (reduce-scatter per column chunk): same rows, ragged last chunk, and a
        # cast that writes each chunk's columns of the preallocated output.
        n2 = 700
        b2 = torch.randn(n2, k, generator=torch.Generator().manual_seed(6)).to(torch.bfloat16)
        want2 = torch.matmul(a.double(), b2.double().t())[s:e]
        sk3 = SplitKGemm(world, rank, partial, chunks=3)
        assert sk3.column_chunks(n2) == [(0, 256), (256, 512), (512, 700)]
        rows3 = sk3(a[:, ks:ke], b2[:, ks:ke], m, n2)
        assert torch.allclose(rows3, want2, rtol=1e-12, atol=1e-9)
        seen = []

        def cast(r, cs, ce, out=None):
            seen.append((cs, ce))
            y = (2 * r).float()
            if out is None:
                return y
            out.copy_(y)
            return out

        skc = SplitKGemm(world, rank, partial, cast, chunks=3, out_dtype=torch.float32)
        rc = skc(a[:, ks:ke], b2[:, ks:ke], m, n2)
        assert rc.dtype == torch.float32 and seen == skc.column_chunks(n2)
        assert torch.allclose(rc.double(), 2 * want2, rtol=1e-6, atol=1e-4)
        q.put((rank, "ok"))
    except Exception as ex:  # pragma: no cover - reported through the queue
        q.put((rank, repr(ex)))
    finally:
        dist.destroy_process_group()


def test_gloo_two_ranks_shard_and_splitk():
    world = 2
    ctx = mp.get_context("spawn")
    q = ctx.Queue()
    port = _free_port()
    procs = [ctx.Process(target=_worker, args=(r, world, port, q)) for r in range(world)]
    for p in procs:
        p.start()
    results = [q.get(timeout=120) for _ in range(world)]
    for p in procs:
        p.join(timeout=60)
    assert sorted(results) == [(0, "ok"), (1, "ok")], results
