"""Multi-GPU paths on real GPUs (NCCL): M-sharding with B replicated, split-K with an NCCL
reduce-scatter of fp32 partials followed by the BF16 cast kernel, and split-K whose GEMM epilogue
adds the partials into the owning ranks' memory over NVLink (PeerSplitK).

Runs one process per visible GPU (at least two, otherwise skipped) with a short process-group
timeout; each rank checks its rows against the fp32 CPU oracle.  NVLS is switched off
(NCCL_NVLS_ENABLE=0) as for every multi-rank test on this pool.
"""
import os
import socket
import subprocess
import sys
import textwrap

import pytest
import torch

from conftest import ROOT

pytestmark = pytest.mark.gpu

WORKER = textwrap.dedent(r'''
    import datetime, os, sys
    sys.path.insert(0, sys.argv[1])
    import torch, torch.distributed as dist
    rank, world = int(os.environ["RANK"]), int(os.environ["WORLD_SIZE"])
    torch.cuda.set_device(rank)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=60),
                            device_id=torch.device("cuda", rank))
    from cutedsl_pingpong_gemm_b200 import GemmSM90
    from cutedsl_pingpong_gemm_b200.sharding import MShardedGemm, SplitKGemm, k_ranges, row_range
    from oracle import gemm_ref
    ok = True
    # M-shard: LLM-like shape scaled down, bias, B replicated, no collective on the data path.
    m, n, k = 1024 + 128 * world, 1536, 1024
    a, b, bias = gemm_ref.make_inputs(m, n, k, seed=3, b_scale=0.02, with_bias=True)
    gemm = GemmSM90((128, 256), (128, 32), (2, 1, 1), (1, 1), ab_stage=6, reuse_ab=False,
                    is_persistent=True)
    sh = MShardedGemm(gemm, world, rank)
    s, e = sh.rows(m)
    d = torch.empty(e - s, n, dtype=torch.bfloat16, device="cuda")
    sh(a[s:e].cuda(), b.cuda(), d, bias=bias.cuda())
    torch.cuda.synchronize()
    res = gemm_ref.check(d.cpu(), a[s:e], b, bias=bias)
    ok &= res["ok"]
    # Split-K over ranks: tall K, fp32 partials, NCCL reduce-scatter, cast to BF16.
    m2, n2, k2 = 512, 768, 8192
    a2, b2, _ = gemm_ref.make_inputs(m2, n2, k2, seed=5, b_scale=k2 ** -0.5)
    ks, ke = k_ranges(k2, world)[rank]
    sk = SplitKGemm.on_gpu(gemm, world, rank, local_split_k=2)
    rows = sk(a2[:, ks:ke].cuda().contiguous(), b2[:, ks:ke].cuda().contiguous(), m2, n2)
    torch.cuda.synchronize()
    r0, r1 = row_range(m2, world, rank)
    res2 = gemm_ref.check(rows.cpu(), a2[r0:r1], b2)
    ok &= res2["ok"]
    # The same with the exchange cut into 3 column chunks (reduce-scatter of chunk c overlaps
    # the GEMM of chunk c + 1 on a second stream), each chunk choosing its own in-GPU split.
    skc = SplitKGemm.on_gpu(gemm, world, rank, local_split_k=0, chunks=3)
    rows_c = skc(a2[:, ks:ke].cuda().contiguous(), b2[:, ks:ke].cuda().contiguous(), m2, n2)
    torch.cuda.synchronize()
    res3 = gemm_ref.check(rows_c.cpu(), a2[r0:r1], b2)
    ok &= res3["ok"]
    # Split-K with the reduce-scatter done by the GEMM epilogue over peer memory: three calls
    # (alternating buffers, running arrival count), then a ragged M with bias under the dynamic
    # schedule and an automatic in-GPU split.
    from cutedsl_pingpong_gemm_b200.sharding import PeerSplitK
    pk = PeerSplitK(gemm, world, rank, local_split_k=2)
    res4 = None
    for it in range(3):
        rows_p = pk(a2[:, ks:ke].cuda().contiguous(), b2[:, ks:ke].cuda().contiguous(), m2, n2)
        torch.cuda.synchronize()
        res4 = gemm_ref.check(rows_p.cpu(), a2[r0:r1], b2)
        ok &= res4["ok"] and rows_p.shape == (r1 - r0, n2)
        if not res4["ok"]:
            print(f"RANK {rank} peer call {it} failed: {res4}", flush=True)
    pk.check_status()
    m3, n3, k3 = 128 * (2 * world + 1) - 40, 1000, 6144
    a3, b3, bias3 = gemm_ref.make_inputs(m3, n3, k3, seed=7, b_scale=k3 ** -0.5, with_bias=True)
    ks3, ke3 = k_ranges(k3, world)[rank]
    gemm_dyn = GemmSM90((128, 256), (128, 32), (2, 1, 1), (1, 1), ab_stage=6, reuse_ab=False,
                        is_persistent=True, dynamic_scheduler=True)
    pk3 = PeerSplitK(gemm_dyn, world, rank, bias=bias3.cuda(), local_split_k=0)
    for it in range(2):
        rows3 = pk3(a3[:, ks3:ke3].cuda().contiguous(), b3[:, ks3:ke3].cuda().contiguous(), m3, n3)
        torch.cuda.synchronize()
        q0, q1 = row_range(m3, world, rank)
        res5 = gemm_ref.check(rows3.cpu(), a3[q0:q1], b3, bias=bias3)
        ok &= res5["ok"] and rows3.shape == (q1 - q0, n3)
        if not res5["ok"]:
            print(f"RANK {rank} peer dynamic call {it} failed: {res5}", flush=True)
    pk3.check_status()
    pk.close()
    pk3.close()
    # One 128-row tile on single-CTA clusters (no pair tile past M, whose arrivals would count
    # for the last rank): rank 0 owns every row and the other ranks none, so their finishes wait
    # only for the per-call arrivals.  Rank 0 lags (a spin kernel before each call) while the
    # others issue calls back to back; a rank running ahead into a buffer rank 0 has not read yet
    # would add its partial sums twice.  Every call's rows are checked at the end.
    gemm1 = GemmSM90((128, 256), (128, 32), (1, 1, 1), (1, 1), ab_stage=3, reuse_ab=False,
                     is_persistent=True)
    m4, n4, k4 = 128, 512, 1024 * world
    a4, b4, _ = gemm_ref.make_inputs(m4, n4, k4, seed=9, b_scale=k4 ** -0.5)
    ks4, ke4 = k_ranges(k4, world)[rank]
    a4k, b4k = a4[:, ks4:ke4].cuda().contiguous(), b4[:, ks4:ke4].cuda().contiguous()
    pk4 = PeerSplitK(gemm1, world, rank, local_split_k=1)
    outs4 = []
    for it in range(6):
        if rank == 0:
            torch.cuda._sleep(2_000_000)
        outs4.append(pk4(a4k, b4k, m4, n4))
    torch.cuda.synchronize()
    res6 = {"ok": True}
    if rank == 0:
        for it, o in enumerate(outs4):
            r6 = gemm_ref.check(o.cpu(), a4, b4)
            if not r6["ok"]:
                res6 = r6
                print(f"RANK 0 rows owned alone, call {it} failed: {r6}", flush=True)
    ok &= res6["ok"]
    pk4.check_status()
    pk4.close()
    checks = {"mshard": res["ok"], "splitk_nccl": res2["ok"], "splitk_chunked": res3["ok"],
              "peer": res4["ok"], "peer_dynamic_bias": res5["ok"], "peer_rowless": res6["ok"]}
    print(f"RANK {rank} rows {r0}:{r1} ok={ok} {checks}", flush=True)
    flag = torch.tensor([1 if ok else 0], device="cuda")
    dist.all_reduce(flag, op=dist.ReduceOp.MIN)
    if rank == 0:
        print("RESULT", int(flag.item()), res, res2, res3, res4, res5, res6, flush=True)
    dist.destroy_process_group()
    sys.exit(0 if ok else 1)
''')


def _free_port():
    with socket.socket() as s:
        s.bind(("127.0.0.1", 0))
        return s.getsockname()[1]


def test_multi_gpu_mshard_and_splitk(tmp_path):
    ngpu = torch.cuda.device_count()
    if ngpu < 2:
        pytest.skip("needs at least two GPUs")
    world = min(ngpu, 8)
    script = tmp_path / "worker.py"
    script.write_text(WORKER)
    port = _free_port()
    procs = []
    for r in range(world):
        env = dict(os.environ, RANK=str(r), WORLD_SIZE=str(world), LOCAL_RANK=str(r),
                   MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port), NCCL_NVLS_ENABLE="0")
        procs.append(subprocess.Popen([sys.executable, str(script), ROOT], env=env,
                                      stdout=subprocess.PIPE, stderr=subprocess.STDOUT, text=True))
    outs = []
    for p in procs:
        try:
            out, _ = p.communicate(timeout=240)
        except subprocess.TimeoutExpired:
            p.kill()
            out, _ = p.communicate()
        outs.append((p.returncode, out))
    summary = [ln for _, out in outs for ln in out.splitlines() if ln.startswith("RANK")]
    assert all(rc == 0 for rc, _ in outs), ([rc for rc, _ in outs], summary, outs[0][1][-3000:])
    assert "RESULT 1" in outs[0][1], outs[0][1]


@pytest.mark.slow
@pytest.mark.parametrize("workload,exchange", [("tallk", "p2p"), ("tallk", "nccl"), ("llm", "p2p")])
def test_bench_full_size_parity_on_every_gpu(workload, exchange):
    """The benchmarked multi-GPU configurations at full size, through the bench itself under
    torchrun on every GPU of the box: tall K (2048 x 2048 x 131072 split over the ranks, partial
    sums exchanged by the GEMM epilogue over NVLink or by an NCCL reduce-scatter) and the LLM
    up-projection (16384 x 28672 x 8192 + bias, M split over the ranks).  Each rank checks the
    rows it owns after the timed steps (sampled rows element-wise and fp64 column / row sums,
    the contributions of every K range summed over the ranks for split-K) and the line reports
    the combined verdict."""
    import json
    ngpu = torch.cuda.device_count()
    if ngpu < 2:
        pytest.skip("needs at least two GPUs")
    world = min(ngpu, 8)
    cmd = ["timeout", "-k", "60", "600", sys.executable, "-m", "torch.distributed.run",
           "--nnodes=1", f"--nproc-per-node={world}", "--master-addr", "127.0.0.1",
           f"--master-port={_free_port()}", os.path.join(ROOT, "bench.py"), "--gpus", str(world),
           "--workload", workload, "--exchange", exchange, "--steps", "2", "--warmup", "1",
           "--no-e2e"]
    env = dict(os.environ, NCCL_NVLS_ENABLE="0")
    out = subprocess.run(cmd, cwd=ROOT, env=env, capture_output=True, text=True, timeout=700)
    assert out.returncode == 0, (out.stdout[-2000:], out.stderr[-3000:])
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout[-2000:]
    d = json.loads(lines[0])
    assert d["n_gpus"] == world and d["parity"]["ok"] and d["parity"]["ranks"] == world, d["parity"]
    assert len(d["per_rank"]) == world
