"""bench.py's reference arm runs on host cores alone, so its JSON line is checked here on CPU:
the keys the driver reads, a positive throughput and the e2e / cpu_baseline objects that the
reference arm must carry.  The bench's host-side helpers are checked as well."""
import json
import os
import subprocess
import sys

from conftest import ROOT


def test_reference_arm_prints_the_contract_line():
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload",
         "smallm", "--steps", "3", "--warmup", "3", "--cpu-seconds", "0.2"],
        cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    lines = [ln for ln in out.stdout.splitlines() if ln.startswith("{")]
    assert len(lines) == 1, out.stdout
    d = json.loads(lines[0])
    for key in ("metric", "value", "unit", "n_gpus", "steps", "warmup", "ms_per_step",
                "higher_is_better", "scaling", "vs_baseline", "dtype", "data", "config"):
        assert key in d, key
    assert d["impl"] == "reference" and d["n_gpus"] == 1
    assert d["steps"] == 3 and d["warmup"] == 3 and d["higher_is_better"] is True
    assert d["value"] > 0 and d["unit"] == "TFLOP/s"
    assert d["config"]["workload"] == "smallm"
    cb = d["cpu_baseline"]
    assert cb["value"] == d["value"] and cb["kind"] in ("port", "reference") and cb["cores"] >= 1
    e2e = d["e2e"]
    assert e2e["value"] == d["value"] and e2e["unit"] == d["unit"]
    assert e2e["h2d_bytes_per_step"] == 0 and e2e["d2h_bytes_per_step"] == 0


def test_bench_helpers():
    """The bench's data plumbing: recorded ncu traffic per workload and schedule, metric names,
    and the seeded MoE group sizes."""
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    with open(os.path.join(ROOT, "profiles", "traffic.json")) as f:
        recorded = json.load(f)
    assert bench.load_traffic("bf16_8192", "dynamic") == recorded["bf16_8192"]["dram_bytes_per_launch"]
    assert bench.load_traffic("bf16_8192", "static") == \
        recorded["bf16_8192:static"]["dram_bytes_per_launch"]
    assert bench.load_traffic("moe", "static") is None
    # Both arms print the same metric name; an --m override of the small-M workload names its M.
    for w in bench.WORKLOADS:
        assert bench.metric_name(w) == bench.metric_name(w, 0)
    assert "M=16," in bench.metric_name("smallm", 16)
    sizes = bench.group_sizes(16384, 8, seed=11)
    assert sum(sizes) == 16384 and len(sizes) == 8 and min(sizes) > 0
    assert sizes == bench.group_sizes(16384, 8, seed=11)


def _bench_module():
    import importlib.util
    spec = importlib.util.spec_from_file_location("bench", os.path.join(ROOT, "bench.py"))
    bench = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(bench)
    return bench


def test_both_arms_share_the_workload_config():
    """The reference arm and the GPU arm print the same ``config`` (both from workload_config),
    so the two lines describe the same workload key for key."""
    env = dict(os.environ, CUDA_VISIBLE_DEVICES="")
    out = subprocess.run(
        [sys.executable, os.path.join(ROOT, "bench.py"), "--impl", "reference", "--workload",
         "ref_harness", "--steps", "3", "--warmup", "3"],
        cwd=ROOT, env=env, capture_output=True, text=True, timeout=600)
    assert out.returncode == 0, out.stderr[-2000:]
    d = json.loads([ln for ln in out.stdout.splitlines() if ln.startswith("{")][0])
    bench = _bench_module()

    class Args:
        workload, m, exchange, chunks, activation = "ref_harness", 0, "p2p", 1, None

    assert d["config"] == bench.workload_config(Args, 1)
    assert d["config"]["m_per_gpu"] == 65536 and d["config"]["n"] == 4096
    for w in bench.WORKLOADS:
        Args.workload = w
        cfg = bench.workload_config(Args, 4)
        assert cfg["workload"] == w and cfg["k"] == bench.WORKLOADS[w]["k"]


def test_post_run_parity_check_accepts_the_product_and_rejects_planted_mistakes():
    """bench.py's post-run check on CPU tensors: a correctly rounded D passes, D with one wrong
    element, a missing bias, or a wrong activation fails; the split-K form at one rank too."""
    import torch
    bench = _bench_module()
    g = torch.Generator().manual_seed(3)
    m, n, k = 192, 160, 512
    a = torch.randn(m, k, generator=g).to(torch.bfloat16)
    b = (torch.randn(n, k, generator=g) * k ** -0.5).to(torch.bfloat16)
    bias = torch.randn(n, generator=g).to(torch.bfloat16)
    r = a.double() @ b.double().t() + bias.double()
    d = r.to(torch.bfloat16)
    assert bench.parity_dense(d, a, b, k, bias=bias)["ok"]
    bad = d.clone()
    bad[7, 11] += 0.5
    res = bench.parity_dense(bad, a, b, k, bias=bias)
    assert not res["ok"] and res["max_ratio"] > 1  # caught by the checksums if not sampled
    assert not bench.parity_dense(d, a, b, k)["ok"]  # bias left out of the expectation
    act = bench._act64("silu", r).to(torch.bfloat16)
    assert bench.parity_dense(act, a, b, k, bias=bias, act="silu")["ok"]
    assert not bench.parity_dense(act, a, b, k, bias=bias, act="gelu")["ok"]
    # gated: B = [W_gate; W_up]
    bg = torch.cat([b, b.flip(0)])
    pre = a.double() @ bg.double().t()
    dg = (bench._act64("silu", pre[:, :n]) * pre[:, n:]).to(torch.bfloat16)
    assert bench.parity_dense(dg, a, bg, k, act="silu", gated=True)["ok"]
    assert not bench.parity_dense(dg * 1.05, a, bg, k, act="silu", gated=True)["ok"]
    # split-K at one rank: the rank's rows are all of D
    d0 = (a.double() @ b.double().t()).to(torch.bfloat16)
    assert bench.parity_splitk(d0, a, b, m, n, k, 1, 0)["ok"]
    d1 = d0.clone()
    d1[100] = 0
    assert not bench.parity_splitk(d1, a, b, m, n, k, 1, 0)["ok"]
    # FP8 operands are checked through their dequantised values
    q = torch.randn(256, 300, generator=g).to(torch.float8_e4m3fn)
    s_rows = torch.rand(3, 256, generator=g) + 0.5
    deq = bench.dequantized(q, s_rows, "block", (1, 128))
    assert torch.equal(deq[:, 130], q[:, 130].float() * s_rows[1])
    s_blk = torch.rand(2, 3, generator=g) + 0.5
    deq = bench.dequantized(q, s_blk, "block", (128, 128))
    assert torch.equal(deq[200, 290], q[200, 290].float() * s_blk[1, 2])


def test_external_clock_sampler_reads_a_separate_process(tmp_path, monkeypatch):
    """Coupled multi-GPU runs take their clocks from a separate nvidia-smi process: started and
    producing samples before the timed region, summarised over the region (or the first sample
    after its start when the region is shorter than the polling period), and harmless when the
    tool is missing.  A stand-in nvidia-smi prints the same CSV columns every 10 ms."""
    import time
    sys.path.insert(0, ROOT)
    import bench
    fake = tmp_path / "nvidia-smi"
    fake.write_text("#!/bin/bash\n"
                    "while true; do\n"
                    "  echo \"$(date +'%Y/%m/%d %H:%M:%S.%3N'), 1875, 1965, 0x0000000000000004\"\n"
                    "  sleep 0.01\n"
                    "done\n")
    fake.chmod(0o755)
    monkeypatch.setenv("PATH", f"{tmp_path}:{os.environ.get('PATH', '')}")
    s = bench.ExternalClockSampler(0)
    s.start()
    time.sleep(0.2)
    s.stop()
    c = s.summary()
    assert c["samples"] >= 3 and c["sm_mhz"] == 1875 and c["sm_max_mhz"] == 1965
    assert c["reasons"] == ["sw_power_cap"]
    short = bench.ExternalClockSampler(0)
    short.start()
    short.stop()
    assert short.summary()["samples"] >= 1
    monkeypatch.setenv("PATH", str(tmp_path / "nothing_here"))
    none = bench.ExternalClockSampler(0)
    none.start()
    none.stop()
    assert none.summary() == {"sm_mhz": None, "sm_max_mhz": None, "reasons": [], "samples": 0}
