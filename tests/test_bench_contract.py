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
