#!/usr/bin/env python
"""GEMM benchmark for the sm_100a kernels (one JSON line on rank 0).

Workload (default ``bf16_8192``): the BF16 GEMM D = A . B^T with an 8192 x 8192 x 8192 shard per
GPU, A ~ N(0,1), B ~ N(0,1)/sqrt(K), fp32 accumulate, BF16 output.  With N GPUs
the M dimension is sharded: rank r owns rows [8192 r, 8192 (r+1)) of A and D, B is replicated,
and there is no collective on the data path ("scaling": "weak").  ``value`` is the whole-job
TFLOP/s = total flops / max over ranks of the device time of the timed steps.

Other workloads: ``llm`` (FFN up-projection 16384 x 28672 x 8192 with bias, M split over the N
GPUs: strong scaling of the BASELINE config 3), ``llm_swiglu`` (the same flops as a fused gated
FFN), ``fp8`` / ``fp8_block`` (E4M3 16384 x 8192 x 8192, per-tensor / 1x128 + 128x128 scales),
``smallm`` (M = 128, N = K = 8192: HBM bound), ``moe`` (grouped GEMM over 8 experts) and
``tallk`` (2048 x 2048 x 131072, K split over the GPUs; the partial sums are exchanged by the
GEMM epilogue over NVLink peer memory, or with ``--exchange nccl`` an NCCL reduce-scatter).

The tile schedule (``--scheduler auto``) is the dynamic one (cluster launch control) for the
dense workloads and the reference's static persistent schedule for the grouped MoE, block-scaled
FP8 and the reference harness's own constructor arguments, as measured fastest for each; small M
runs the small-M kernel (one cluster per 128 rows of B).  Under the dynamic schedule the
plan sizes the raster group so that a group's B panel stays within 32 MiB of L2 (``config``'s
``group_size``; the static schedule keeps the reference's 8).

Timing: W untimed warm-up steps, then exactly K steps between a barrier + synchronize on both
sides, timed with CUDA events on the launching stream, max over ranks.  Inputs are larger than
the 126 MB L2 (no flush between steps; stated in ``config.l2``).  SM clocks and throttle reasons
are sampled through NVML during the timed region.

``--impl reference`` times the CPU oracle of the same computation (fp32 matmul on the host
cores, the reference has no other runnable implementation: its kernel is sm_90a-only) on a
bounded sample of the workload; under torchrun only rank 0 runs it.
"""
import argparse
import json
import math
import os
import statistics
import sys
import threading
import time

HERE = os.path.dirname(os.path.abspath(__file__))
if HERE not in sys.path:
    sys.path.insert(0, HERE)

NOMINAL_DENSE_BF16_TFLOPS = 2250.0
FALLBACK_PEAKS = {"hbm_gbs": 6650.0, "bf16_tflops": 1590.0, "bf16_tflops_sustained": 1400.0}

NOMINAL_DENSE_FP8_TFLOPS = 4500.0

GRAPH_STEPS = 20  # calls per captured graph of the small-M workload

WORKLOADS = {
    # m is per GPU when m_is_per_gpu (weak scaling), else the total split over the GPUs.
    "bf16_8192": dict(m=8192, n=8192, k=8192, a_scale=1.0, b_scale=8192 ** -0.5, bias=False,
                      m_is_per_gpu=True, fp8=None),
    "llm": dict(m=16384, n=28672, k=8192, a_scale=1.0, b_scale=0.02, bias=True,
                m_is_per_gpu=False, fp8=None),
    # The same FFN up-projection as a fused SwiGLU: B = [W_gate; W_up] (2 x 14336 rows), D =
    # silu(A W_gate^T) * A W_up^T (14336 columns); the same flops as "llm".
    "llm_swiglu": dict(m=16384, n=14336, k=8192, a_scale=1.0, b_scale=0.02, bias=False,
                       m_is_per_gpu=False, fp8=None, gated=True, act="silu"),
    # Decode-like: HBM bound (B is 128 MiB, A 2 MiB); the small-M kernel (B rows on the MMA's
    # M side, K split over a cluster and reduced in shared memory) fills the SMs.
    "smallm": dict(m=128, n=8192, k=8192, a_scale=1.0, b_scale=8192 ** -0.5, bias=False,
                   m_is_per_gpu=True, fp8=None, small_m=True),
    # FP8 E4M3, A and B ~ N(0,1) quantised on the GPU (s = amax / 448) before timing.
    "fp8": dict(m=16384, n=8192, k=8192, a_scale=1.0, b_scale=1.0, bias=False,
                m_is_per_gpu=True, fp8="tensor"),
    "fp8_block": dict(m=16384, n=8192, k=8192, a_scale=1.0, b_scale=1.0, bias=False,
                      m_is_per_gpu=True, fp8="block"),
    # MoE expert FFN up-projection as one grouped GEMM: 8 experts of [W_gate; W_up]
    # (2 x 14336 rows, K = 4096), 16384 routed token rows per GPU spread unevenly over the
    # experts (seeded), fused SwiGLU; experts replicated, tokens per GPU (weak scaling).
    "moe": dict(m=16384, n=14336, k=4096, a_scale=1.0, b_scale=0.02, bias=False,
                m_is_per_gpu=True, fp8=None, gated=True, act="silu", groups=8),
    # Tall K: M = N = 2048, K = 131072 split over the GPUs (and inside each GPU); fp32 partials
    # reduced with one NCCL reduce-scatter, then cast to BF16 (strong scaling).
    "tallk": dict(m=2048, n=2048, k=131072, a_scale=1.0, b_scale=131072 ** -0.5, bias=False,
                  m_is_per_gpu=False, fp8=None, split="k"),
    # The reference's own benchmark (gemm_base.py:578-609): 65536 x 4096 x 8192 BF16, A and B
    # ~ N(0,1), with its constructor arguments: tile (128, 256), epi (128, 32), cluster (2, 1, 1),
    # atom (2, 1), ab_stage=3, reuse_ab=False, is_persistent=True (the static schedule).
    "ref_harness": dict(m=65536, n=4096, k=8192, a_scale=1.0, b_scale=1.0, bias=False,
                        m_is_per_gpu=True, fp8=None, ref_ctor=True),
}


def parse_args():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["cpg", "reference"], default="cpg")
    ap.add_argument("--workload", choices=sorted(WORKLOADS), default="bf16_8192")
    ap.add_argument("--tile-n", type=int, default=0, help="0 = 512 for BF16/FP8 (pairs), 256 for block FP8")
    ap.add_argument("--cluster-m", type=int, default=2)
    ap.add_argument("--stages", type=int, default=0, help="0 = deepest that fits")
    ap.add_argument("--epi-stages", type=int, default=0,
                    help="epilogue staging buffers per warp (0 = 2; block FP8 picks its own)")
    ap.add_argument("--split-k", type=int, default=0,
                    help="small-M only: 0 auto (the small-M kernel, -3), -1 Stream-K, S splits")
    ap.add_argument("--e2e-steps", type=int, default=10)
    ap.add_argument("--cpu-seconds", type=float, default=10.0)
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-e2e", action="store_true")
    ap.add_argument("--m", type=int, default=0,
                    help="override the workload's M (per GPU for weak scaling; for smaller "
                         "profiling cases)")
    ap.add_argument("--chunks", type=int, default=1,
                    help="tallk: column chunks whose reduce-scatter overlaps the next chunk's "
                         "GEMM (measured slower than 1 on two GPUs)")
    ap.add_argument("--graph", choices=["auto", "on", "off"], default="auto",
                    help="replay the timed steps from CUDA graphs of up to 20 consecutive calls "
                         "captured through the public API (auto: for the launch-bound small-M "
                         "workload)")
    ap.add_argument("--exchange", choices=["nccl", "p2p"], default="p2p",
                    help="tallk at N > 1: p2p: the GEMM epilogue adds the FP32 partials into the "
                         "owning rank's memory over NVLink (measured 6-8%% faster than NCCL on "
                         "four GPUs, equal on two), or an NCCL reduce-scatter of the partials")
    ap.add_argument("--scheduler", choices=["auto", "static", "dynamic"], default="auto",
                    help="tile schedule: the reference's static persistent schedule, or dynamic "
                         "(cluster launch control; not with Stream-K).  auto: "
                         "dynamic for the dense GEMM workloads (measured 3-10%% faster there "
                         "under the power cap), static for the small-M kernel, the grouped MoE "
                         "and block-scaled FP8 (measured equal or slower)")
    ap.add_argument("--activation", default=None,
                    choices=["relu", "silu", "gelu", "gelu_tanh"],
                    help="fused epilogue activation for the GEMM workloads")
    return ap.parse_args()


def load_peaks():
    path = os.path.join(HERE, "MEASURED_PEAKS.json")
    if os.path.exists(path):
        with open(path) as f:
            d = json.load(f)
        return d, "measured"
    return dict(FALLBACK_PEAKS), "fallback"


def load_traffic(workload, scheduler, m_override=0):
    """ncu DRAM bytes of one launch of the workload's kernel under this tile schedule (and, for
    an --m override, that M), or None when no capture of that combination is recorded."""
    path = os.path.join(HERE, "profiles", "traffic.json")
    if not os.path.exists(path):
        return None
    with open(path) as f:
        d = json.load(f)
    keys = [f"{workload}:{scheduler}", workload]
    if m_override and m_override != WORKLOADS[workload]["m"]:
        keys = [f"{workload}:m{m_override}"]
    for key in keys:
        e = d.get(key)
        if e is not None and e.get("scheduler", scheduler) == scheduler:
            return e.get("dram_bytes_per_launch")
    return None


# ------------------------------------------------------------------ clocks (NVML)
class ClockSampler:
    """Samples SM clock and clock-event reasons of one GPU on a background thread."""

    REASONS = [
        (0x4, "sw_power_cap"), (0x8, "hw_slowdown"), (0x20, "sw_thermal_slowdown"),
        (0x40, "hw_thermal_slowdown"), (0x80, "hw_power_brake_slowdown"),
        (0x2, "applications_clocks_setting"), (0x10, "sync_boost"),
    ]

    def __init__(self, cuda_index, period_s=0.002):
        self.samples = []
        self.reasons = 0
        self.period = period_s
        self.max_mhz = None
        self._stop = threading.Event()
        self._thread = None
        self.h = None
        try:
            import pynvml
            self.nv = pynvml
            pynvml.nvmlInit()
            self.h = self._handle(cuda_index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self.h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self.h = None

    def _handle(self, cuda_index):
        import torch
        nv = self.nv
        try:
            p = torch.cuda.get_device_properties(cuda_index)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
            return nv.nvmlDeviceGetHandleByPciBusId(bus.encode())
        except Exception:
            return nv.nvmlDeviceGetHandleByIndex(cuda_index)

    def _run(self):
        nv = self.nv
        while not self._stop.is_set():
            try:
                self.samples.append(nv.nvmlDeviceGetClockInfo(self.h, nv.NVML_CLOCK_SM))
                try:
                    r = nv.nvmlDeviceGetCurrentClocksEventReasons(self.h)
                except AttributeError:
                    r = nv.nvmlDeviceGetCurrentClocksThrottleReasons(self.h)
                self.reasons |= int(r)
            except Exception:
                pass
            time.sleep(self.period)

    def start(self):
        if self.h is not None:
            self._thread = threading.Thread(target=self._run, daemon=True)
            self._thread.start()

    def stop(self):
        if self._thread is not None:
            self._stop.set()
            self._thread.join()

    def summary(self):
        if self.h is None or not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        names = [n for bit, n in self.REASONS if self.reasons & bit]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


class ExternalClockSampler:
    """The same summary as ClockSampler from a separate ``nvidia-smi`` process polling every
    10 ms (started before the barrier, its output in a temporary file), for steps coupled across
    ranks: there an in-process polling thread stalled a rank's launches and with them every other
    rank (tall K on 8 GPUs: 268-270 us per step against 216-218 us without the thread).  The
    constructor waits (at most 10 s) for the first sample, so the sampler is running before the
    timed region; when no sample falls inside a short timed region, the first one after its start
    is taken."""

    def __init__(self, cuda_index, period_ms=10):
        import subprocess
        import tempfile
        import torch
        self.samples, self.reasons, self.max_mhz = [], 0, None
        self.window = (None, None)
        self.proc = None
        self.out = tempfile.NamedTemporaryFile(mode="w+", prefix="clocks_", suffix=".csv")
        try:
            p = torch.cuda.get_device_properties(cuda_index)
            bus = f"{p.pci_domain_id:08x}:{p.pci_bus_id:02x}:{p.pci_device_id:02x}.0"
        except Exception:
            bus = str(cuda_index)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", bus, "--query-gpu=timestamp,clocks.sm,clocks.max.sm,"
                 "clocks_event_reasons.active", "--format=csv,noheader,nounits",
                 f"--loop-ms={period_ms}"], stdout=self.out, stderr=subprocess.DEVNULL, text=True)
        except OSError:
            self.proc = None
            return
        deadline = time.time() + 10.0
        while time.time() < deadline and self.proc.poll() is None:
            if os.path.getsize(self.out.name) > 0:
                break
            time.sleep(0.01)

    def start(self):
        self.window = (time.time(), None)

    def _parse(self):
        import datetime as _dt
        rows = []
        with open(self.out.name) as f:
            for line in f:
                parts = [x.strip() for x in line.split(",")]
                if len(parts) != 4:
                    continue
                try:
                    ts = _dt.datetime.strptime(parts[0], "%Y/%m/%d %H:%M:%S.%f").timestamp()
                    rows.append((ts, int(parts[1]), int(parts[2]), int(parts[3], 16)))
                except ValueError:
                    continue
        return rows

    def stop(self):
        self.window = (self.window[0], time.time() + 0.02)
        if self.proc is None:
            return
        time.sleep(0.03)  # at least one sample after the timed region
        self.proc.terminate()
        try:
            self.proc.wait(timeout=10)
        except Exception:
            self.proc.kill()
            self.proc.wait()
        rows = self._parse()
        self.out.close()
        t0, t1 = self.window
        if t0 is None:
            return
        inside = [r for r in rows if t0 <= r[0] <= t1]
        if not inside:
            inside = [r for r in rows if r[0] >= t0][:1]
        for _, mhz, max_mhz, reasons in inside:
            self.samples.append(mhz)
            self.reasons |= reasons
            self.max_mhz = max_mhz
        if self.max_mhz is None and rows:
            self.max_mhz = rows[-1][2]

    def summary(self):
        if not self.samples:
            return {"sm_mhz": None, "sm_max_mhz": self.max_mhz, "reasons": [], "samples": 0}
        names = [n for bit, n in ClockSampler.REASONS if self.reasons & bit]
        return {"sm_mhz": statistics.median(self.samples), "sm_max_mhz": self.max_mhz,
                "reasons": names, "samples": len(self.samples)}


class NvlinkCounter:
    """NVLink data bytes this GPU sent and received (NVML throughput counters, summed over its
    links), read before and after the timed region; None where the driver does not expose them."""

    LINKS = 18

    def __init__(self, cuda_index):
        self.h = None
        try:
            import pynvml
            self.nv = pynvml
            pynvml.nvmlInit()
            self.h = ClockSampler._handle(self, cuda_index)
        except Exception:
            self.h = None
        self.start_tx = self.start_rx = None

    def read(self):
        if self.h is None:
            return None
        nv = self.nv
        fields = []
        for link in range(self.LINKS):
            fields.append((nv.NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_TX, link))
            fields.append((nv.NVML_FI_DEV_NVLINK_THROUGHPUT_DATA_RX, link))
        try:
            vals = nv.nvmlDeviceGetFieldValues(self.h, fields)
        except Exception:
            return None
        tx = rx = 0
        seen = False
        for i, v in enumerate(vals):
            if v.nvmlReturn != 0:
                continue
            seen = True
            kib = int(v.value.ullVal)
            if i % 2 == 0:
                tx += kib
            else:
                rx += kib
        return (tx * 1024, rx * 1024) if seen else None

    def start(self):
        r = self.read()
        self.start_tx, self.start_rx = r if r is not None else (None, None)

    def delta(self):
        r = self.read()
        if r is None or self.start_tx is None:
            return None
        return r[0] - self.start_tx, r[1] - self.start_rx


# ------------------------------------------------------------------ distributed plumbing
def dist_setup(ngpus):
    import torch
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    if world != ngpus:
        raise SystemExit(f"--gpus {ngpus} but WORLD_SIZE={world}")
    if world > 1:
        import datetime
        import torch.distributed as dist
        os.environ.setdefault("MASTER_ADDR", "127.0.0.1")
        torch.cuda.set_device(local)
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    else:
        torch.cuda.set_device(local)
    return world, rank, local


def barrier(world):
    if world > 1:
        import torch.distributed as dist
        dist.barrier()


def align_start(world, dev):
    """Start the ranks' timed steps together on the device: a one-element all-reduce on the
    current stream, after which every rank's next kernel starts at (nearly) the same time,
    however late each host left the barrier."""
    if world > 1:
        import torch
        import torch.distributed as dist
        dist.all_reduce(torch.ones(1, device=dev))


def reduce_max(x, world):
    if world == 1:
        return x
    import torch
    import torch.distributed as dist
    t = torch.tensor([x], dtype=torch.float64, device="cuda")
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    return float(t.item())


def gather_floats(values, world):
    """Every rank's list of floats (same length on every rank), in rank order."""
    if world == 1:
        return [list(values)]
    import torch
    import torch.distributed as dist
    t = torch.tensor([float("nan") if v is None else v for v in values], dtype=torch.float64,
                     device="cuda")
    out = [torch.empty_like(t) for _ in range(world)]
    dist.all_gather(out, t)
    return [[None if math.isnan(x) else x for x in o.tolist()] for o in out]


def per_rank_summary(ms_local, clocks, world):
    """Each rank's CUDA-event time per step and median SM clock, so that a multi-GPU line names
    the rank (and clock) that set its max-over-ranks time."""
    rows = gather_floats([ms_local, clocks.get("sm_mhz")], world)
    return [{"rank": r, "ms_per_step": v[0], "sm_mhz": v[1]} for r, v in enumerate(rows)]


# ------------------------------------------------------------------ post-run parity check
# After the timed region every rank checks the D its last timed step wrote, on its own GPU in
# fp64, against the product of the same device inputs: sampled rows element-wise and, for the
# linear epilogues, the column and row sums of the whole of D (O(MK + NK) work: (1^T A) B^T and
# A (B^T 1)).  Tolerance (the project spec, as in the tests): relative Frobenius <= 1e-2 (BF16) /
# 3e-2 (FP8) and element-wise |D - R| <= 2^-8 |R| + K 2^-23 (|A| |B|^T) (+ the activation terms).
# The reference harness checked its timed output the same way, right after the launch
# (gemm_base.py:609-619: allclose and a count of wrong elements).
BF16_REL = 2.0 ** -8
ACC_SLACK_PER_K = 2.0 ** -23
ACT_SLOPE = 1.13      # max |act'(y)| of relu, silu, gelu, gelu_tanh
ACT_REL = 2.0 ** -18  # the device's expf / erff / tanhf against fp64
PARITY_ROWS = 64


def _act64(name, y):
    import torch
    if name is None:
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


def expected_rows(pre, s, k, n, bias=None, act=None, gated=False):
    """Expected D rows and their element-wise tolerance from the fp64 products of those rows,
    ``pre`` = A_rows B^T and ``s`` = |A_rows| |B|^T (gated: B = [W_gate; W_up], 2n columns)."""
    slack = k * ACC_SLACK_PER_K
    if gated:
        g, u = pre[:, :n], pre[:, n:]
        tg, tu = slack * s[:, :n], slack * s[:, n:]
        ag = _act64(act, g)
        r = ag * u
        tol = (BF16_REL * r.abs() + ACT_SLOPE * tg * (u.abs() + tu) + ag.abs() * tu
               + ACT_REL * (g.abs() * u.abs() + r.abs()) + 1e-6)
        return r, tol
    tol_pre = slack * s
    if bias is not None:
        pre = pre + bias.double()
        tol_pre = tol_pre + 2.0 ** -24 * bias.double().abs()
    if act is None:
        return pre, BF16_REL * pre.abs() + tol_pre
    r = _act64(act, pre)
    return r, BF16_REL * r.abs() + ACT_SLOPE * tol_pre + ACT_REL * pre.abs() + 1e-6


def rows_verdict(d_rows, r, tol):
    """(worst |D - R| / tol, relative Frobenius error) of sampled rows."""
    import torch
    diff = d_rows.double() - r
    ratio = float((diff.abs() / tol.clamp_min(1e-300)).max()) if diff.numel() else 0.0
    den = float(torch.linalg.vector_norm(r))
    frob = float(torch.linalg.vector_norm(diff)) / den if den > 0 else 0.0
    return ratio, frob


def checksum_ratio(d, a, b64, k, bias=None):
    """Worst |sum - expected| / bound over the column sums and row sums of the whole of D."""
    import torch
    f64 = torch.float64
    m, n = d.shape
    ref_col = torch.mv(b64, a.sum(0, dtype=f64))
    abs_col = torch.mv(b64.abs(), a.abs().sum(0, dtype=f64))
    ref_row = torch.mv(a.double(), b64.sum(0))
    abs_row = torch.mv(a.double().abs(), b64.abs().sum(0))
    if bias is not None:
        ref_col = ref_col + m * bias.double()
        ref_row = ref_row + bias.double().sum()
    da = d.abs()
    bound_col = BF16_REL * da.sum(0, dtype=f64) + k * ACC_SLACK_PER_K * abs_col + 1e-6 * m
    bound_row = BF16_REL * da.sum(1, dtype=f64) + k * ACC_SLACK_PER_K * abs_row + 1e-6 * n
    r_col = float(((d.sum(0, dtype=f64) - ref_col).abs() / bound_col).max())
    r_row = float(((d.sum(1, dtype=f64) - ref_row).abs() / bound_row).max())
    return max(r_col, r_row)


def parity_dense(d, a, b, k, bias=None, act=None, gated=False, frob_tol=1e-2, seed=0):
    """Post-run check of one rank's whole D = epilogue(A B^T) (A, B: the kernel's operands, or
    their dequantised values for FP8).  Returns the rank's verdict dict."""
    import torch
    m = d.shape[0]
    n = d.shape[1]
    g = torch.Generator().manual_seed(seed)
    rows = torch.randperm(m, generator=g)[:PARITY_ROWS].sort().values.to(d.device)
    b64 = b.double()
    a_s = a[rows].double()
    pre = a_s @ b64.t()
    s = a_s.abs() @ b64.abs().t()
    r, tol = expected_rows(pre, s, k, n, bias, act, gated)
    ratio, frob = rows_verdict(d[rows], r, tol)
    checks = f"{rows.numel()} sampled rows element-wise"
    if act is None and not gated:
        ratio = max(ratio, checksum_ratio(d, a, b64, k, bias))
        checks += " + fp64 column and row sums of all of D"
    nan = bool(torch.isnan(d).any())
    return {"ok": ratio <= 1.0 and frob <= frob_tol and not nan, "max_ratio": ratio,
            "frob_sampled": frob, "frob_tol": frob_tol, "checks": checks}


def parity_reduce(res, world):
    """Combine the ranks' verdicts (collective: every rank calls it once)."""
    if world == 1:
        return dict(res, ranks=1)
    vals = gather_floats([1.0 if res["ok"] else 0.0, res["max_ratio"], res["frob_sampled"]],
                         world)
    return dict(res, ok=all(v[0] == 1.0 for v in vals), max_ratio=max(v[1] for v in vals),
                frob_sampled=max(v[2] for v in vals), ranks=world)


def dequantized(q, scales, mode, block=None):
    """FP32 values of E4M3 operands on the device: q * s per tensor or per block."""
    qf = q.float()
    if mode == "tensor":
        return qf * scales
    rows, cols = qf.shape
    if block == (1, 128):  # scales [ceil(K/128), rows]
        return qf * scales.t().repeat_interleave(128, dim=1)[:, :cols]
    return qf * scales.repeat_interleave(128, dim=0).repeat_interleave(128, dim=1)[:rows, :cols]


# ------------------------------------------------------------------ CPU baseline (oracle)
def cpu_matmul_rate(rows, n, k, seconds, max_reps=50, seed=0):
    """fp32 CPU matmul of a rows x k slab against B^T (the oracle's computation)."""
    import torch
    from oracle import gemm_ref
    cores = gemm_ref.set_threads()
    g = torch.Generator().manual_seed(seed)
    a = torch.randn(rows, k, generator=g).to(torch.bfloat16).float()
    b = (torch.randn(n, k, generator=g) * k ** -0.5).to(torch.bfloat16).float()
    torch.matmul(a[: min(rows, 64)], b.t())  # warm the thread pool
    reps, t0 = 0, time.perf_counter()
    while True:
        torch.matmul(a, b.t())
        reps += 1
        el = time.perf_counter() - t0
        if el >= seconds or reps >= max_reps:
            break
    return 2.0 * rows * n * k * reps / el / 1e12, cores, reps, el


def workload_config(args, world):
    """The workload's ``config``: the same dict in both arms (the kernel's own choices go to the
    GPU arm's ``kernel_config``)."""
    w = WORKLOADS[args.workload]
    n, k = w["n"], w["k"]
    m_w = args.m or w["m"]
    if w.get("split") == "k":
        peer = args.exchange == "p2p" and world > 1
        if world == 1:
            par = "1 GPU, K split inside the GPU"
        elif peer:
            par = (f"split-K x{world} (GEMM epilogue adds partials into the owners' memory over "
                   f"NVLink), K split again inside each GPU")
        else:
            par = f"split-K x{world} (NCCL reduce-scatter), K split again inside each GPU"
        return {"workload": args.workload, "m": m_w, "n": n, "k": k, "parallelism": par,
                "rs_chunks": max(1, args.chunks) if not peer else 1,
                "l2": "A and B 512 MiB per GPU at 1 GPU; no flush"}
    if w.get("groups"):
        return {"workload": args.workload, "rows_per_gpu": m_w, "n": n, "k": k,
                "groups": w["groups"], "gated": bool(w.get("gated")), "activation": w.get("act"),
                "parallelism": f"tokens per GPU x{world}, experts replicated",
                "l2": "B is 1.9 GB; no flush"}
    m = m_w if w["m_is_per_gpu"] else m_w // world
    return {"workload": args.workload, "m_per_gpu": m, "n": n, "k": k, "m_total": m * world,
            "parallelism": f"m-shard x{world}, B replicated", "bias": bool(w["bias"]),
            "activation": w.get("act") or args.activation, "gated": bool(w.get("gated")),
            "fp8_scales": w["fp8"],
            "l2": ("inputs larger than L2 (B 128 MiB, A 2 MiB, read once per step); no flush"
                   if w.get("small_m") else "inputs larger than L2 (126 MB); no flush")}


def run_reference(args, world, rank):
    """--impl reference: the CPU oracle on the host cores, rank 0 only."""
    import torch
    from oracle import gemm_ref
    if rank != 0:
        return
    w = WORKLOADS[args.workload]
    n, k = w["n"], w["k"]
    cores = gemm_ref.set_threads()
    g = torch.Generator().manual_seed(0)
    gated = bool(w.get("gated"))
    b_rows = 2 * n if gated else n
    b = (torch.randn(b_rows, k, generator=g) * w["b_scale"]).to(torch.bfloat16).float()

    def cpu_step(a):
        r = torch.matmul(a, b.t())
        if gated:  # the fused epilogue of the gated form, on the host
            r = gemm_ref.activation(w.get("act"), r[:, :n]) * r[:, n:]
        return r

    # Calibrate the per-step sample so the whole run stays within about a minute.
    probe_rows = 64
    a = torch.randn(probe_rows, k, generator=g).to(torch.bfloat16).float()
    cpu_step(a)
    t0 = time.perf_counter()
    cpu_step(a)
    t_probe = max(time.perf_counter() - t0, 1e-4)
    per_step_budget = 60.0 / max(1, args.steps + args.warmup)
    rows = int(max(8, min(args.m or w["m"], probe_rows * per_step_budget / t_probe)))
    rows = max(8, rows // 8 * 8)
    a = torch.randn(rows, k, generator=g).to(torch.bfloat16).float()
    for _ in range(args.warmup):
        cpu_step(a)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        cpu_step(a)
    el = time.perf_counter() - t0
    flops = 2.0 * rows * b_rows * k * args.steps
    value = flops / el / 1e12
    sample = (f"{rows}x{n}x{k} fp32 row slab of the {args.workload} GEMM per step "
              f"(torch.matmul on {cores} host threads)")
    line = {
        "impl": "reference", "metric": metric_name(args.workload, args.m), "value": value,
        "unit": "TFLOP/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": el / args.steps * 1e3, "higher_is_better": True,
        "scaling": "weak" if w["m_is_per_gpu"] else "strong", "vs_baseline": None,
        "dtype": "f32", "data": "synthetic",
        "config": workload_config(args, world),
        "cpu_baseline": {"value": value, "unit": "TFLOP/s", "cores": cores, "kind": "port",
                         "sample": sample, "rows_per_step": rows},
        "e2e": {"value": value, "unit": "TFLOP/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
        "note": "reference kernel is sm_90a CuTe-DSL (wgmma) and cannot run on sm_100; the "
                "reference arm is the fp32 CPU oracle of D = A @ B.T",
    }
    print(json.dumps(line), flush=True)


def metric_name(workload, m_override=0):
    """The metric string of a workload (both arms print the same one); an --m override of the
    small-M workload names its M."""
    if workload == "smallm" and m_override:
        return f"GEMM TFLOPS (BF16 M={m_override}, N=K=8192, HBM-bound)"
    return {"bf16_8192": "GEMM TFLOPS (BF16 8192^3 per GPU, M-sharded, B replicated)",
            "llm": "GEMM TFLOPS (BF16 LLM FFN up 16384x28672x8192 + bias, M-sharded)",
            "llm_swiglu": "GEMM TFLOPS (BF16 LLM FFN up 16384x28672x8192 as fused SwiGLU, "
                          "D 16384x14336, M-sharded)",
            "smallm": "GEMM TFLOPS (BF16 M=128, N=K=8192, HBM-bound)",
            "fp8": "GEMM TFLOPS (FP8 E4M3 16384x8192x8192 per GPU, per-tensor scales)",
            "fp8_block": "GEMM TFLOPS (FP8 E4M3 16384x8192x8192 per GPU, 1x128 / 128x128 block scales)",
            "tallk": "GEMM TFLOPS (BF16 2048x2048x131072 split-K over GPUs)",
            "moe": "GEMM TFLOPS (BF16 grouped MoE up-projection, 8 experts x [2x14336, 4096], "
                   "16384 token rows per GPU, fused SwiGLU)",
            "ref_harness": "GEMM TFLOPS (BF16 65536x4096x8192 per GPU, the reference harness "
                           "shape and constructor arguments)",
            }[workload]


def parity_splitk(out, a_k, b_k, m, n, k, world, rank):
    """Post-run check of this rank's rows of a split-K D = sum_q A_q B_q^T, where rank q holds
    the K range q of A and B.  Every rank computes its fp64 contributions to the sampled rows
    (PARITY_ROWS // world rows of every rank's range) and to every rank's column and row sums;
    summed over the ranks (all-reduce, the same collectives on every rank) they give the
    expected values of this rank's rows."""
    import torch
    import torch.distributed as dist
    from cutedsl_pingpong_gemm_b200.sharding import row_range
    f64 = torch.float64
    dev = a_k.device
    a64, b64 = a_k.double(), b_k.double()
    per = max(1, PARITY_ROWS // world)
    g = torch.Generator().manual_seed(5)
    samples, ranges = [], []
    for q in range(world):
        s0, s1 = row_range(m, world, q)
        ranges.append((s0, s1))
        samples.append((torch.randperm(s1 - s0, generator=g)[:per] + s0).sort().values)
    rows = torch.cat(samples).to(dev)
    pre = a64[rows] @ b64.t()
    sab = a64[rows].abs() @ b64.abs().t()
    col = torch.stack([torch.mv(b64, a64[s0:s1].sum(0)) for s0, s1 in ranges])
    col_abs = torch.stack([torch.mv(b64.abs(), a64[s0:s1].abs().sum(0)) for s0, s1 in ranges])
    row = torch.mv(a64, b64.sum(0))
    row_abs = torch.mv(a64.abs(), b64.abs().sum(0))
    if world > 1:
        for t in (pre, sab, col, col_abs, row, row_abs):
            dist.all_reduce(t)
    s0, s1 = ranges[rank]
    mine = slice(rank * per, rank * per + samples[rank].numel())
    r, tol = expected_rows(pre[mine], sab[mine], k, n)
    ratio, frob = rows_verdict(out[(samples[rank] - s0).to(dev)], r, tol)
    da = out.abs()
    bound_col = BF16_REL * da.sum(0, dtype=f64) + k * ACC_SLACK_PER_K * col_abs[rank] + 1e-6 * (s1 - s0)
    bound_row = BF16_REL * da.sum(1, dtype=f64) + k * ACC_SLACK_PER_K * row_abs[s0:s1] + 1e-6 * n
    ratio = max(ratio, float(((out.sum(0, dtype=f64) - col[rank]).abs() / bound_col).max()),
                float(((out.sum(1, dtype=f64) - row[s0:s1]).abs() / bound_row).max()))
    nan = bool(torch.isnan(out).any())
    return {"ok": ratio <= 1.0 and frob <= 1e-2 and not nan, "max_ratio": ratio,
            "frob_sampled": frob, "frob_tol": 1e-2,
            "checks": (f"{per} sampled rows per rank element-wise + fp64 column and row sums of "
                       f"each rank's rows (contributions of every K range summed over ranks)")}


# ------------------------------------------------------------------ GPU arm: tall-K split-K
def run_tallk(args, world, rank, local):
    """Split-K over GPUs: rank r multiplies its K range (and splits it again inside the GPU)
    into fp32 partials, one NCCL reduce-scatter sums them, the cast kernel writes BF16 rows."""
    import torch
    from cutedsl_pingpong_gemm_b200 import GemmSM90, RasterOrder
    from cutedsl_pingpong_gemm_b200.sharding import PeerSplitK, SplitKGemm, k_ranges, row_range

    w = WORKLOADS[args.workload]
    m, n, k = w["m"], w["n"], w["k"]
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    ks, ke = k_ranges(k, world)[rank]
    gen = torch.Generator(device=dev).manual_seed(2000 + rank)
    a_k = (torch.randn(m, ke - ks, generator=gen, device=dev) * w["a_scale"]).to(torch.bfloat16)
    b_k = (torch.randn(n, ke - ks, generator=gen, device=dev) * w["b_scale"]).to(torch.bfloat16)
    tile_n = args.tile_n or 256
    cm = args.cluster_m
    stages = args.stages or (6 if cm == 2 else 4)
    gemm = GemmSM90(tile_shape_mn=(128, tile_n), epi_tile_mn=(128, 32),
                    cluster_shape_mnk=(cm, 1, 1), atom_layout_mn=(1, 1), ab_stage=stages,
                    epi_stage=2, raster_order=RasterOrder.AlongN, reuse_ab=False, is_persistent=True,
                    dynamic_scheduler=args.scheduler == "dynamic")
    chunks = max(1, args.chunks)
    peer = args.exchange == "p2p" and world > 1
    if peer:
        # The GEMM epilogue adds the partials into the owners' memory; one finish kernel each.
        sk = PeerSplitK(gemm, world, rank, local_split_k=0)
        chunks = 1
    else:
        # The in-GPU split of each (chunk's) GEMM is picked from its tile count (auto_split_k).
        sk = SplitKGemm.on_gpu(gemm, world, rank, local_split_k=0, chunks=chunks)

    launches = [0]

    def step():
        out = sk(a_k, b_k, m, n)
        if peer:
            launches[0] += 3  # GEMM (exchange in its epilogue), per-call arrival, finish
        else:
            launches[0] += 2 * len(sk.column_chunks(n)) if chunks > 1 else 2  # GEMM + cast each
        return out

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    # Host-side set-up (NVML handles and counter reads take milliseconds) before the barrier:
    # the ranks exchange partial sums every step, so a rank that starts late makes the others
    # wait inside their timed region.
    # The ranks exchange partial sums every step, so their steps are coupled: anything that
    # stalls one rank's host stalls every rank.  Clocks then come from a separate process, and
    # the ranks start together on the device, however late each host leaves the barrier.
    sampler = ExternalClockSampler(local) if world > 1 else ClockSampler(local)
    nvl = NvlinkCounter(local)
    nvl.start()
    launches[0] = 0
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    barrier(world)
    torch.cuda.synchronize()
    align_start(world, dev)
    e0.record(stream)
    for i in range(args.steps):
        out = step()
        if i == 0:
            sampler.start()  # the GPU is busy from here on: no idle-clock samples
    e1.record(stream)
    torch.cuda.synchronize()
    sampler.stop()
    nv_delta = nvl.delta()
    barrier(world)
    ms_local = e0.elapsed_time(e1) / args.steps
    ms = reduce_max(ms_local, world)
    clocks = sampler.summary()
    per_rank = per_rank_summary(ms_local, clocks, world)
    nv_rows = gather_floats([None if nv_delta is None else nv_delta[0] / args.steps,
                             None if nv_delta is None else nv_delta[1] / args.steps], world)
    for r, v in enumerate(nv_rows):
        per_rank[r]["nvlink_tx_bytes_per_step"] = v[0]
        per_rank[r]["nvlink_rx_bytes_per_step"] = v[1]
    if peer:
        sk.check_status()
    parity = parity_reduce(parity_splitk(out, a_k, b_k, m, n, k, world, rank), world)
    total_flops = 2.0 * m * n * k
    value = total_flops / (ms * 1e-3) / 1e12
    peaks, peak_src = load_peaks()
    if rank == 0:
        s0, s1 = row_range(m, world, rank)
        line = {
            "metric": metric_name(args.workload, args.m), "value": value, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": workload_config(args, world),
            "kernel_config": {"scheduler": args.scheduler, "tile": [128, tile_n],
                              "cluster": [cm, 1, 1], "ab_stage": stages,
                              "exchange": "p2p" if peer else ("nccl" if world > 1 else None),
                              "rows_per_rank": s1 - s0},
            "roofline": {"bound": "tensor", "achieved": total_flops / world / (ms_local * 1e-3) / 1e12,
                         "peak": peaks["bf16_tflops"], "unit": "TFLOP/s",
                         "frac": total_flops / world / (ms_local * 1e-3) / 1e12 / peaks["bf16_tflops"],
                         "peak_source": f"{peak_src} bf16_tflops", "traffic": None,
                         "note": "achieved covers GEMM + reduce-scatter + cast per step"},
            # What must cross NVLink per rank and step: the FP32 partial sums of the rows other
            # ranks own, (world - 1) / world of the M x N partial.
            "nvlink_min_bytes_per_rank": int(4 * m * n * (world - 1) / world),
            "clocks": clocks, "per_rank": per_rank, "parity": parity,
            "gpu_launches": launches[0] * world, "e2e": None, "cpu_baseline": None,
        }
        print(json.dumps(line), flush=True)
    del out
    if peer:
        sk.close()
    if not parity["ok"]:
        raise SystemExit(f"parity check failed: {parity}")


# ------------------------------------------------------------------ GPU arm: grouped (MoE)
def group_sizes(rows, groups, seed=0):
    """Seeded uneven split of ``rows`` token rows over ``groups`` experts (router-like skew)."""
    import torch
    g = torch.Generator().manual_seed(seed)
    p = torch.softmax(torch.randn(groups, generator=g) * 0.5, 0)
    sizes = torch.floor(p * rows).long()
    sizes[0] += rows - int(sizes.sum())
    return [int(x) for x in sizes]


def run_grouped(args, world, rank, local):
    import torch
    from cutedsl_pingpong_gemm_b200 import GemmSM90, RasterOrder

    w = WORKLOADS[args.workload]
    n, k, groups = w["n"], w["k"], w["groups"]
    t = args.m or w["m"]
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)
    gated, act = bool(w.get("gated")), w.get("act")
    b_rows = 2 * n if gated else n
    gen_a = torch.Generator(device=dev).manual_seed(1000 + rank)
    gen_b = torch.Generator(device=dev).manual_seed(7)
    a = (torch.randn(t, k, generator=gen_a, device=dev) * w["a_scale"]).to(torch.bfloat16)
    b = (torch.randn(groups, b_rows, k, generator=gen_b, device=dev) * w["b_scale"]).to(
        torch.bfloat16)
    d = torch.empty(t, n, dtype=torch.bfloat16, device=dev)
    sizes = group_sizes(t, groups, seed=11 + rank)
    off = [0]
    for sz in sizes:
        off.append(off[-1] + sz)
    offs = torch.tensor(off, dtype=torch.int32, device=dev)
    cm = args.cluster_m
    tile_n = 512 if gated else (args.tile_n or (512 if cm == 2 else 256))
    stages = args.stages or {(512, 2): 3, (512, 1): 2}.get((tile_n, cm), 6 if cm == 2 else 4)
    gemm = GemmSM90(tile_shape_mn=(128, tile_n), epi_tile_mn=(128, 32),
                    cluster_shape_mnk=(cm, 1, 1), atom_layout_mn=(1, 1), ab_stage=stages,
                    epi_stage=2, raster_order=RasterOrder.AlongN, reuse_ab=False,
                    is_persistent=True, dynamic_scheduler=args.scheduler == "dynamic")

    def step():
        gemm.grouped(a, b, d, offs, stream, activation=act, gated=gated)

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()
    sampler = ClockSampler(local)
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i in range(args.steps):
        step()
        if i == 0:
            sampler.start()
    e1.record(stream)
    torch.cuda.synchronize()
    sampler.stop()
    barrier(world)
    ms_local = e0.elapsed_time(e1) / args.steps
    ms = reduce_max(ms_local, world)
    clocks = sampler.summary()
    per_rank = per_rank_summary(ms_local, clocks, world)
    # Post-run check: sampled rows of every non-empty group against that group's weights.
    worst, frob, bad_nan = 0.0, 0.0, bool(torch.isnan(d).any())
    g = torch.Generator().manual_seed(9)
    for gi in range(groups):
        r0, r1 = off[gi], off[gi + 1]
        if r1 <= r0:
            continue
        rows = (torch.randperm(r1 - r0, generator=g)[:max(1, PARITY_ROWS // groups)] + r0).sort().values
        rows = rows.to(dev)
        b64 = b[gi].double()
        pre = a[rows].double() @ b64.t()
        sab = a[rows].double().abs() @ b64.abs().t()
        r, tol = expected_rows(pre, sab, k, n, None, act, gated)
        ratio_g, frob_g = rows_verdict(d[rows], r, tol)
        worst, frob = max(worst, ratio_g), max(frob, frob_g)
    parity = parity_reduce({"ok": worst <= 1.0 and frob <= 1e-2 and not bad_nan,
                            "max_ratio": worst, "frob_sampled": frob, "frob_tol": 1e-2,
                            "checks": f"{max(1, PARITY_ROWS // groups)} sampled rows per group "
                                      f"element-wise (fused SwiGLU: no linear checksums)"}, world)
    flops_per_gpu = 2.0 * t * b_rows * k
    value = flops_per_gpu * world / (ms * 1e-3) / 1e12
    achieved = flops_per_gpu / (ms_local * 1e-3) / 1e12
    peaks, peak_src = load_peaks()
    if rank == 0:
        line = {
            "metric": metric_name(args.workload, args.m), "value": value, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16",
            "data": "synthetic",
            "config": workload_config(args, world),
            "kernel_config": {"group_rows": sizes, "tile": [128, tile_n], "cluster": [cm, 1, 1],
                              "ab_stage": stages, "scheduler": args.scheduler},
            "per_rank": per_rank, "parity": parity,
            "roofline": {"bound": "tensor", "achieved": achieved, "peak": peaks["bf16_tflops"],
                         "unit": "TFLOP/s", "frac": achieved / peaks["bf16_tflops"],
                         "peak_source": f"{peak_src} bf16_tflops (cuBLAS burst)",
                         "frac_sustained": achieved / peaks.get("bf16_tflops_sustained",
                                                                peaks["bf16_tflops"]),
                         "traffic": None, "algorithmic_flops_per_launch": flops_per_gpu,
                         "kernel": "group_tile_prefix_kernel + cpg::gemm_sm100_kernel (grouped)"},
            "clocks": clocks, "gpu_launches": 2 * args.steps * world, "e2e": None,
            "cpu_baseline": None,
        }
        print(json.dumps(line), flush=True)
    if not parity["ok"]:
        raise SystemExit(f"parity check failed: {parity}")


# ------------------------------------------------------------------ GPU arm
def run_cpg(args, world, rank, local):
    import torch
    from cutedsl_pingpong_gemm_b200 import GemmSM90, RasterOrder, compile as cpg_compile

    w = WORKLOADS[args.workload]
    n, k = w["n"], w["k"]
    m_w = args.m or w["m"]
    m = m_w if w["m_is_per_gpu"] else m_w // world
    dev = torch.device("cuda", local)
    stream = torch.cuda.current_stream(dev)

    # Inputs generated on the device with the workload's distribution (A rows differ per rank,
    # B is the same replicated weight on every rank).
    gen_a = torch.Generator(device=dev).manual_seed(1000 + rank)
    gen_b = torch.Generator(device=dev).manual_seed(7)
    gated = bool(w.get("gated"))
    act = w.get("act") or args.activation
    b_rows = 2 * n if gated else n
    a = (torch.randn(m, k, generator=gen_a, device=dev) * w["a_scale"]).to(torch.bfloat16)
    b = (torch.randn(b_rows, k, generator=gen_b, device=dev) * w["b_scale"]).to(torch.bfloat16)
    bias = (torch.randn(n, generator=gen_b, device=dev)).to(torch.bfloat16) if w["bias"] else None
    d = torch.empty(m, n, dtype=torch.bfloat16, device=dev)
    scale_a = scale_b = None
    if w.get("small_m"):
        args.cluster_m = 1  # one 128-row tile: the pair's second CTA would have no rows
    ref_ctor = bool(w.get("ref_ctor"))  # the reference harness's own constructor arguments
    tile_n = args.tile_n or (128 if w.get("small_m") else 256 if ref_ctor else
                             (512 if args.cluster_m == 2 or gated else 256))
    if w["fp8"] is not None:
        from cutedsl_pingpong_gemm_b200.quant import quantize_e4m3
        if w["fp8"] == "tensor":
            a, scale_a = quantize_e4m3(a)
            b, scale_b = quantize_e4m3(b)
        else:
            a, scale_a = quantize_e4m3(a, (1, 128))
            b, scale_b = quantize_e4m3(b, (128, 128))
            tile_n = args.tile_n if args.tile_n in (128, 256) else 256
        torch.cuda.synchronize()

    cm = args.cluster_m
    stages = args.stages or (3 if ref_ctor else
                             {(512, 2): 3, (512, 1): 2, (256, 2): 6, (256, 1): 4}.get(
                                 (tile_n, cm), 8 if cm == 2 else 6))
    epi_stage = args.epi_stages or 2
    if w["fp8"] == "block" and not args.stages:
        # Deepest ring that fits 227 KiB next to 8 promotion warps' epilogue staging (4 KiB per
        # warp and epilogue stage).
        stages, epi_stage = {(128, 1): (5, 2), (128, 2): (8, 1), (256, 1): (4, 1),
                             (256, 2): (6, 1)}[(tile_n, cm)]
    gemm = GemmSM90(tile_shape_mn=(128, tile_n), epi_tile_mn=(128, 32),
                    cluster_shape_mnk=(cm, 1, 1), atom_layout_mn=(2, 1) if ref_ctor else (1, 1),
                    ab_stage=stages, epi_stage=epi_stage, raster_order=RasterOrder.AlongN,
                    reuse_ab=False, is_persistent=True,
                    dynamic_scheduler=args.scheduler == "dynamic")
    compiled = cpg_compile(gemm, a, b, d, stream, scale_a=scale_a, scale_b=scale_b, gated=gated)
    # The split is picked from the tile count (M <= 128: the small-M kernel; few tiles: K ranges
    # or Stream-K); fused epilogues and block scales run whole.
    fused_epi = gated or act is not None or w["fp8"] == "block"
    split_k = args.split_k if args.split_k else (1 if fused_epi else compiled.auto_split_k(m, n, k))
    compiled(a, b, d, stream, bias=bias, scale_a=scale_a, scale_b=scale_b, split_k=split_k,
             activation=act, gated=gated)
    torch.cuda.synchronize()
    ws_path = split_k > 1 or split_k == -1  # FP32 workspace + cast kernel (BF16 D)
    if ws_path:
        plan = compiled.plan_for(a, b, compiled._workspace(d), 0, split_k)
    else:
        plan = compiled.plan_for(a, b, d, 1 if w["fp8"] == "block" else 0, split_k, gated=gated)
    info = plan.launch_info()
    # The raster group size the plan uses (the reference's 8; lowered under the dynamic schedule).
    group_size = plan.sched_params().dm_group_size.divisor
    # K ranges and Stream-K into a BF16 D add the cast kernel (the hybrid finishes in the GEMM).
    kernels_per_step = 2 if ws_path else 1

    launches = [0]

    def step():
        compiled(a, b, d, stream, bias=bias, scale_a=scale_a, scale_b=scale_b, split_k=split_k,
                 activation=act, gated=gated)
        launches[0] += kernels_per_step

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()
    use_graph = args.graph == "on" or (args.graph == "auto" and bool(w.get("small_m")))
    # The timed region runs `units`: (callable, steps it makes) in order, exactly args.steps.
    units = [(step, 1)] * args.steps
    if use_graph:
        # A step of tens of microseconds is bound by the host's launch path (measured: 40.5 us
        # eager vs 32.9 us replayed one call per graph for M = 128); a serving loop replays a
        # graph of consecutive calls, in which each GEMM (a programmatic dependent of the one
        # before) sets up while the previous one finishes.  Graphs of up to GRAPH_STEPS calls.
        def capture(count):
            cap = torch.cuda.Stream(dev)
            cap.wait_stream(stream)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=cap):
                for _ in range(count):
                    compiled(a, b, d, cap, bias=bias, scale_a=scale_a, scale_b=scale_b,
                             split_k=split_k, activation=act, gated=gated)
            stream.wait_stream(cap)
            return g

        group = max(1, min(args.steps, GRAPH_STEPS))
        graphs = {group: capture(group)}
        rem = args.steps % group
        if rem:
            graphs[rem] = capture(rem)

        def replayer(count):
            def run():
                graphs[count].replay()
                launches[0] += kernels_per_step * count
            return run

        units = [(replayer(group), group)] * (args.steps // group)
        if rem:
            units.append((replayer(rem), rem))
        for _ in range(3):
            replayer(group)()
    torch.cuda.synchronize()
    barrier(world)
    torch.cuda.synchronize()

    sampler = ClockSampler(local)
    launches[0] = 0
    e0 = torch.cuda.Event(enable_timing=True)
    e1 = torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for i, (run_unit, _) in enumerate(units):
        run_unit()
        if i == 0:
            sampler.start()  # the GPU is busy from here on: no idle-clock samples
    assert sum(c for _, c in units) == args.steps
    e1.record(stream)
    torch.cuda.synchronize()
    sampler.stop()
    barrier(world)
    n_launch = launches[0]
    ms_local = e0.elapsed_time(e1) / args.steps
    ms = reduce_max(ms_local, world)
    status = plan.status()
    if status != 0:
        raise SystemExit(f"kernel status {status:#x}")
    clocks = sampler.summary()
    per_rank = per_rank_summary(ms_local, clocks, world)

    # ---------------- post-run parity of the D the last timed step wrote (every rank)
    if w["fp8"] is None:
        a_ref, b_ref = a, b
    elif w["fp8"] == "tensor":
        a_ref, b_ref = dequantized(a, scale_a, "tensor"), dequantized(b, scale_b, "tensor")
    else:
        a_ref = dequantized(a, scale_a, "block", (1, 128))
        b_ref = dequantized(b, scale_b, "block", (128, 128))
    frob_tol = 3e-2 if w["fp8"] else 1e-2
    parity = parity_reduce(parity_dense(d, a_ref, b_ref, k, bias=bias, act=act, gated=gated,
                                        frob_tol=frob_tol, seed=rank), world)

    flops_per_gpu = 2.0 * m * b_rows * k  # a gated step computes gate and up: 2 N columns
    total_flops = flops_per_gpu * world
    value = total_flops / (ms * 1e-3) / 1e12
    achieved = flops_per_gpu / (ms_local * 1e-3) / 1e12  # one kernel launch per step
    peaks, peak_src = load_peaks()
    # HBM-bound shapes: the roofline is bytes moved / time against the measured copy bandwidth.
    min_bytes = (m * k + b_rows * k) * a.element_size() + m * n * d.element_size()

    # ---------------- end to end through the public API with host buffers
    e2e = None
    if not args.no_e2e:
        # Every step uploads its A and B from pinned host memory and downloads its D, through
        # the public API.  Steps are pipelined over two device buffer sets and three streams:
        # the upload of step i + 1 and the download of step i - 1 overlap the GEMM of step i
        # (PCIe moves both directions at once), as a serving loop would run them.
        a_h = a.cpu().pin_memory()
        b_h = b.cpu().pin_memory()
        h2d = torch.cuda.Stream(dev)
        d2h = torch.cuda.Stream(dev)
        sets = [(torch.empty_like(a), torch.empty_like(b), torch.empty_like(d),
                 torch.empty(d.shape, dtype=d.dtype).pin_memory()) for _ in range(2)]
        in_ready = [torch.cuda.Event() for _ in range(2)]
        gemm_done = [torch.cuda.Event() for _ in range(2)]
        out_done = [torch.cuda.Event() for _ in range(2)]
        for j in range(2):
            gemm_done[j].record(stream)
            out_done[j].record(stream)

        def e2e_step(i):
            j = i % 2
            a2, b2, d2, dh = sets[j]
            h2d.wait_event(gemm_done[j])  # the GEMM that last read this buffer set is done
            with torch.cuda.stream(h2d):
                a2.copy_(a_h, non_blocking=True)
                b2.copy_(b_h, non_blocking=True)
            in_ready[j].record(h2d)
            stream.wait_event(in_ready[j])
            stream.wait_event(out_done[j])  # D of the previous use of this set is downloaded
            compiled(a2, b2, d2, stream, bias=bias, scale_a=scale_a, scale_b=scale_b,
                     split_k=split_k, activation=act, gated=gated)
            gemm_done[j].record(stream)
            d2h.wait_event(gemm_done[j])
            with torch.cuda.stream(d2h):
                dh.copy_(d2, non_blocking=True)
            out_done[j].record(d2h)

        for i in range(2):
            e2e_step(i)
        torch.cuda.synchronize()
        barrier(world)
        torch.cuda.synchronize()
        f0 = torch.cuda.Event(enable_timing=True)
        f1 = torch.cuda.Event(enable_timing=True)
        f0.record(stream)
        h2d.wait_stream(stream)  # no upload starts before the timed region
        for i in range(args.e2e_steps):
            e2e_step(i)
        stream.wait_stream(h2d)
        stream.wait_stream(d2h)
        f1.record(stream)
        torch.cuda.synchronize()
        barrier(world)
        e2e_ms = reduce_max(f0.elapsed_time(f1) / args.e2e_steps, world)
        # The downloaded D of the last step passes the same check as the timed run's D (split-K
        # and Stream-K add partial sums in an order that varies between launches, so the bytes
        # may differ within the tolerance).
        last = sets[(args.e2e_steps - 1) % 2][3]
        e2e_parity = parity_dense(last.to(dev), a_ref, b_ref, k, bias=bias, act=act, gated=gated,
                                  frob_tol=frob_tol, seed=rank + 1)
        same = reduce_max(0.0 if e2e_parity["ok"] else 1.0, world) == 0.0
        e2e = {"value": total_flops / (e2e_ms * 1e-3) / 1e12, "unit": "TFLOP/s",
               "output_parity_ok": same,
               "h2d_bytes_per_step": int((a.numel() + b.numel()) * a.element_size() * world),
               "d2h_bytes_per_step": int(d.numel() * d.element_size() * world),
               "steps": args.e2e_steps, "ms_per_step": e2e_ms,
               "gpu_launches": args.e2e_steps * world,
               "path": "GemmSM90 compiled call (C ABI cpg_gemm_run); every step uploads A, B from "
                       "pinned host memory and downloads D; uploads of step i + 1 and the "
                       "download of step i - 1 overlap the GEMM of step i (two buffer sets)"}

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        rows = 512
        rate, cores, reps, el = cpu_matmul_rate(rows, n, k, args.cpu_seconds)
        cpu = {"value": rate, "unit": "TFLOP/s", "cores": cores, "kind": "port",
               "sample": f"{reps} x fp32 torch.matmul of a {rows}x{k} row slab against B^T "
                         f"({n}x{k}) on the host, {el:.1f} s"}

    if rank == 0:
        peak = peaks["bf16_tflops"]
        nominal = NOMINAL_DENSE_BF16_TFLOPS
        peak_note = f"{peak_src} bf16_tflops (cuBLAS burst)"
        if w["fp8"] is not None:
            # No measured FP8 tensor peak exists on this pool; the dense nominal is the bound.
            nominal = NOMINAL_DENSE_FP8_TFLOPS
            peak = NOMINAL_DENSE_FP8_TFLOPS
            peak_note = "nominal dense FP8 (no measured FP8 peak available)"
        line = {
            "metric": metric_name(args.workload, args.m), "value": value, "unit": "TFLOP/s",
            "n_gpus": world, "steps": args.steps, "warmup": args.warmup, "ms_per_step": ms,
            "higher_is_better": True, "scaling": "weak" if w["m_is_per_gpu"] else "strong",
            "vs_baseline": None, "dtype": "e4m3" if w["fp8"] else "bf16", "data": "synthetic",
            "pct_nominal_dense_peak": 100.0 * value / (nominal * world),
            "config": workload_config(args, world),
            "kernel_config": {"tile": [128, tile_n], "cluster": [cm, 1, 1],
                              "atom": list(gemm.atom_layout_mnk[:2]), "ab_stage": stages,
                              "epi_stage": epi_stage, "grid": list(info["grid"]),
                              "smem_bytes": info["smem_bytes"], "split_k": split_k,
                              "scheduler": gemm.dynamic_scheduler and "dynamic" or "static",
                              "group_size": group_size,
                              "cuda_graph": (f"graphs of {min(args.steps, GRAPH_STEPS)} calls"
                                             if use_graph else False),
                              "reference_constructor": ref_ctor},
            "per_rank": per_rank, "parity": parity,
            "roofline": ({"bound": "hbm", "achieved": min_bytes / (ms_local * 1e-3) / 1e9,
                          "peak": peaks["hbm_gbs"], "unit": "GB/s",
                          "frac": min_bytes / (ms_local * 1e-3) / 1e9 / peaks["hbm_gbs"],
                          "peak_source": f"{peak_src} hbm_gbs",
                          "traffic": (load_traffic(args.workload, args.scheduler, args.m)
                                      if split_k == -3 else None),
                          "algorithmic_bytes_per_step": min_bytes, "split_k": split_k,
                          "kernel": ("cpg::gemm_decode_kernel" if split_k == -3 else
                                     ("cpg::gemm_sm100_kernel (Stream-K)" if split_k == -1 else
                                      "cpg::gemm_sm100_kernel (split-K)") +
                                     " + cast_f32_bf16_kernel")}
                         if w.get("small_m") else
                         {"bound": "tensor", "achieved": achieved, "peak": peak, "unit": "TFLOP/s",
                         "frac": achieved / peak, "peak_source": peak_note,
                         "frac_sustained": (achieved / peaks.get("bf16_tflops_sustained", peak)
                                            if w["fp8"] is None else None),
                         "traffic": load_traffic(args.workload, args.scheduler, args.m),
                         "algorithmic_flops_per_launch": flops_per_gpu,
                         "kernel": ("cpg::gemm_fp8_block_kernel" if w["fp8"] == "block"
                                    else "cpg::gemm_sm100_kernel")}),
            "clocks": clocks,
            "gpu_launches": n_launch * world,
            "e2e": e2e,
            "cpu_baseline": cpu,
        }
        print(json.dumps(line), flush=True)
    del a_ref, b_ref
    if not parity["ok"] or (e2e is not None and not e2e["output_parity_ok"]):
        raise SystemExit(f"parity check failed: {parity}")


def main():
    args = parse_args()
    if args.scheduler == "auto":
        w = WORKLOADS[args.workload]
        dense = not (w.get("small_m") or w.get("groups") or w["fp8"] == "block"
                     or w.get("ref_ctor"))
        args.scheduler = "dynamic" if dense else "static"
    if args.impl == "reference":
        world = int(os.environ.get("WORLD_SIZE", "1"))
        rank = int(os.environ.get("RANK", "0"))
        run_reference(args, world, rank)
        return
    world, rank, local = dist_setup(args.gpus)
    try:
        if WORKLOADS[args.workload].get("split") == "k":
            run_tallk(args, world, rank, local)
        elif WORKLOADS[args.workload].get("groups"):
            run_grouped(args, world, rank, local)
        else:
            run_cpg(args, world, rank, local)
    finally:
        if world > 1:
            import torch.distributed as dist
            dist.destroy_process_group()


if __name__ == "__main__":
    main()
