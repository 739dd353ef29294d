"""The GEMM operator with the interface of the reference's ``gemm_base.GemmSM90``.

Drop-in surface (adelmuursepp/cutedsl_pingpong_gemm, gemm_base.py):

* ``GemmSM90(tile_shape_mn, epi_tile_mn, cluster_shape_mnk, atom_layout_mn, ab_stage=2,
  epi_stage=2, raster_order=RasterOrder.AlongN, reuse_ab=True, is_persistent=False,
  gemm_n_prologue=0)`` -- same arguments, defaults and constructor asserts (gemm_base.py:50-122).
* ``compile(gemm, a, b, c, stream, options=None)`` -- stands in for ``cute.compile(gemm, a, b, c,
  stream, options=...)`` (gemm_base.py:608) and returns a callable ``compiled(a, b, c, stream)``
  (gemm_base.py:609) that writes ``c = a @ b.T`` in place, stream-ordered, without syncing.
* ``gemm(a, b, c, stream)`` compiles on first use and runs.

``a`` is [M, K], ``b`` is [N, K] and ``c`` is [M, N], all BF16 CUDA tensors with unit stride in
the last dimension (the reference's harness layout, gemm_base.py:587-590).  Beyond the reference,
``a``/``b`` may be FP8 E4M3 (``torch.float8_e4m3fn``, with per-tensor ``scale_a``/``scale_b``
device scalars) and ``c`` may be FP32 (split-K partials); ``bias`` adds a BF16 per-column vector.  Underneath, every call
goes through the C ABI of ``libcpgemm.so`` into hand-written sm_100a kernels (tcgen05 MMA into
TMEM, TMA loads/stores, persistent grouped tile scheduler); there is no other execution path.

Argument meaning on sm_100a:

* ``tile_shape_mn``: the CTA tile, (128, N) with N in {64, 128, 256, 512} (512: CTA pairs only,
  the benchmarks' default: a 256 x 512 pair tile fills the 512 TMEM columns).
* ``cluster_shape_mnk``: (1,1,1) runs one CTA per tile; (2,1,1) runs CTA pairs that issue
  ``tcgen05.mma.cta_group::2`` on a 256-row tile (each CTA loads its own A rows and half of B);
  (1,2,1) and (2,2,1) group independent CTAs/pairs along N.  Clusters only change the tile order
  otherwise; no TMA load is multicast.
* ``ab_stage``: depth of the shared-memory A/B ring; ``epi_stage``: TMA-store staging buffers per
  epilogue warp; ``reuse_ab``: the epilogue stages through the A/B ring (single-tile CTAs only).
* ``atom_layout_mn``, ``epi_tile_mn`` and ``gemm_n_prologue`` are validated exactly as in the
  reference; the tcgen05 kernel issues its MMAs from one thread into TMEM, so they do not change
  the launch.
"""
import ctypes
import functools
import math
from typing import Optional, Tuple

from . import _lib
from .tile_scheduler import RasterOrder, SimpleTileScheduler, get_max_active_clusters

THREADS_PER_WG = 128
# Threads per CTA of the sm_100a kernel: TMA warp + MMA warp + 4 epilogue warps; 512-wide tiles
# add 2 idle warps to complete the first warpgroup and use 8 epilogue warps.
THREADS_PER_CTA_SM100 = 192
THREADS_PER_CTA_SM100_WIDE = 384


@functools.lru_cache(maxsize=None)
def _dtype_tables():
    """(A/B dtype -> CPG code, D dtype -> CPG code)."""
    import torch
    ab = {torch.bfloat16: _lib.CPG_DTYPE_BF16, torch.float8_e4m3fn: _lib.CPG_DTYPE_E4M3}
    d = {torch.bfloat16: _lib.CPG_DTYPE_BF16, torch.float32: _lib.CPG_DTYPE_F32}
    return ab, d


def _stream_handle(stream, device) -> int:
    """cudaStream_t value for None / torch stream / cuda-python CUstream / int."""
    import torch
    if stream is None:
        return torch.cuda.current_stream(device).cuda_stream
    if isinstance(stream, torch.cuda.Stream):
        return stream.cuda_stream
    if isinstance(stream, int):
        return stream
    get_ptr = getattr(stream, "getPtr", None)
    if get_ptr is not None:
        return int(get_ptr())
    return int(stream)


class CompiledGemm:
    """Result of ``compile``: ``compiled(a, b, c, stream)`` launches the sm_100a kernel.

    Plans (validated problem + launch shape) are cached per (M, N, K, strides, device), so a
    compiled GEMM accepts any shape its configuration supports, like the reference's kernel
    compiled on symbolic shapes.  The FP32 split-K workspaces are cached per stream as well, so
    launches on two streams never share one.  A plan's own device state (the grouped GEMM's tile
    prefix, the hybrid split's fixup workspace and counters) is rebuilt by each launch, so
    launches of such a plan must be stream-ordered: concurrent streams use one ``CompiledGemm``
    each.  (Plans are not keyed by stream: creating one allocates device memory, which a CUDA
    graph capture on a fresh stream would forbid.)  ``release()`` drops the caches.  One host
    thread at a time may call a compiled GEMM (its plans cache tensor maps).
    """

    def __init__(self, gemm: "GemmSM90"):
        self.gemm = gemm
        self._plans = {}
        self._workspaces = {}

    def _plan(self, a, b, c, scale_mode: int = 0, split_k: int = 1, gated: bool = False):
        import torch
        gemm = self.gemm
        ab_codes, d_codes = _dtype_tables()
        # gemm_base.py:514 requires BF16 everywhere; sm_100a adds FP8 E4M3 operands and FP32 D.
        assert a.dtype == b.dtype and a.dtype in ab_codes and c.dtype in d_codes, \
            "A, B and D must be BF16 (gemm_base.py:514), or FP8 E4M3 A/B, or FP32 D"
        nd = a.dim()
        if nd not in (2, 3) or b.dim() != nd or c.dim() != nd:
            raise _lib.CpgError(_lib.CPG_ERR_INVALID_SHAPE,
                                "A, B and D must all be 2-D, or all 3-D [L, rows, cols] (batched)")
        batches = a.shape[0] if nd == 3 else 1
        if nd == 3 and (b.shape[0] != batches or c.shape[0] != batches):
            raise _lib.CpgError(_lib.CPG_ERR_INVALID_SHAPE,
                                f"batch counts differ: A{tuple(a.shape)} B{tuple(b.shape)} "
                                f"D{tuple(c.shape)}")
        m, k = a.shape[-2:]
        n, kb = b.shape[-2:]
        b_rows = n
        if gated:
            # B = [W_gate; W_up] (2N rows), D is M x N.
            n //= 2
            if b_rows != 2 * n:
                raise _lib.CpgError(_lib.CPG_ERR_INVALID_SHAPE,
                                    f"gated B must have an even number of rows, got {b_rows}")
        if kb != k or tuple(c.shape[-2:]) != (m, n):
            raise _lib.CpgError(_lib.CPG_ERR_INVALID_SHAPE,
                                f"shapes A{tuple(a.shape)} B{tuple(b.shape)} D{tuple(c.shape)} "
                                f"do not form D = A @ B.T" + (" (gated)" if gated else ""))
        for name, t in (("A", a), ("B", b), ("D", c)):
            if t.numel() > 0 and t.stride(-1) != 1:
                raise _lib.CpgError(_lib.CPG_ERR_UNSUPPORTED,
                                    f"{name} must have unit stride in its last dimension")
            if t.numel() > 0 and not t.is_cuda:
                raise _lib.CpgError(_lib.CPG_ERR_NO_DEVICE, f"{name} must be a CUDA tensor")
        def row_stride(t, rows, cols):
            # A single-row or empty tensor's row stride is never used; give the padded row length.
            per16 = 16 // t.element_size()
            if rows > 1 and cols > 0:
                return t.stride(-2)
            return max(per16, -(-cols // per16) * per16)

        lda, ldb, ldd = row_stride(a, m, k), row_stride(b, b_rows, k), row_stride(c, m, n)
        # The L mode of the reference's (M, K, L) tensors (gemm_base.py:221 fixes it at one).
        l = batches if batches > 1 else 0
        bsa, bsb, bsd = (a.stride(0), b.stride(0), c.stride(0)) if l else (0, 0, 0)
        dev = c.device.index if c.is_cuda else torch.cuda.current_device()
        dt_ab, dt_d = ab_codes[a.dtype], d_codes[c.dtype]
        key = (m, n, k, lda, ldb, ldd, dev, dt_ab, dt_d, scale_mode, split_k, bool(gated), l,
               bsa, bsb, bsd)
        plan = self._plans.get(key)
        if plan is None:
            plan = _Plan(gemm, m, n, k, lda, ldb, ldd, dev, dt_ab, dt_d, scale_mode, split_k,
                         gated, l, bsa, bsb, bsd)
            self._plans[key] = plan
        return plan

    def plan_for(self, a, b, c, scale_mode: int = 0, split_k: int = 1,
                 gated: bool = False) -> "_Plan":
        return self._plan(a, b, c, scale_mode, split_k, gated)

    def __call__(self, a, b, c, stream=None, *, bias=None, alpha: float = 1.0, scale_a=None,
                 scale_b=None, split_k: int = 1, activation: Optional[str] = None,
                 source=None, beta: float = 1.0, gated: bool = False):
        """``split_k`` > 1 cuts K into that many ranges scheduled as the kernel's L dimension;
        ``split_k=-1`` is Stream-K (every resident cluster takes an equal share of the (tile,
        k-block) pairs); with a BF16 ``c`` both add their partial sums into an FP32 workspace
        that is then rounded into ``c`` (plus bias).  ``split_k=-2`` computes all full waves but
        the last whole and shares the rest Stream-K style, the kernel finishing each split tile
        from its own FP32 workspace.  ``split_k=0`` picks from the tile count (``auto_split_k``).

        Fused epilogue (none of it exists in the reference, whose kernel computes D = A . B^T,
        gemm_base.py:133): ``c = act(alpha * A . B^T + bias + beta * source)`` with
        ``activation`` one of None, "relu", "silu", "gelu", "gelu_tanh" and ``source`` an
        optional tensor of c's type and shape (it may be ``c`` itself).  ``gated=True`` (tile_n
        512): ``b`` is the stacked [W_gate; W_up] of 2 N rows and
        ``c = act(alpha * A . W_gate^T) * (alpha * A . W_up^T)`` (SwiGLU with "silu").
        Activations, ``source`` and ``gated`` need the whole K in one pass (split_k 1)."""
        import torch
        if activation not in _lib.ACTIVATIONS:
            raise _lib.CpgError(_lib.CPG_ERR_INVALID_CONFIG, f"unknown activation {activation!r}")
        act = _lib.ACTIVATIONS[activation]
        fused = act != _lib.CPG_ACT_NONE or source is not None or gated
        # More than one scale per operand selects the block-scaled FP8 kernel (A: 1 x 128,
        # B: 128 x 128 blocks, layouts of cpgemm.h); one value each is a per-tensor scale.
        block = scale_a is not None and scale_a.numel() > 1
        mode = _lib.CPG_SCALE_BLOCK if block else _lib.CPG_SCALE_TENSOR
        if a.dim() == 3 and a.shape[0] == 0:
            return None  # no batches: nothing to compute
        if split_k == 0:
            batches = a.shape[0] if a.dim() == 3 else 1
            split_k = 1 if (block or fused) else self.auto_split_k(
                a.shape[-2], b.shape[-2], a.shape[-1], batches)
        split_k = int(split_k)
        if (split_k > 1 or split_k == _lib.CPG_SPLIT_K_STREAM) and c.dtype == torch.bfloat16:
            if c.dim() == 3 and not c.is_contiguous():
                raise _lib.CpgError(_lib.CPG_ERR_UNSUPPORTED,
                                    "batched split-K into BF16 needs a contiguous D")
            ws = self._workspace(c, stream)
            plan = self._plan(a, b, ws, mode, split_k)
            plan.run(a, b, ws, stream, bias=None, alpha=alpha, scale_a=scale_a, scale_b=scale_b)
            from .quant import cast_f32_bf16
            n = c.shape[-1]
            cast_f32_bf16(ws.reshape(-1, n), bias, out=c.reshape(-1, n), stream=stream)
            return None
        plan = self._plan(a, b, c, mode, split_k, gated)
        plan.run(a, b, c, stream, bias=bias, alpha=alpha, scale_a=scale_a, scale_b=scale_b,
                 activation=act, source=source, beta=beta)
        return None

    def grouped(self, a, b, c, group_offsets, stream=None, *, bias=None, alpha: float = 1.0,
                scale_a=None, scale_b=None, activation: Optional[str] = None, source=None,
                beta: float = 1.0, gated: bool = False):
        """Grouped GEMM (ragged groups, e.g. the experts of an MoE layer), on the device alone:
        for every group g, ``c[r] = epilogue(a[r] @ b[g].T)`` for the rows
        ``group_offsets[g] <= r < group_offsets[g + 1]``.

        ``a`` [T, K] holds the groups' rows one after the other, ``b`` [G, N, K] (or
        [G, 2N, K] with ``gated``), ``c`` [T, N]; ``group_offsets`` is an int32 CUDA tensor of
        G + 1 non-decreasing offsets within [0, T] (read on the device: no host synchronisation);
        rows outside every group are not written.  Epilogue options as in ``__call__``; no
        split-K and no block scales.  The reference has no grouped form (its kernel fixes the L
        mode at one, gemm_base.py:221)."""
        import torch
        if activation not in _lib.ACTIVATIONS:
            raise _lib.CpgError(_lib.CPG_ERR_INVALID_CONFIG, f"unknown activation {activation!r}")
        if a.dim() != 2 or b.dim() != 3 or c.dim() != 2:
            raise _lib.CpgError(_lib.CPG_ERR_INVALID_SHAPE,
                                "grouped: a [T, K], b [G, N, K] and c [T, N]")
        groups = b.shape[0]
        if not (group_offsets.is_cuda and group_offsets.dtype == torch.int32
                and group_offsets.dim() == 1 and group_offsets.numel() == groups + 1
                and group_offsets.is_contiguous()):
            raise _lib.CpgError(_lib.CPG_ERR_INVALID_SHAPE,
                                "group_offsets must be a contiguous int32 CUDA tensor of G + 1")
        if groups == 0 or a.shape[0] == 0:
            return None
        plan = self._grouped_plan(a, b, c, gated)
        plan.run(a, b, c, stream, bias=bias, alpha=alpha, scale_a=scale_a, scale_b=scale_b,
                 activation=_lib.ACTIVATIONS[activation], source=source, beta=beta,
                 group_offsets=group_offsets)
        return None

    def _grouped_plan(self, a, b, c, gated):
        import torch
        ab_codes, d_codes = _dtype_tables()
        assert a.dtype == b.dtype and a.dtype in ab_codes and c.dtype in d_codes, \
            "A, B and D must be BF16 (gemm_base.py:514), or FP8 E4M3 A/B, or FP32 D"
        t, k = a.shape
        groups, b_rows, kb = b.shape
        n = b_rows // 2 if gated else b_rows
        if kb != k or tuple(c.shape) != (t, n) or (gated and b_rows != 2 * n):
            raise _lib.CpgError(_lib.CPG_ERR_INVALID_SHAPE,
                                f"grouped shapes A{tuple(a.shape)} B{tuple(b.shape)} "
                                f"D{tuple(c.shape)} do not match")
        for name, x in (("A", a), ("B", b), ("D", c)):
            if x.numel() > 0 and (x.stride(-1) != 1 or not x.is_cuda):
                raise _lib.CpgError(_lib.CPG_ERR_UNSUPPORTED,
                                    f"{name} must be a CUDA tensor with unit last stride")
        per16 = 16 // a.element_size()
        lda = a.stride(0) if t > 1 else max(per16, -(-k // per16) * per16)
        ldb = b.stride(1) if b_rows > 1 else max(per16, -(-k // per16) * per16)
        ldd = c.stride(0) if t > 1 else max(16 // c.element_size(), n)
        dev = c.device.index
        dt_ab, dt_d = ab_codes[a.dtype], d_codes[c.dtype]
        key = ("grouped", t, n, k, groups, lda, ldb, ldd, b.stride(0), dev, dt_ab, dt_d, bool(gated))
        plan = self._plans.get(key)
        if plan is None:
            plan = _Plan(self.gemm, t, n, k, lda, ldb, ldd, dev, dt_ab, dt_d, 0, 1, gated, groups,
                         0, b.stride(0), 0, grouped=True)
            self._plans[key] = plan
        return plan

    def _workspace(self, c, stream=None):
        """FP32 [M, N] buffer for split-K partial sums (kept and reused per shape, device and
        stream: each launch clears it on its own stream first)."""
        import torch
        key = (tuple(c.shape), c.device, _stream_handle(stream, c.device))
        ws = self._workspaces.get(key)
        if ws is None:
            ws = torch.empty(c.shape, dtype=torch.float32, device=c.device)
            self._workspaces[key] = ws
        return ws

    def release(self) -> None:
        """Drop the cached plans and split-K workspaces; their device memory is freed and the next
        call plans again.  Call it only when no launch that uses them is still running and no
        captured CUDA graph will replay them (a graph keeps the pointers it was captured with)."""
        self._plans.clear()
        self._workspaces.clear()

    def auto_split_k(self, m: int, n: int, k: int, batches: int = 1) -> int:
        """When the output tiles alone cannot fill the GPU: K ranges that fill whole waves of
        the resident clusters when K is long enough (``wave_split_k``), else Stream-K for a
        persistent kernel (-1; decode-like small M), else about three waves of K ranges; 1 when
        the tiles fill the GPU.

        Measured on one B200, 2048 x 2048 output tiles of 256 x 256 (32 clusters) with K = 65536:
        Stream-K 981 TFLOP/s, 5 ranges (2.2 waves) 1272, 2 ranges (one 86 % wave) 1319.

        One batch of M <= 128 rows takes the small-M kernel instead (CPG_SPLIT_K_DECODE, -3: B's
        rows on the MMA's M side, K split over a cluster and reduced in shared memory, one
        launch): on N = K = 8192 it measured 28.2 / 31.1 / 34.5 us for M = 16 / 64 / 128 against
        32.8 / 34.6 / 34.8 us for Stream-K + cast."""
        if m <= 128 and batches == 1:
            return _lib.CPG_SPLIT_K_DECODE
        gemm = self.gemm
        cm, cn, _ = gemm.cluster_shape_mnk
        tiles = -(-max(m, 1) // (128 * cm)) * -(-max(n, 1) // gemm.cta_tile_shape_mnk[1])
        tiles = -(-tiles // cn) * max(batches, 1)
        slots = gemm.max_active_clusters
        if tiles >= slots:
            # Whole tiles even when the last wave is partial: on one GPU's 2048-row shard of the
            # LLM shape (448 pair tiles on 74 pairs, 6.05 waves) the data-parallel + Stream-K
            # hybrid (split_k=-2) measured 1342 vs 1357 TFLOP/s: the few clusters of a partial
            # last wave run faster under the power cap than the full waves.
            return 1
        kblocks = -(-max(k, 1) // 64)
        # Very long K: split-K ranges advance through K together and share A / B in L2, while
        # Stream-K clusters sit at unrelated K offsets and stream all of A and B (measured 30 %
        # slower at K = 65536); any reasonably full wave of ranges is better there.
        s = wave_split_k(tiles, kblocks, slots, min_fill=0.85 if kblocks >= 256 else 0.95)
        if s is not None:
            return s
        if gemm.is_persistent and not gemm.dynamic_scheduler and kblocks >= 8:
            return _lib.CPG_SPLIT_K_STREAM
        want = -(-3 * slots // tiles)
        return max(1, min(want, kblocks // 4))


def wave_split_k(clusters: int, kblocks: int, slots: int, min_kblocks: int = 32,
                 min_fill: float = 0.95) -> Optional[int]:
    """Number of K ranges s >= 2 (each keeping >= ``min_kblocks`` k-blocks) whose
    clusters * s work units best fill their last wave of ``slots`` resident clusters; among
    fills within 5 % of the best, the smallest s (fewer partial-sum passes).  None when the best
    fill is below ``min_fill``."""
    fills = []
    for s in range(2, kblocks // min_kblocks + 1):
        units = clusters * s
        fills.append((units / (-(-units // slots) * slots), s))
    if not fills:
        return None
    best = max(f for f, _ in fills)
    if best < min_fill:
        return None
    return min(s for f, s in fills if f >= best - 0.05)


class _Plan:
    """One ``cpg_gemm`` handle: fixed problem, kernel variant and launch grid."""

    def __init__(self, gemm: "GemmSM90", m, n, k, lda, ldb, ldd, device, dtype_ab, dtype_d,
                 scale_mode=0, split_k=1, gated=False, l=0, batch_stride_a=0, batch_stride_b=0,
                 batch_stride_d=0, grouped=False):
        self.lib = _lib.load()
        self.m, self.n, self.k = m, n, k
        self.l = l
        self.device = device
        self.scale_mode = scale_mode
        cfg = gemm._config_c()
        prob = _lib.GemmProblemC(m, n, k, lda, ldb, ldd, dtype_ab, dtype_d, scale_mode, split_k,
                                 1 if gated else 0, l, batch_stride_a, batch_stride_b,
                                 batch_stride_d, 1 if grouped else 0)
        self.grouped = grouped
        h = ctypes.c_void_p()
        _lib.check(self.lib.cpg_gemm_create(ctypes.byref(cfg), ctypes.byref(prob), int(device),
                                            ctypes.byref(h)), "compile")
        self.handle = h

    def __del__(self):
        h = getattr(self, "handle", None)
        if h is not None and h.value:
            try:
                self.lib.cpg_gemm_destroy(h)
            except Exception:
                pass
            self.handle = None

    def launch_info(self):
        grid = (ctypes.c_int32 * 3)()
        cluster = (ctypes.c_int32 * 3)()
        threads, smem, mac = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_int32()
        _lib.check(self.lib.cpg_gemm_launch_info(self.handle, grid, cluster, ctypes.byref(threads),
                                                 ctypes.byref(smem), ctypes.byref(mac)))
        return {"grid": tuple(grid), "cluster": tuple(cluster), "threads": threads.value,
                "smem_bytes": smem.value, "max_active_clusters": mac.value}

    def sched_params(self) -> SimpleTileScheduler.Params:
        c = _lib.SchedParamsC()
        _lib.check(self.lib.cpg_gemm_sched_params(self.handle, ctypes.byref(c)))
        return SimpleTileScheduler.Params.from_c(c)

    def set_trace(self, buf, tiles_per_cta: int) -> None:
        ptr = None if buf is None else buf.data_ptr()
        _lib.check(self.lib.cpg_gemm_set_trace(self.handle, ptr, int(tiles_per_cta)), "set_trace")

    def set_timeout_ms(self, ms: int) -> None:
        _lib.check(self.lib.cpg_gemm_set_timeout_ms(self.handle, int(ms)), "set_timeout_ms")

    def set_fault_injection(self, flags: int) -> None:
        """Test hook (see cpg_gemm_set_fault_injection): 1 = producer issues no loads."""
        _lib.check(self.lib.cpg_gemm_set_fault_injection(self.handle, int(flags)),
                   "set_fault_injection")

    def status(self) -> int:
        s = ctypes.c_int32()
        rc = self.lib.cpg_gemm_status(self.handle, ctypes.byref(s))
        if rc not in (_lib.CPG_OK, _lib.CPG_ERR_DEVICE_TIMEOUT):
            _lib.check(rc, "status")
        return s.value

    def run(self, a, b, c, stream=None, *, bias=None, alpha: float = 1.0, scale_a=None,
            scale_b=None, activation: int = 0, source=None, beta: float = 1.0,
            group_offsets=None) -> None:
        import torch
        if bias is not None:
            if not (bias.dtype == torch.bfloat16 and bias.is_cuda and bias.numel() == self.n
                    and (bias.dim() == 1 or bias.is_contiguous())):
                raise _lib.CpgError(_lib.CPG_ERR_INVALID_SHAPE,
                                    "bias must be a contiguous BF16 CUDA tensor of length N")
            if bias.stride(-1) != 1:
                raise _lib.CpgError(_lib.CPG_ERR_UNSUPPORTED, "bias must be contiguous")
        scales = []
        if self.scale_mode == _lib.CPG_SCALE_BLOCK:
            nkb, nnb = -(-self.k // 128), -(-self.n // 128)
            want = {"scale_a": (nkb, self.m), "scale_b": (nnb, nkb)}
        else:
            want = {"scale_a": (1,), "scale_b": (1,)}
        for name, sc in (("scale_a", scale_a), ("scale_b", scale_b)):
            if sc is not None and not (sc.is_cuda and sc.dtype == torch.float32 and sc.is_contiguous()
                                       and sc.numel() == math.prod(want[name])):
                raise _lib.CpgError(_lib.CPG_ERR_INVALID_SHAPE,
                                    f"{name} must be a contiguous float32 CUDA tensor of shape "
                                    f"{want[name]}")
            scales.append(None if sc is None else sc.data_ptr())
        src_ptr, ld_src, bs_src = None, 0, 0
        if source is not None:
            if not (source.is_cuda and source.dtype == c.dtype and source.shape == c.shape
                    and (source.numel() == 0 or source.stride(-1) == 1)):
                raise _lib.CpgError(_lib.CPG_ERR_INVALID_SHAPE,
                                    "source must be a CUDA tensor of D's dtype and shape with unit "
                                    "column stride")
            per16 = 16 // source.element_size()
            ld_src = source.stride(-2) if self.m > 1 else max(per16, -(-self.n // per16) * per16)
            bs_src = source.stride(0) if source.dim() == 3 else 0
            src_ptr = source.data_ptr() if source.numel() else None
        epi = _lib.EpilogueC(float(alpha), None if bias is None else bias.data_ptr(), *scales,
                             float(beta), int(activation), src_ptr, int(ld_src), int(bs_src))
        st = _stream_handle(stream, c.device)
        if self.grouped:
            rc = self.lib.cpg_gemm_run_grouped(self.handle, a.data_ptr() if a.numel() else None,
                                               b.data_ptr() if b.numel() else None, c.data_ptr(),
                                               group_offsets.data_ptr(), ctypes.byref(epi), st)
        else:
            rc = self.lib.cpg_gemm_run(self.handle, a.data_ptr() if a.numel() else None,
                                       b.data_ptr() if b.numel() else None, c.data_ptr(),
                                       ctypes.byref(epi), st)
        _lib.check(rc, "gemm")


class GemmSM90:
    """gemm_base.py:49-566: constructor surface and asserts of the reference, sm_100a kernels."""

    def __init__(
        self,
        tile_shape_mn: Tuple[int, int],
        epi_tile_mn: Tuple[int, int],
        cluster_shape_mnk: Tuple[int, int, int],
        atom_layout_mn: Tuple[int, int],
        ab_stage: int = 2,
        epi_stage: int = 2,
        raster_order: RasterOrder = RasterOrder.AlongN,
        reuse_ab: bool = True,
        is_persistent: bool = False,
        gemm_n_prologue: int = 0,
        *,
        dynamic_scheduler: bool = False,
    ):
        """dynamic_scheduler (not in the reference): one cluster per cluster tile in the grid and
        cluster launch control, so running clusters take over the tiles of clusters that have
        not started (the tile map is the same; is_persistent is then ignored)."""
        import torch
        self.acc_dtype = torch.float32
        self.raster_order = raster_order
        self.scheduler_group_size = 8
        self.cluster_shape_mnk = tuple(cluster_shape_mnk)
        # K tile: one 128-byte swizzled row of the operands (64 BF16; compile() sets 128 for
        # FP8 E4M3 operands, see cta_tile_k).
        self.cta_tile_shape_mnk = (*tile_shape_mn, 64)
        tile_M, tile_N = self.cta_tile_shape_mnk[0], self.cta_tile_shape_mnk[1]

        # Atom layout (gemm_base.py:72-75)
        assert atom_layout_mn[0] in [1, 2, 3] and atom_layout_mn[1] in [1, 2]
        assert atom_layout_mn[0] == 1 or tile_M % (atom_layout_mn[0] * 64) == 0
        assert atom_layout_mn[1] == 1 or tile_N % (atom_layout_mn[1] * 32) == 0
        self.atom_layout_mnk = (*atom_layout_mn, 1)

        # Multicast fan-out the reference derives (gemm_base.py:77-82); kept for introspection.
        # The sm_100a kernels never multicast a TMA load.
        self.mcast_ctas_a = self.cluster_shape_mnk[1]
        self.mcast_ctas_b = self.cluster_shape_mnk[0]
        self.is_a_mcast = False
        self.is_b_mcast = False

        self.occupancy = 1
        self.mma_warpgroups = math.prod(self.atom_layout_mnk)
        assert self.mma_warpgroups in [1, 2, 3]
        self.threads_per_cta = THREADS_PER_CTA_SM100_WIDE if tile_N == 512 else THREADS_PER_CTA_SM100

        self.ab_stage = ab_stage
        self.epi_stage = epi_stage
        self.dtype = torch.bfloat16
        self.buffer_align_bytes = 1024

        self.epi_tile_mn = tuple(epi_tile_mn)
        self.reuse_ab = reuse_ab
        assert not (self.atom_layout_mnk[1] > 1) or self.epi_tile_mn[1] == self.cta_tile_shape_mnk[1], \
            'When atom layout n > 1, we need epi tile n = cta tile n'

        self.is_persistent = is_persistent
        self._max_active_clusters = None
        self.gemm_n_prologue = gemm_n_prologue

        assert not (self.reuse_ab and self.is_persistent), "Persistent kernel can't reuse AB for epilogue"
        self.dynamic_scheduler = bool(dynamic_scheduler)
        assert not (self.reuse_ab and self.dynamic_scheduler), \
            "Dynamic scheduler runs several tiles per CTA and can't reuse AB for epilogue"
        self._compiled: Optional[CompiledGemm] = None

    @staticmethod
    def cta_tile_k(dtype) -> int:
        """K extent of one pipeline stage: a 128-byte swizzled row of the operand type (64 BF16
        elements, 128 FP8 E4M3)."""
        import torch
        return 128 if dtype == torch.float8_e4m3fn else 64

    @property
    def max_active_clusters(self) -> int:
        """gemm_base.py:117, queried lazily (it needs the GPU)."""
        if self._max_active_clusters is None:
            self._max_active_clusters = get_max_active_clusters(math.prod(self.cluster_shape_mnk))
        return self._max_active_clusters

    def _config_c(self) -> "_lib.GemmConfigC":
        cm, cn, ck = self.cluster_shape_mnk
        return _lib.GemmConfigC(
            self.cta_tile_shape_mnk[0], self.cta_tile_shape_mnk[1],
            self.epi_tile_mn[0], self.epi_tile_mn[1],
            cm, cn, ck,
            self.atom_layout_mnk[0], self.atom_layout_mnk[1],
            self.ab_stage, self.epi_stage, int(self.raster_order),
            int(bool(self.reuse_ab)), int(bool(self.is_persistent)), int(self.gemm_n_prologue),
            int(self.scheduler_group_size), int(self.dynamic_scheduler))

    def validate(self) -> None:
        """Run the C ABI's copy of the constructor checks (no GPU needed)."""
        lib = _lib.load()
        cfg = self._config_c()
        _lib.check(lib.cpg_config_validate(ctypes.byref(cfg)), "GemmSM90")

    def compile(self, a, b, c, stream=None, *, scale_a=None, scale_b=None,
                gated: bool = False) -> CompiledGemm:
        """Validate and plan for the example tensors.  Block scales (``scale_a`` with more than
        one element, as in ``__call__``) plan the block-scaled FP8 kernel instead of the plain one;
        ``gated`` plans the gated FFN form (B = [W_gate; W_up])."""
        compiled = CompiledGemm(self)
        self.cta_tile_shape_mnk = (*self.cta_tile_shape_mnk[:2], self.cta_tile_k(a.dtype))
        block = scale_a is not None and scale_a.numel() > 1
        compiled.plan_for(a, b, c, _lib.CPG_SCALE_BLOCK if block else _lib.CPG_SCALE_TENSOR,
                          gated=gated)
        self._compiled = compiled
        return compiled

    def release(self) -> None:
        """Free what the implicit compiled GEMM of ``__call__`` / ``grouped`` caches (see
        ``CompiledGemm.release``)."""
        if self._compiled is not None:
            self._compiled.release()

    def grouped(self, a, b, c, group_offsets, stream=None, **epilogue):
        """Grouped GEMM (see ``CompiledGemm.grouped``)."""
        if self._compiled is None:
            self._compiled = CompiledGemm(self)
        return self._compiled.grouped(a, b, c, group_offsets, stream, **epilogue)

    def __call__(self, a, b, c, stream=None, *, bias=None, alpha: float = 1.0, scale_a=None,
                 scale_b=None, split_k: int = 1, activation: Optional[str] = None, source=None,
                 beta: float = 1.0, gated: bool = False):
        if self._compiled is None:
            self._compiled = CompiledGemm(self)
        self._compiled(a, b, c, stream, bias=bias, alpha=alpha, scale_a=scale_a, scale_b=scale_b,
                       split_k=split_k, activation=activation, source=source, beta=beta,
                       gated=gated)


# The B200 name of the same operator.
GemmSM100 = GemmSM90


def compile(gemm: GemmSM90, a, b, c, stream=None, options: Optional[str] = None, *,
            scale_a=None, scale_b=None, gated: bool = False) -> CompiledGemm:
    """Stand-in for ``cute.compile(gemm, a, b, c, stream, options=...)`` (gemm_base.py:608).

    ``options`` is accepted for call-site compatibility and ignored (there is no JIT).  FP8
    callers may pass their scales so that the plan matches the kernel the call will use.
    """
    return gemm.compile(a, b, c, stream, scale_a=scale_a, scale_b=scale_b, gated=gated)
