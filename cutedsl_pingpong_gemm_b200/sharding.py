"""Multi-GPU GEMM on one node: one process per GPU, torch.distributed for the plumbing.

Two decompositions of D = A . B^T (the reference has none; it is a single-GPU kernel):

* ``MShardedGemm`` -- rows of A and D are split across ranks in whole 128-row tiles, B (the
  weight) is replicated, and every rank runs the sm_100a GEMM on its rows.  There is no
  collective on the data path, so the ranks scale independently.
* ``SplitKGemm`` -- for tall-K shapes (M, N small, K large) each rank multiplies its K range into
  an fp32 partial [M, N] with the same kernel (fp32 epilogue), the partials are summed with one
  NCCL reduce-scatter over NVLink (rank r receives rows ``row_range(M, world, r)``), and a cast
  kernel rounds the reduced rows to BF16.
* ``PeerSplitK`` -- the same split-K without the collective: each rank's GEMM epilogue adds its
  FP32 partial tiles straight into the buffer of the rank owning their rows (NVLink atomics into
  memory mapped between the processes), overlapping the exchange with the next tiles' math, and
  each rank rounds its own rows once every rank's tiles have arrived.

The range arithmetic is plain Python so that the decomposition can be exercised on CPU ranks
(gloo) with any per-rank compute function; the GPU compute always goes through the C ABI.
"""
from typing import Callable, List, Optional, Tuple

TILE_M = 128
K_ALIGN = 64


def row_range(m: int, world: int, rank: int, align: int = TILE_M) -> Tuple[int, int]:
    """Rows [start, stop) of rank ``rank`` when ``m`` rows are split over ``world`` ranks.

    Whole ``align``-row tiles are dealt out as evenly as possible (earlier ranks take the extra
    tile); the last rank also takes the ragged remainder.  Ranges are disjoint and cover [0, m).
    """
    if world < 1 or not (0 <= rank < world):
        raise ValueError(f"bad rank {rank} of world {world}")
    tiles = -(-m // align) if m > 0 else 0
    base, extra = divmod(tiles, world)
    start_tile = rank * base + min(rank, extra)
    ntiles = base + (1 if rank < extra else 0)
    start = min(start_tile * align, m)
    stop = min((start_tile + ntiles) * align, m)
    return start, stop


def k_ranges(k: int, parts: int, align: int = K_ALIGN) -> List[Tuple[int, int]]:
    """Split [0, k) into ``parts`` contiguous ranges whose starts are multiples of ``align``."""
    return [row_range(k, parts, p, align) for p in range(parts)]


def reduce_scatter_rows(partial, world: int, group=None):
    """Sum ``partial`` [M, N] over ranks; return this rank's rows (``row_range`` split, padded
    so every rank holds the same number of rows for the collective).

    NCCL: one ``reduce_scatter_tensor``.  Other backends (gloo on CPU, used by the tests): an
    all-reduce followed by a slice, which has the same result.
    """
    import torch
    import torch.distributed as dist
    m, n = partial.shape
    rank = dist.get_rank(group)
    per = max(row_range(m, world, r)[1] - row_range(m, world, r)[0] for r in range(world))
    if dist.get_backend(group) == "nccl":
        if per * world == m:  # equal shards: reduce-scatter straight from the partial
            out = partial.new_empty((per, n))
            dist.reduce_scatter_tensor(out, partial.contiguous(), op=dist.ReduceOp.SUM, group=group)
            return out
        padded = partial.new_zeros((per * world, n))
        for r in range(world):
            s, e = row_range(m, world, r)
            padded[r * per: r * per + (e - s)] = partial[s:e]
        out = partial.new_empty((per, n))
        dist.reduce_scatter_tensor(out, padded, op=dist.ReduceOp.SUM, group=group)
        s, e = row_range(m, world, rank)
        return out[: e - s]
    full = partial.clone()
    dist.all_reduce(full, op=dist.ReduceOp.SUM, group=group)
    s, e = row_range(m, world, rank)
    return full[s:e].contiguous()


class MShardedGemm:
    """M-sharded GEMM: this rank computes D[rows] = A[rows] . B^T (+ bias) with its own GPU."""

    def __init__(self, gemm, world: int, rank: int):
        self.gemm = gemm
        self.world = world
        self.rank = rank

    def rows(self, m: int) -> Tuple[int, int]:
        return row_range(m, self.world, self.rank)

    def __call__(self, a_shard, b, d_shard, stream=None, *, bias=None, alpha: float = 1.0):
        """``a_shard``/``d_shard`` are this rank's rows (see ``rows``); B is the full weight."""
        self.gemm(a_shard, b, d_shard, stream, bias=bias, alpha=alpha)


class SplitKGemm:
    """Split-K across ranks with an NCCL reduce-scatter of fp32 partials.

    ``partial_fn(a_k, b_k) -> fp32 [M, N]`` computes one rank's partial product (for the B rows
    it is given) and ``cast_fn(rows, cs, ce, out)`` turns reduced fp32 rows of columns [cs, ce)
    into the output (writing ``out`` when given); ``SplitKGemm.on_gpu`` builds both from the
    sm_100a kernels (FP32-epilogue GEMM, ``cpg_cast_f32_bf16``).

    With ``chunks`` > 1 the columns are cut into that many ranges: chunk c's GEMM runs on the
    caller's stream while the reduce-scatter (and cast) of chunk c - 1 runs on a second stream,
    so the collective overlaps the compute and only the last chunk's exchange is exposed.
    """

    CHUNK_ALIGN = 256  # column chunks start on tile boundaries

    @staticmethod
    def on_gpu(gemm, world: int, rank: int, group=None, bias=None, local_split_k: int = 1,
               chunks: int = 1):
        """GPU instance: partials by ``gemm`` (a GemmSM90) into FP32, cast to BF16 (+ bias).

        ``local_split_k`` additionally splits each rank's K range inside the GPU (the kernel's
        L dimension; 0 picks from the tile count, Stream-K for few tiles) when the per-rank
        problem has too few tiles to fill the SMs.
        """
        import torch
        from .quant import cast_f32_bf16

        def partial(a_k, b_k):
            out = torch.empty(a_k.shape[0], b_k.shape[0], dtype=torch.float32, device=a_k.device)
            gemm(a_k, b_k, out, None, split_k=local_split_k)
            return out

        def cast(rows, cs, ce, out=None):
            return cast_f32_bf16(rows, None if bias is None else bias[cs:ce], out=out)

        return SplitKGemm(world, rank, partial, cast, group, chunks=chunks,
                          out_dtype=torch.bfloat16)

    def __init__(self, world: int, rank: int, partial_fn: Callable, cast_fn: Optional[Callable] = None,
                 group=None, chunks: int = 1, out_dtype=None):
        self.world = world
        self.rank = rank
        self.partial_fn = partial_fn
        self.cast_fn = cast_fn
        self.group = group
        self.chunks = max(1, int(chunks))
        self.out_dtype = out_dtype  # dtype of cast_fn's output (None: the partials' dtype)
        self._comm = {}

    def k_range(self, k: int) -> Tuple[int, int]:
        return k_ranges(k, self.world)[self.rank]

    def column_chunks(self, n: int) -> List[Tuple[int, int]]:
        """Non-empty column ranges [cs, ce) of the chunked exchange, in order."""
        cols = [row_range(n, self.chunks, c, self.CHUNK_ALIGN) for c in range(self.chunks)]
        return [(cs, ce) for cs, ce in cols if ce > cs]

    def __call__(self, a_k, b_k, m: int, n: int):
        """``a_k`` [M, k_r] and ``b_k`` [N, k_r] hold this rank's K range.  Returns this rank's
        rows of D (``row_range(m, world, rank)``), cast by ``cast_fn`` when given."""
        if self.world > 1 and self.chunks > 1 and n > self.CHUNK_ALIGN:
            return self._chunked(a_k, b_k, m, n)
        partial = self.partial_fn(a_k, b_k)
        if tuple(partial.shape) != (m, n):
            raise ValueError(f"partial has shape {tuple(partial.shape)}, expected {(m, n)}")
        rows = partial if self.world == 1 else reduce_scatter_rows(partial, self.world, self.group)
        return self.cast_fn(rows, 0, n) if self.cast_fn is not None else rows

    def _chunked(self, a_k, b_k, m: int, n: int):
        import torch
        s, e = row_range(m, self.world, self.rank)
        on_gpu = a_k.is_cuda
        out = None
        if on_gpu:
            compute = torch.cuda.current_stream(a_k.device)
            comm = self._comm.get(a_k.device)
            if comm is None:
                comm = self._comm[a_k.device] = torch.cuda.Stream(a_k.device)
        for cs, ce in self.column_chunks(n):
            partial = self.partial_fn(a_k, b_k[cs:ce])
            if tuple(partial.shape) != (m, ce - cs):
                raise ValueError(f"partial has shape {tuple(partial.shape)}, "
                                 f"expected {(m, ce - cs)}")
            if not on_gpu:
                rows = reduce_scatter_rows(partial, self.world, self.group)
                out = self._place(rows, cs, ce, s, e, n, out)
                continue
            ready = torch.cuda.Event()
            ready.record(compute)
            with torch.cuda.stream(comm):
                comm.wait_event(ready)
                partial.record_stream(comm)
                rows = reduce_scatter_rows(partial, self.world, self.group)
                out = self._place(rows, cs, ce, s, e, n, out)
        if on_gpu:
            compute.wait_stream(comm)
            out.record_stream(compute)
        return out

    def _place(self, rows, cs, ce, s, e, n, out):
        """Write reduced rows of columns [cs, ce) into this rank's [e - s, n] output."""
        if out is None:
            dtype = self.out_dtype if self.cast_fn is not None and self.out_dtype else rows.dtype
            out = rows.new_empty((e - s, n), dtype=dtype)
        if self.cast_fn is None:
            out[:, cs:ce] = rows
        else:
            self.cast_fn(rows, cs, ce, out[:, cs:ce])
        return out


def peer_row_starts(m: int, world: int) -> List[int]:
    """Row block boundaries of the split-K output: rank q owns rows [starts[q], starts[q + 1])
    (``row_range``), so starts[0] = 0 and starts[world] = m."""
    return [row_range(m, world, q)[0] for q in range(world)] + [m]


class PeerSplitK:
    """Split-K across ranks with the reduce-scatter done by the GEMM's epilogue over peer memory.

    Rank r passes its K range of A and B (``k_ranges``); the sm_100a GEMM adds every FP32
    partial tile into the owning rank's buffer (``cpg_gemm_run_reduce_scatter``) and counts
    itself there; ``cpg_peer_finish`` then waits on this rank's counter for every rank's tiles
    and writes this rank's rows of D in BF16 (+ bias), clearing its buffer.  Two buffers per rank
    alternate between calls, so a rank that runs one call ahead adds into the other one; the
    counter only grows, and each finish waits for the running total of arrivals.

    The buffers are ``cudaMalloc`` memory mapped into the other processes with CUDA IPC handles
    exchanged once per shape over ``group`` (no multicast objects), so the first call with a new
    shape is collective: every rank makes its calls with the same shapes in the same order.
    Needs N a multiple of 4 and GPUs that can map each other's memory (NVLink / NVSwitch).
    ``check_status()`` raises if a finish gave up waiting (a rank missing); ``close()``
    (collective) frees everything: call it on every rank before the process group goes away.
    """

    def __init__(self, gemm, world: int, rank: int, group=None, bias=None, local_split_k: int = 0,
                 timeout_ms: int = 10000):
        if world > 8:
            raise ValueError("at most 8 ranks")
        self.gemm = gemm
        self.world, self.rank, self.group = world, rank, group
        self.bias = bias
        self.local_split_k = local_split_k
        self.timeout_ms = int(timeout_ms)
        self._states = {}
        self._status = None

    # -------------------------------------------------------------- setup (once per shape)
    def _split(self, compiled, m: int, n: int, k: int) -> int:
        from . import _lib
        if self.local_split_k > 0:
            return self.local_split_k
        s = compiled.auto_split_k(m, n, k)
        if s < 1:
            # Stream-K cuts tiles into partial ranges; the exchange counts whole (tile, K range)
            # segments, so take K ranges (about three waves of them) instead.
            gemm = self.gemm
            cm, cn, _ = gemm.cluster_shape_mnk
            col_tiles = -(-n // gemm.cta_tile_shape_mnk[1])
            tiles = -(-m // (128 * cm)) * -(-col_tiles // cn)
            kblocks = -(-k // 64)
            s = max(1, min(-(-3 * gemm.max_active_clusters // max(tiles, 1)), kblocks // 4))
        return s

    def _state(self, a_k, b_k, m: int, n: int):
        import ctypes
        import torch
        import torch.distributed as dist
        from . import _lib
        from .gemm_base import CompiledGemm, _Plan
        k = a_k.shape[1]
        dev = a_k.device
        key = (m, n, k, a_k.stride(0), b_k.stride(0), dev.index)
        st = self._states.get(key)
        if st is not None:
            return st
        if n % 4 != 0:
            raise _lib.CpgError(_lib.CPG_ERR_ALIGNMENT, "the peer reduce-scatter needs N % 4 == 0")
        lib = _lib.load()
        starts = peer_row_starts(m, self.world)
        ld = n
        rows_max = max(starts[q + 1] - starts[q] for q in range(self.world))
        compiled = CompiledGemm(self.gemm)
        split = self._split(compiled, m, n, k)
        dt_ab = {torch.bfloat16: _lib.CPG_DTYPE_BF16, torch.float8_e4m3fn: _lib.CPG_DTYPE_E4M3}[a_k.dtype]
        lda = a_k.stride(0) if m > 1 else max(8, k)
        ldb = b_k.stride(0) if n > 1 else max(8, k)
        plan = _Plan(self.gemm, m, n, k, lda, ldb, ld, dev.index, dt_ab, _lib.CPG_DTYPE_F32, 0,
                     split)
        # Two buffers of this rank's rows and one 64-byte counter, mapped by every rank.
        own, handles = [], []
        for nbytes in (max(rows_max, 1) * ld * 4, max(rows_max, 1) * ld * 4, 64):
            ptr, h = ctypes.c_void_p(), _lib.IpcHandleC()
            _lib.check(lib.cpg_peer_alloc(nbytes, ctypes.byref(ptr), ctypes.byref(h)), "peer_alloc")
            own.append(ptr.value)
            handles.append(bytes(h.bytes))
        gathered = [None] * self.world
        dist.all_gather_object(gathered, handles, group=self.group)
        opened, mapped = [], []
        for q in range(self.world):
            if q == self.rank:
                mapped.append(list(own))
                continue
            row = []
            for hb in gathered[q]:
                h = _lib.IpcHandleC()
                ctypes.memmove(h.bytes, hb, 64)
                ptr = ctypes.c_void_p()
                _lib.check(lib.cpg_peer_open(ctypes.byref(h), ctypes.byref(ptr)), "peer_open")
                opened.append(ptr.value)
                row.append(ptr.value)
            mapped.append(row)
        rs = []
        for buf in range(2):
            r = _lib.ReduceScatterC()
            r.ranks, r.rank, r.ld = self.world, self.rank, ld
            for q in range(self.world + 1):
                r.row_start[q] = starts[q]
            for q in range(self.world):
                r.dst[q] = mapped[q][buf]
                r.count[q] = mapped[q][2]
            rs.append(r)
        per_rank = (ctypes.c_uint32 * self.world)()
        _lib.check(lib.cpg_gemm_rs_arrivals(plan.handle, ctypes.byref(rs[0]), per_rank),
                   "rs_arrivals")
        all_arrivals = [None] * self.world
        dist.all_gather_object(all_arrivals, list(per_rank), group=self.group)
        expected = sum(arr[self.rank] for arr in all_arrivals) & 0xFFFFFFFF
        if self._status is None:
            self._status = torch.zeros(1, dtype=torch.int32, device=dev)
        st = dict(plan=plan, rs=rs, own=own, opened=opened, expected=expected, calls=0,
                  rows=(starts[self.rank], starts[self.rank + 1]), ld=ld, split=split)
        self._states[key] = st
        return st

    # -------------------------------------------------------------- one call
    def __call__(self, a_k, b_k, m: int, n: int, stream=None):
        """This rank's rows of D = A . B^T (BF16, + bias), from its K range ``a_k`` [M, k_r],
        ``b_k`` [N, k_r]."""
        import ctypes
        import torch
        from . import _lib
        from .gemm_base import _stream_handle
        st = self._state(a_k, b_k, m, n)
        lib = _lib.load()
        dev = a_k.device
        h = _stream_handle(stream, dev)
        buf = st["calls"] % 2
        epi = _lib.EpilogueC(1.0, None, None, None, 0.0, 0, None, 0, 0)
        _lib.check(lib.cpg_gemm_run_reduce_scatter(
            st["plan"].handle, a_k.data_ptr() if a_k.numel() else None,
            b_k.data_ptr() if b_k.numel() else None, ctypes.byref(st["rs"][buf]),
            ctypes.byref(epi), h), "gemm_run_reduce_scatter")
        st["calls"] += 1
        target = (st["calls"] * st["expected"]) & 0xFFFFFFFF
        r0, r1 = st["rows"]
        out = torch.empty(r1 - r0, n, dtype=torch.bfloat16, device=dev)
        bias = self.bias
        _lib.check(lib.cpg_peer_finish(st["own"][buf], st["ld"], st["own"][2], target, r1 - r0, n,
                                       out.data_ptr() if out.numel() else None, n,
                                       None if bias is None else bias.data_ptr(),
                                       self._status.data_ptr(), self.timeout_ms, h),
                   "peer_finish")
        return out

    def check_status(self) -> None:
        """Raise if a finish gave up waiting for the other ranks (synchronises)."""
        from . import _lib
        if self._status is not None and int(self._status.item()) != 0:
            raise _lib.CpgError(_lib.CPG_ERR_DEVICE_TIMEOUT,
                                f"peer reduce-scatter status {int(self._status.item()):#x}")

    def close(self) -> None:
        """Collective: wait for every rank, then unmap the peers' buffers and free this rank's."""
        import torch
        import torch.distributed as dist
        from . import _lib
        if not self._states:
            return
        torch.cuda.synchronize()
        dist.barrier(group=self.group)
        lib = _lib.load()
        for st in self._states.values():
            for ptr in st["opened"]:
                lib.cpg_peer_close(ptr)
        dist.barrier(group=self.group)
        for st in self._states.values():
            for ptr in st["own"]:
                lib.cpg_peer_free(ptr)
        self._states.clear()
