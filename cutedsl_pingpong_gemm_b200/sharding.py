"""Multi-GPU GEMM on one node: one process per GPU, torch.distributed for the plumbing.

Two decompositions of D = A . B^T (the reference has none; it is a single-GPU kernel):

* ``MShardedGemm`` -- rows of A and D are split across ranks in whole 128-row tiles, B (the
  weight) is replicated, and every rank runs the sm_100a GEMM on its rows.  There is no
  collective on the data path, so the ranks scale independently.
* ``SplitKGemm`` -- for tall-K shapes (M, N small, K large) each rank multiplies its K range into
  an fp32 partial [M, N] with the same kernel (fp32 epilogue), the partials are summed with one
  NCCL reduce-scatter over NVLink (rank r receives rows ``row_range(M, world, r)``), and a cast
  kernel rounds the reduced rows to BF16.

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
