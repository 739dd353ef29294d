"""CPU oracle for the GEMM hot path -- TEST INFRASTRUCTURE ONLY.

Nothing in the product package imports this directory.  Only ``tests/``,
``__graft_entry__.smoke()`` and the ``cpu_baseline`` / ``--impl reference`` legs of
``bench.py`` use it, and only as the checker or the timed CPU baseline.

Contents:

* ``fast_math_ref``      -- restatement of the reference's ``FastDivmod`` (fast_math.py:17-81).
* ``tile_scheduler_ref`` -- restatement of ``SimpleTileScheduler`` (tile_scheduler.py:20-183).
* ``gemm_ref``           -- fp32 CPU matmul ``D = A @ B.T`` (gemm_base.py:590) and the
  tolerance checks stated by the project spec.

Pinning: ``fast_math_ref`` and ``tile_scheduler_ref`` are checked bit-exact against golden
vectors produced by executing the reference's own Python code under CuTe-DSL
(``tests/golden/gen_golden.py``).  The numerical GEMM oracle is the spec itself
(``ref = a @ b.t()``, gemm_base.py:590); the reference kernel is sm_90a-only and ships no
golden outputs, so numeric parity against the reference kernel's outputs is unpinned and is
stated as a tolerance against the fp32 product instead.
"""
