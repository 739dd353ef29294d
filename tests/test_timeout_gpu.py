"""Failure detection without a GPU fault: the kernel's bounded waits.

With the host-side fault injection the producer issues no loads, so the MMA warp's `full` wait
can never complete.  The kernel must give up after the plan's deadline, record the wait site in
the status word, stop its other roles, free TMEM and return; the context stays usable and the
next normal launch is correct.
"""
import time

import pytest
import torch

from cutedsl_pingpong_gemm_b200 import GemmSM90, _lib, compile as cpg_compile
from oracle import gemm_ref

pytestmark = pytest.mark.gpu

SITE_MMA_FULL = 2
SITE_EPI_TMEM_FULL = 4


@pytest.mark.parametrize("cluster", [(1, 1, 1), (2, 1, 1)])
def test_wait_deadline_reports_status_and_recovers(cluster):
    m, n, k = 512, 512, 256
    a, b, _ = gemm_ref.make_inputs(m, n, k, seed=2)
    da, db = a.cuda(), b.cuda()
    d = torch.zeros(m, n, dtype=torch.bfloat16, device="cuda")
    gemm = GemmSM90((128, 256), (128, 32), cluster, (1, 1), ab_stage=4, reuse_ab=False,
                    is_persistent=True)
    compiled = cpg_compile(gemm, da, db, d)
    plan = compiled.plan_for(da, db, d)
    plan.set_timeout_ms(300)
    plan.set_fault_injection(_lib.CPG_INJECT_SKIP_LOADS)
    t0 = time.time()
    compiled(da, db, d)
    torch.cuda.synchronize()
    elapsed = time.time() - t0
    status = plan.status()
    assert status & 0x100, hex(status)
    assert status & 0xFF in (SITE_MMA_FULL, SITE_EPI_TMEM_FULL), hex(status)
    assert elapsed < 10.0
    # Normal operation afterwards: correct output and a clean status word.
    plan.set_fault_injection(0)
    compiled(da, db, d)
    torch.cuda.synchronize()
    assert plan.status() == 0
    res = gemm_ref.check(d.cpu(), a, b)
    assert res["ok"], res
