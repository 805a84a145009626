"""Failure detection on the GPU without a fault: a kernel-side bounded wait is
made to run out on purpose and reports B2G_ERR_TIMEOUT, and the handle then runs
a normal GEMM that matches the CPU oracle.

The reference's waits are unbounded spins (umma_throughput/umma_tput.cu:510-520),
so a lost arrival hangs the GPU.  b2g_selftest_wait has one warp wait, through the
GEMM's own bounded-wait code and with a 1 ms limit set by b2g_set_wait_limit, on an
mbarrier phase that no thread arrives at (mode 0) or a global flag that nothing
sets (mode 1, the split-tail epilogue's wait).  Nothing else is in flight: no TMA,
no MMA, no TMEM held.
"""
import pytest

import b2g
from b2g import _lib
from test_gemm_gpu import check_small

pytestmark = pytest.mark.gpu

LIMIT_NS = 1_000_000  # 1 ms


@pytest.mark.parametrize("mode", [0, 1], ids=["mbarrier", "flag"])
def test_bounded_wait_expires_and_handle_recovers(engine, mode):
    engine.set_wait_limit(LIMIT_NS)
    try:
        st, elapsed = engine.selftest_wait(mode)
        assert st == _lib.B2G_ERR_TIMEOUT, f"status {st}"
        # the wait gave up after its limit, not long after it
        assert LIMIT_NS <= elapsed < 200 * LIMIT_NS, elapsed
        # b2g_selftest_wait cleared the error word: the next check is clean
        engine.check()
        # a GEMM on the same handle, under the same short limit, runs and is right
        check_small(engine, "bf16", 256, 256, 512, cta_group=2)
        check_small(engine, "e4m3", 300, 200, 528, cta_group=1)
    finally:
        engine.set_wait_limit(0)
    # and again with the default limit
    check_small(engine, "bf16", 256, 256, 512, cta_group=1)


def test_wait_limit_range_is_checked(engine):
    for bad in (1, 999, 2_000_000_001):
        with pytest.raises(b2g.B2GError) as e:
            engine.set_wait_limit(bad)
        assert e.value.status == 1
    engine.set_wait_limit(1000)
    engine.set_wait_limit(0)
    with pytest.raises(b2g.B2GError):
        st = engine.lib.b2g_selftest_wait(engine.h, 2, None, None)
        engine._ok(st, "b2g_selftest_wait")
