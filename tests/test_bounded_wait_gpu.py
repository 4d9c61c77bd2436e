"""The device-side bounded wait (no counterpart in the reference, whose
kernels have no waits with limits).

Every tensor-core pipeline waits on mbarriers through one helper that gives
up after a time limit, records a stage code in the kernel's error word and
returns; the host then reports VRS_ERR_TIMEOUT instead of hanging. Here that
helper waits for 1 ms on an mbarrier nothing arrives on (no copy or MMA in
flight): the call must report the timeout through the C ABI and the device
must keep working afterwards."""
import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def test_bounded_wait_gives_up_and_reports_timeout(vc, orc, gpu):
    L = vc.lib()
    st = L.vrs_selftest_bounded_wait(1_000_000)
    assert st == 7, L.vrs_last_error()
    assert b"stage code 99" in L.vrs_last_error()
    # The context is still usable: a search right after is exact.
    s = vc.config_seed(900)
    base = vc.gen_rows_host(vc.GEN_NORMAL, s, 0, 0, 3000, 64)
    qs = vc.gen_rows_host(vc.GEN_NORMAL, s, 1, 0, 20, 64)
    eng = vc.DistributedKnnEngine.try_new(base, 64, 1, vc.GpuShardMode.Sharded, vc.DistanceMetric.L2Squared)
    dg, ig = eng.search_arrays(qs, 10)
    eng.close()
    do, io = orc.knn_search(base, qs, 10, 0)
    assert np.array_equal(ig, io) and np.array_equal(dg.view(np.uint32), do.view(np.uint32))


def test_bounded_wait_rejects_out_of_range_limits(vc, gpu):
    L = vc.lib()
    assert L.vrs_selftest_bounded_wait(10) == 5
    assert L.vrs_selftest_bounded_wait(5_000_000_000) == 5
