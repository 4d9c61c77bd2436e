"""The allocation-free kNN entry point (vrs_knn_search_noalloc).

It exists for callers that cannot allocate device memory while searching:
code in allocation-free or captured regions, plugin hosts and caching pools
that own all device memory, latency-critical loops. This test calls it
through the C ABI with device buffers it owns and checks two calls in a row
against the allocating entry point (vrs_knn_search), bit for bit. It runs
last (file name) so a failure here never hides other tests' results, and it
passes alone in a fresh process as well as after the rest of the suite.
"""
import ctypes

import numpy as np
import pytest

pytestmark = pytest.mark.gpu


def _noalloc(vc):
    L = vc.lib()
    f = L.vrs_knn_search_noalloc
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64,
                  ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                  ctypes.POINTER(ctypes.c_int32), ctypes.c_void_p]
    return f


def _check_pair(vc, fn, base, qs, k, metric):
    """Two calls in a row of the allocation-free entry point, each compared
    bit for bit with the allocating vrs_knn_search on the same rows."""
    import torch
    n, d = base.shape
    nq = qs.shape[0]
    eng = vc.DistributedKnnEngine.try_new(base, d, 1, vc.GpuShardMode.Sharded, vc.DistanceMetric(metric))
    d_ref, i_ref = eng.search_arrays(qs, k)
    eng.close()
    kk_ref = min(k, n)
    assert d_ref.shape == (nq, kk_ref)
    db = torch.from_numpy(base).cuda()
    dq = torch.from_numpy(qs).cuda()
    for _ in range(2):  # the shared scratch keeps the previous call's contents
        od = torch.full((nq, kk_ref), float("nan"), dtype=torch.float32, device="cuda")
        oi = torch.full((nq, kk_ref), -1, dtype=torch.int32, device="cuda")
        kk = ctypes.c_int32(0)
        st = fn(db.data_ptr(), n, d, dq.data_ptr(), nq, k, metric, od.data_ptr(), oi.data_ptr(),
                ctypes.byref(kk), None)
        assert st == 0, vc.lib().vrs_last_error()
        torch.cuda.synchronize()
        assert kk.value == kk_ref
        assert np.array_equal(oi.cpu().numpy().view(np.uint32), i_ref)
        assert np.array_equal(od.cpu().numpy().view(np.uint32), d_ref.view(np.uint32))


# Every metric the entry point accepts: L2, dot (ranked by negated score),
# Manhattan, Minkowski (cube root), Chebyshev, Hamming, Mahalanobis, Jaccard.
@pytest.mark.parametrize("metric", [0, 1, 3, 4, 5, 6, 7, 8])
def test_noalloc_matches_allocating_search(vc, gpu, metric):
    n, d, nq, k = 6000, 96, 300, 50
    s = vc.config_seed(300 + metric)
    base = vc.gen_rows_host(vc.GEN_NORMAL, s, 0, 0, n, d)
    qs = vc.gen_rows_host(vc.GEN_NORMAL, s, 1, 0, nq, d)
    _check_pair(vc, _noalloc(vc), base, qs, k, metric)


def test_noalloc_k_above_n(vc, gpu):
    # k' = min(k, n): 100 neighbours asked of a 60-row base.
    s = vc.config_seed(320)
    base = vc.gen_rows_host(vc.GEN_NORMAL, s, 0, 0, 60, 24)
    qs = vc.gen_rows_host(vc.GEN_NORMAL, s, 1, 0, 40, 24)
    _check_pair(vc, _noalloc(vc), base, qs, 100, 0)


def test_noalloc_largest_batch_at_k_2048(vc, gpu):
    # At k' = 2048 a list holds 8192 candidates: the 8 MiB scratch takes 127
    # queries in one segment, the largest batch it accepts at that k.
    s = vc.config_seed(321)
    base = vc.gen_rows_host(vc.GEN_NORMAL, s, 0, 0, 5000, 16)
    qs = vc.gen_rows_host(vc.GEN_NORMAL, s, 1, 0, 127, 16)
    _check_pair(vc, _noalloc(vc), base, qs, 2048, 0)


def test_noalloc_rejects_oversized_batch(vc, gpu):
    # Every buffer is sized for the full request, so nothing would be read or
    # written out of bounds even if a batch were accepted.
    import torch
    fn = _noalloc(vc)
    n, d = 5000, 16
    db = torch.zeros((n, d), dtype=torch.float32, device="cuda")
    kk = ctypes.c_int32(0)
    for nq, k in ((3000, 100), (128, 2048)):  # 2043 and 127 queries fit at these k'
        dq = torch.zeros((nq, d), dtype=torch.float32, device="cuda")
        od = torch.zeros((nq, k), dtype=torch.float32, device="cuda")
        oi = torch.zeros((nq, k), dtype=torch.int32, device="cuda")
        st = fn(db.data_ptr(), n, d, dq.data_ptr(), nq, k, 0, od.data_ptr(), oi.data_ptr(), ctypes.byref(kk),
                None)
        assert st == 5 and b"no-alloc scratch" in vc.lib().vrs_last_error()
        assert kk.value == 0
    torch.cuda.synchronize()


def test_noalloc_rejects_huge_query_count_before_device_work(vc, gpu):
    # A query count whose scratch size would wrap 64-bit arithmetic is
    # refused by the first size check; the pointers are never touched.
    fn = _noalloc(vc)
    kk = ctypes.c_int32(0)
    for nq in (2 ** 61 + 300, 2 ** 62, 2 ** 63 - 1, 3000):
        st = fn(None, 1000, 16, None, nq, 100, 0, None, None, ctypes.byref(kk), None)
        assert st == 5 and b"no-alloc scratch" in vc.lib().vrs_last_error()
        assert kk.value == 0
