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


@pytest.mark.parametrize("metric", [0, 3, 5, 7])
def test_noalloc_matches_allocating_search(vc, gpu, metric):
    import torch
    n, d, nq, k = 6000, 96, 300, 50
    s = vc.config_seed(300 + metric)
    base = vc.gen_rows_host(vc.GEN_NORMAL, s, 0, 0, n, d)
    qs = vc.gen_rows_host(vc.GEN_NORMAL, s, 1, 0, nq, d)
    eng = vc.DistributedKnnEngine.try_new(base, d, 1, vc.GpuShardMode.Sharded, vc.DistanceMetric(metric))
    d_ref, i_ref = eng.search_arrays(qs, k)
    eng.close()
    fn = _noalloc(vc)
    db = torch.from_numpy(base).cuda()
    dq = torch.from_numpy(qs).cuda()
    for _ in range(2):  # the shared scratch keeps the previous call's contents
        od = torch.full((nq, k), float("nan"), dtype=torch.float32, device="cuda")
        oi = torch.full((nq, k), -1, dtype=torch.int32, device="cuda")
        kk = ctypes.c_int32(0)
        st = fn(db.data_ptr(), n, d, dq.data_ptr(), nq, k, metric, od.data_ptr(), oi.data_ptr(),
                ctypes.byref(kk), None)
        assert st == 0, vc.lib().vrs_last_error()
        torch.cuda.synchronize()
        assert kk.value == k
        assert np.array_equal(oi.cpu().numpy().view(np.uint32), i_ref)
        assert np.array_equal(od.cpu().numpy().view(np.uint32), d_ref.view(np.uint32))


def test_noalloc_rejects_oversized_batch(vc, gpu):
    import torch
    fn = _noalloc(vc)
    n, d, nq, k = 1000, 16, 200000, 100
    db = torch.zeros((n, d), dtype=torch.float32, device="cuda")
    dq = torch.zeros((8, d), dtype=torch.float32, device="cuda")
    kk = ctypes.c_int32(0)
    st = fn(db.data_ptr(), n, d, dq.data_ptr(), nq, k, 0, dq.data_ptr(), dq.data_ptr(), ctypes.byref(kk), None)
    assert st == 5 and b"no-alloc scratch" in vc.lib().vrs_last_error()
