"""CPU tests of the C ABI: the library loads, exports every function that
include/vrs.h declares, and reports errors the way CudaError does
(crates/vector-cuda/src/error.rs:7-29) without needing a GPU."""
import ctypes
import os
import re
import subprocess

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    src = open(os.path.join(ROOT, "include", "vrs.h")).read()
    return sorted(set(re.findall(r"VRS_API\s+[\w\s\*]+?\b(vrs_\w+)\s*\(", src)))


def test_header_declares_api():
    names = _declared()
    for n in ["vrs_knn_create", "vrs_knn_search", "vrs_knn_destroy", "vrs_kmeans_fit",
              "vrs_device_count", "vrs_last_error", "vrs_comm_init", "vrs_knn_create_rank",
              "vrs_kmeans_fit_rank", "vrs_gen_rows_host", "vrs_gen_rows_device"]:
        assert n in names


def test_library_exports_every_declared_symbol(vc):
    out = subprocess.run(["nm", "-D", "--defined-only", vc.LIB_PATH], capture_output=True,
                         text=True, check=True).stdout
    exported = set(re.findall(r" T (vrs_\w+)", out))
    missing = [n for n in _declared() if n not in exported]
    assert not missing, missing
    L = ctypes.CDLL(vc.LIB_PATH)
    for n in _declared():
        assert getattr(L, n) is not None


def test_device_count_and_errors_without_gpu(vc):
    n = vc.CudaDeviceContext.device_count()
    assert n >= 0
    req = n + 100
    with pytest.raises(vc.CudaError) as e:
        vc.DistributedKnnEngine.try_new(np.zeros(8, np.float32), 2, req, vc.GpuShardMode.Sharded,
                                        vc.DistanceMetric.L2Squared)
    assert e.value.kind == "InsufficientDevices"
    assert e.value.requested == req and e.value.available == n
    with pytest.raises(vc.CudaError) as e:
        vc.DistributedKMeansEngine.try_new(req)
    assert e.value == vc.CudaError(1, "", requested=req, available=n)


def test_invalid_config_rejected(vc):
    L = vc.lib()
    h = ctypes.c_void_p()
    # bad metric code
    st = L.vrs_knn_create(None, 0, 4, 1, 0, 42, ctypes.byref(h))
    assert st in (1, 5)
    assert L.vrs_last_error()
    # null out_k
    assert L.vrs_knn_search(None, None, 0, 1, None, None, None) == 5


def test_metric_higher_is_better(vc):
    L = vc.lib()
    assert [L.vrs_metric_higher_is_better(m) for m in range(10)] == [0, 1, 1, 0, 0, 0, 0, 0, 0, 0]
    assert [vc.DistanceMetric(m).higher_is_better() for m in range(10)] == \
        [False, True, True] + [False] * 7


def test_noalloc_refuses_huge_query_count_on_cpu(vc):
    # The allocation-free entry point refuses a query count that no scratch
    # layout can hold before any size arithmetic or CUDA call, so this runs
    # without a GPU (and a count that would wrap 64-bit sizes is refused too).
    f = vc.lib().vrs_knn_search_noalloc
    f.argtypes = [ctypes.c_void_p, ctypes.c_int64, ctypes.c_int32, ctypes.c_void_p, ctypes.c_int64,
                  ctypes.c_int32, ctypes.c_int32, ctypes.c_void_p, ctypes.c_void_p,
                  ctypes.POINTER(ctypes.c_int32), ctypes.c_void_p]
    kk = ctypes.c_int32(7)
    for nq in (2 ** 61 + 300, 2 ** 63 - 1, 2044):
        assert f(None, 1000, 16, None, nq, 100, 0, None, None, ctypes.byref(kk), None) == 5
        assert b"no-alloc scratch" in vc.lib().vrs_last_error()
        assert kk.value == 0


def test_ivfpq_create_rejects_bad_index_on_cpu(vc):
    # Argument checks run before any device work.
    L = vc.lib()
    h = ctypes.c_void_p()
    cc = np.zeros(8, np.float32)
    cb = np.zeros(64, np.float32)
    off = np.array([0, 2], np.int64)
    ids = np.array([1, 2], np.uint32)
    codes = np.array([[0, 1], [1, 0]], np.uint8)
    P = lambda a: a.ctypes.data  # noqa: E731
    # d not a multiple of num_subvectors
    assert L.vrs_ivfpq_create(P(cc), 1, 7, P(cb), 2, 2, P(off), P(ids), P(codes), 0, ctypes.byref(h)) == 5
    # more than 256 sub-centroids (u8 codes)
    assert L.vrs_ivfpq_create(P(cc), 1, 8, P(cb), 2, 257, P(off), P(ids), P(codes), 0, ctypes.byref(h)) == 5
    # decreasing offsets
    bad_off = np.array([0, -1], np.int64)
    assert L.vrs_ivfpq_create(P(cc), 1, 8, P(cb), 2, 2, P(bad_off), P(ids), P(codes), 0, ctypes.byref(h)) == 5
    # a code not below sub_clusters
    bad_codes = np.array([[0, 2], [1, 0]], np.uint8)
    assert L.vrs_ivfpq_create(P(cc), 1, 8, P(cb), 2, 2, P(off), P(ids), P(bad_codes), 0, ctypes.byref(h)) == 5
    assert b"sub_clusters" in L.vrs_last_error()
    assert not h.value
