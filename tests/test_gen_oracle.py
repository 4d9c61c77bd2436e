"""CPU tests: the oracle's own generator (oracle/orc_gen.c) gives the same
bits as the product's (vrs_gen_rows_host), so the reference arm of the bench
consumes identical inputs without loading libvrs; and the row-split oracle
search equals the query-split one."""
import numpy as np
import pytest


def test_seed_matches(vc, orc):
    for i in range(6):
        assert orc.config_seed(i) == vc.config_seed(i)


@pytest.mark.parametrize("kind,d", [(0, 128), (1, 128), (2, 96), (3, 96), (0, 13), (1, 7)])
def test_oracle_generator_bits(vc, orc, kind, d):
    s = vc.config_seed(kind + 1)
    for stream, row0, rows in ((0, 0, 700), (1, 123456, 300), (5, 10 ** 8 - 50, 50)):
        a = vc.gen_rows_host(kind, s, stream, row0, rows, d)
        b = orc.gen_rows(kind, s, stream, row0, rows, d, nthreads=4)
        assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_oracle_generator_mixture_bits(vc, orc):
    s = vc.config_seed(2)
    c = vc.gen_rows_host(vc.GEN_NORMAL, s, 2, 0, 1024, 128)
    assert np.array_equal(c, orc.gen_rows(orc.GEN_NORMAL, s, 2, 0, 1024, 128))
    a = vc.gen_rows_host(vc.GEN_MIXTURE, s, 0, 5000, 2000, 128, c, 1024, 0.1)
    b = orc.gen_rows(orc.GEN_MIXTURE, s, 0, 5000, 2000, 128, c, 1024, 0.1, nthreads=3)
    assert np.array_equal(a.view(np.uint32), b.view(np.uint32))


def test_oracle_generator_rejects_bad_arguments(orc):
    with pytest.raises(ValueError):
        orc.gen_rows(7, 1, 0, 0, 4, 4)
    with pytest.raises(ValueError):
        orc.gen_rows(orc.GEN_MIXTURE, 1, 0, 0, 4, 4)  # no centres


@pytest.mark.parametrize("metric", [0, 1, 2, 3, 5, 6, 9])
def test_row_split_search_equals_query_split(orc, metric):
    rng = np.random.default_rng(metric)
    base = rng.standard_normal((5000, 33)).astype(np.float32)
    if metric == 9:
        base = np.abs(base)
    base[1000:1100] = base[0]  # exact ties across thread row ranges
    q = np.vstack([base[:3], rng.standard_normal((9, 33)).astype(np.float32)])
    if metric == 9:
        q = np.abs(q)
    for k in (1, 10, 150):
        d1, i1 = orc.knn_search(base, q, k, metric, nthreads=4)
        d2, i2 = orc.knn_search_rows(base, q, k, metric, nthreads=7)
        assert np.array_equal(i1, i2)
        assert np.array_equal(d1.view(np.uint32), d2.view(np.uint32))


def test_row_split_search_chunks_merge(orc):
    # A base fed in chunks with id offsets, merged per query, equals the
    # whole-base search (the bench's large parity samples work this way).
    rng = np.random.default_rng(7)
    base = rng.standard_normal((9000, 24)).astype(np.float32)
    q = rng.standard_normal((5, 24)).astype(np.float32)
    d_all, i_all = orc.knn_search(base, q, 20, 0, nthreads=4)
    parts = [orc.knn_search_rows(base[r:r + 2500], q, 20, 0, nthreads=3, id_offset=r)
             for r in range(0, 9000, 2500)]
    for qi in range(5):
        dm, im = orc.topk_reduce([(p[0][qi], p[1][qi]) for p in parts], 20, 0)
        assert np.array_equal(im, i_all[qi]) and np.array_equal(dm, d_all[qi])
