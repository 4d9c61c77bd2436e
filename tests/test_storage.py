"""VECRSTOR vector files (crates/vector-index/src/storage/mmap.rs:7-16).

CPU tests restate the reference's own MmapStorage tests (mmap.rs:276-430)
through libvrs's `vrs_vecrstor_info` / `vrs_vecrstor_write` and the Python
`MmapStorage` mirror, check the bytes against the format as the reference's
dataset writer packs it (scripts/generate_dataset.py:50-66: struct "<QQQ"
header, "<{d}f" rows), and reject headers no file could back. The GPU test
builds an engine straight from a file and checks it answers exactly as one
built from the same rows in memory.
"""
import struct

import numpy as np
import pytest

MAGIC = 0x56454352_53544F52


def _pack_reference_layout(vectors, dimension):
    """The byte layout generate_dataset.py:50-66 writes, restated."""
    out = struct.pack("<QQQ", MAGIC, len(vectors), dimension)
    return out + b"".join(struct.pack(f"<{dimension}f", *v) for v in vectors)


def test_create_and_open_round_trip(vc, tmp_path):
    p = tmp_path / "test_vectors.bin"
    vs = [[1.0, 2.0, 3.0, 4.0], [5.0, 6.0, 7.0, 8.0], [9.0, 10.0, 11.0, 12.0]]
    vc.MmapStorage.create(p, 4, vs)
    s = vc.MmapStorage.open(p)
    assert s.dimension() == 4 and s.len() == 3 and not s.is_empty()
    for i, v in enumerate(vs):
        assert list(s.get(i)) == v
    assert p.read_bytes() == _pack_reference_layout(vs, 4)


def test_create_from_flat_round_trip(vc, tmp_path):
    p = tmp_path / "flat_vectors.bin"
    flat = np.arange(12, dtype=np.float32) * 1.5
    vc.MmapStorage.create_from_flat(p, 3, flat)
    s = vc.MmapStorage.open(p)
    assert (s.len(), s.dimension()) == (4, 3)
    assert np.array_equal(s.as_raw_slice(), flat)
    with pytest.raises(ValueError):
        vc.MmapStorage.create_from_flat(tmp_path / "bad.bin", 5, flat)


def test_empty_storage(vc, tmp_path):
    p = tmp_path / "empty.bin"
    vc.MmapStorage.create(p, 128, [])
    s = vc.MmapStorage.open(p)
    assert s.len() == 0 and s.is_empty() and s.dimension() == 128
    assert s.as_raw_slice().size == 0


def test_invalid_magic(vc, tmp_path):
    p = tmp_path / "bad_magic.bin"
    p.write_bytes(bytes(24))
    with pytest.raises(vc.CudaError) as e:
        vc.MmapStorage.open(p)
    assert e.value.status == 9 and "invalid magic number" in str(e.value)


def test_truncated_file(vc, tmp_path):
    p = tmp_path / "truncated.bin"
    p.write_bytes(struct.pack("<QQQ", MAGIC, 10, 4))  # 160 bytes of rows missing
    with pytest.raises(vc.CudaError) as e:
        vc.MmapStorage.open(p)
    assert e.value.status == 9 and "size mismatch" in str(e.value)


def test_trailing_bytes_accepted(vc, tmp_path):
    # mmap.rs:202-211 only rejects files shorter than header + rows
    p = tmp_path / "trailing.bin"
    p.write_bytes(_pack_reference_layout([[1.0, 2.0]], 2) + b"\x00" * 7)
    s = vc.MmapStorage.open(p)
    assert s.len() == 1 and list(s.get(0)) == [1.0, 2.0]


def test_header_overflow_rejected(vc, tmp_path):
    # N*D*4 beyond 2^64: no file can hold it; must not wrap to a small size
    p = tmp_path / "overflow.bin"
    p.write_bytes(struct.pack("<QQQ", MAGIC, 2 ** 62, 2 ** 4) + bytes(64))
    with pytest.raises(vc.CudaError) as e:
        vc.MmapStorage.open(p)
    assert e.value.status == 9


def test_dimension_mismatch_on_create(vc, tmp_path):
    with pytest.raises(ValueError):
        vc.MmapStorage.create(tmp_path / "mismatch.bin", 3, [[1.0, 2.0, 3.0], [4.0, 5.0]])


def test_high_dimensional_round_trip(vc, tmp_path):
    p = tmp_path / "high_dim.bin"
    dim = 1536
    v1 = (np.arange(dim) * np.float32(0.001)).astype(np.float32)
    v2 = ((dim - np.arange(dim)) * np.float32(0.001)).astype(np.float32)
    vc.MmapStorage.create(p, dim, [v1, v2])
    s = vc.MmapStorage.open(p)
    assert (s.dimension(), s.len()) == (dim, 2)
    assert np.array_equal(s.get(0), v1) and np.array_equal(s.get(1), v2)


def test_get_out_of_bounds(vc, tmp_path):
    p = tmp_path / "oob.bin"
    vc.MmapStorage.create(p, 2, [[1.0, 2.0]])
    with pytest.raises(IndexError, match="out of bounds"):
        vc.MmapStorage.open(p).get(1)


def test_file_too_small(vc, tmp_path):
    p = tmp_path / "tiny.bin"
    p.write_bytes(bytes(10))
    with pytest.raises(vc.CudaError) as e:
        vc.MmapStorage.open(p)
    assert e.value.status == 9 and "too small" in str(e.value)


def test_missing_file(vc, tmp_path):
    with pytest.raises(vc.CudaError) as e:
        vc.MmapStorage.open(tmp_path / "nope.bin")
    assert e.value.status == 9


def test_engine_from_bad_file_fails_before_the_gpu(vc, tmp_path):
    # File problems surface as InvalidFile (status 9), a zero dimension as
    # InvalidConfig (status 5), both before any device work.
    M, Sm = vc.DistanceMetric.L2Squared, vc.GpuShardMode.Sharded
    with pytest.raises(vc.CudaError) as e:
        vc.DistributedKnnEngine.from_file(tmp_path / "missing.bin", 1, Sm, M)
    assert e.value.status == 9
    bad = tmp_path / "short.bin"
    bad.write_bytes(struct.pack("<QQQ", MAGIC, 3, 4) + bytes(8))
    with pytest.raises(vc.CudaError) as e:
        vc.DistributedKnnEngine.from_file(bad, 1, Sm, M)
    assert e.value.status == 9 and "size mismatch" in str(e.value)
    zero = tmp_path / "zero_dim.bin"
    zero.write_bytes(struct.pack("<QQQ", MAGIC, 5, 0))
    assert vc.MmapStorage.open(zero).len() == 5  # valid storage, empty rows
    with pytest.raises(vc.CudaError) as e:
        vc.DistributedKnnEngine.from_file(zero, 1, Sm, M)
    assert e.value.status == 5


@pytest.mark.gpu
@pytest.mark.parametrize("metric,mode,g", [(0, 0, 1), (2, 0, 1), (3, 1, 1), (0, 0, 2)])
def test_engine_from_file_matches_memory(vc, gpu, tmp_path, metric, mode, g):
    if g > gpu:
        pytest.skip(f"needs {g} GPUs")
    kind = vc.GEN_UNIFORM if metric == 3 else vc.GEN_NORMAL
    base = vc.gen_rows_host(kind, vc.config_seed(500 + metric), 0, 0, 20_000, 72)
    qs = vc.gen_rows_host(kind, vc.config_seed(500 + metric), 1, 0, 64, 72)
    p = tmp_path / "base.bin"
    vc.MmapStorage.create_from_flat(p, 72, base)
    M, Sm = vc.DistanceMetric(metric), vc.GpuShardMode(mode)
    ef = vc.DistributedKnnEngine.from_file(p, g, Sm, M)
    em = vc.DistributedKnnEngine.try_new(base, 72, g, Sm, M)
    assert (ef.num_vectors(), ef.dimension(), ef.num_gpus()) == (20_000, 72, g)
    df, i_f = ef.search_arrays(qs, 25)
    dm, im = em.search_arrays(qs, 25)
    assert np.array_equal(i_f, im) and np.array_equal(df.view(np.uint32), dm.view(np.uint32))
    ef.close()
    em.close()
    # An empty file gives an empty engine, as an empty storage does.
    e = tmp_path / "empty.bin"
    vc.MmapStorage.create(e, 8, [])
    ee = vc.DistributedKnnEngine.from_file(e, 1, vc.GpuShardMode.Sharded, M)
    assert ee.num_vectors() == 0 and ee.search(np.zeros(8, np.float32), 5) == []
    ee.close()


# ------------------------------------------------------------ centroid files
# IvfPqSerializer::save_centroid_file / load_centroid_file
# (crates/vector-index/src/ivf/serializer.rs:255-370), tests after
# serializer.rs:552-615.

def _pack_centroid_layout(centroids, d, k, metric, iters, inertia):
    """The packed header the reference writes field by field (serializer.rs:285-302)."""
    hdr = struct.pack("<QIBIIIf", 0x5652_534B_4D45_414E, 1, metric, d, k, iters, inertia)
    return hdr + struct.pack(f"<{len(centroids)}f", *centroids)


def test_centroid_file_roundtrip(vc, tmp_path):
    p = tmp_path / "c.bin"
    c = [1.0, 2.0, 3.0, 4.0, 5.0, 6.0, 7.0, 8.0]
    vc.IvfPqSerializer.save_centroid_file(p, c, 4, 2, vc.DistanceMetric.L2Squared, 15, 42.5)
    assert p.read_bytes() == _pack_centroid_layout(c, 4, 2, 0, 15, 42.5)
    assert len(p.read_bytes()) == 29 + 32
    ld = vc.IvfPqSerializer.load_centroid_file(p)
    assert list(ld.centroids.ravel()) == c
    assert (ld.dimension, ld.k, ld.metric, ld.iterations) == (4, 2, vc.DistanceMetric.L2Squared, 15)
    assert abs(ld.inertia - 42.5) < 1e-6


def test_centroid_file_all_metrics(vc, tmp_path):
    p = tmp_path / "m.bin"
    for m in vc.DistanceMetric:
        vc.IvfPqSerializer.save_centroid_file(p, [1.0, 2.0], 2, 1, m, 1, 0.0)
        assert vc.IvfPqSerializer.load_centroid_file(p).metric == m


def test_centroid_file_invalid_magic(vc, tmp_path):
    p = tmp_path / "bad.bin"
    p.write_bytes(b"NOTCENTR12345678")
    with pytest.raises(vc.CudaError) as e:
        vc.IvfPqSerializer.load_centroid_file(p)
    assert e.value.status == 9 and "expected centroid magic" in str(e.value)


def test_centroid_file_bad_version_metric_and_truncation(vc, tmp_path):
    good = _pack_centroid_layout([1.0, 2.0, 3.0, 4.0], 2, 2, 3, 7, 1.25)
    p = tmp_path / "v.bin"
    p.write_bytes(good[:8] + struct.pack("<I", 2) + good[12:])
    with pytest.raises(vc.CudaError, match="unsupported centroid file version: 2"):
        vc.IvfPqSerializer.load_centroid_file(p)
    p.write_bytes(good[:12] + bytes([10]) + good[13:])
    with pytest.raises(vc.CudaError, match="invalid metric code: 10"):
        vc.IvfPqSerializer.load_centroid_file(p)
    for cut in (5, 20, 29 + 6):
        p.write_bytes(good[:cut])
        with pytest.raises(vc.CudaError) as e:
            vc.IvfPqSerializer.load_centroid_file(p)
        assert e.value.status == 9
    p.write_bytes(good)
    ld = vc.IvfPqSerializer.load_centroid_file(p)
    assert ld.metric == vc.DistanceMetric.Manhattan and ld.centroids.shape == (2, 2)


def test_centroid_file_empty_and_size_check(vc, tmp_path):
    p = tmp_path / "e.bin"
    vc.IvfPqSerializer.save_centroid_file(p, [], 16, 0, vc.DistanceMetric.CosineSimilarity, 0, 0.0)
    ld = vc.IvfPqSerializer.load_centroid_file(p)
    assert ld.k == 0 and ld.dimension == 16 and ld.centroids.shape == (0, 16)
    with pytest.raises(ValueError):
        vc.IvfPqSerializer.save_centroid_file(p, [1.0, 2.0, 3.0], 2, 2, vc.DistanceMetric.L2Squared, 1, 0.0)
