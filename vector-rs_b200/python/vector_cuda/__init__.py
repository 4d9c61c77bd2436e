"""vector_cuda -- Python mirror of VectorRS's ``vector-cuda`` crate API over libvrs.

Names, argument meaning and error behaviour follow the Rust crate
(crates/vector-cuda/src/lib.rs:20-26): ``DistributedKnnEngine.try_new``,
``GpuShardMode``, ``CudaKnnEngine``, ``CudaKMeansEngine``,
``DistributedKMeansEngine``, ``DistanceMetric``, ``SearchResult``,
``CudaError``. Every call goes through the C ABI in include/vrs.h; there is
no CPU fallback -- a missing library or GPU raises.
"""
from __future__ import annotations

import ctypes
import enum
import importlib.util
import os
from dataclasses import dataclass, field
from typing import List, Optional, Sequence, Tuple

import numpy as np

_PKG_ROOT = os.path.dirname(os.path.dirname(os.path.dirname(os.path.abspath(__file__))))
LIB_PATH = os.path.join(_PKG_ROOT, "lib", "libvrs.so")

# ----------------------------------------------------------------- enums


class DistanceMetric(enum.IntEnum):
    """crates/vector-index/src/lib.rs:49-83; codes = knn.rs:235-246."""

    L2Squared = 0
    DotProduct = 1
    CosineSimilarity = 2
    Manhattan = 3
    Minkowski = 4
    Chebyshev = 5
    Hamming = 6
    Mahalanobis = 7
    Jaccard = 8
    Hellinger = 9

    def higher_is_better(self) -> bool:
        """crates/vector-index/src/lib.rs:85-94."""
        return self in (DistanceMetric.DotProduct, DistanceMetric.CosineSimilarity)


class GpuShardMode(enum.IntEnum):
    """crates/vector-cuda/src/ddp/distributed_knn.rs:14-19."""

    Sharded = 0
    Replicated = 1


# ----------------------------------------------------------------- errors

VRS_OK = 0
_STATUS_NAMES = {
    1: "InsufficientDevices",
    2: "DeviceNotFound",
    3: "DriverError",
    4: "HardwareNotAvailable",
    5: "InvalidConfig",
    6: "NcclError",
    7: "Timeout",
    8: "OutOfMemory",
    9: "InvalidFile",
}


class CudaError(Exception):
    """Mirrors CudaError (crates/vector-cuda/src/error.rs:7-29) plus the
    NCCL / timeout / OOM statuses of the C ABI."""

    def __init__(self, status: int, message: str, **fields):
        self.status = status
        self.kind = _STATUS_NAMES.get(status, f"Status{status}")
        self.message = message
        self.fields = fields
        super().__init__(f"{self.kind}: {message}")

    @property
    def requested(self):
        return self.fields.get("requested")

    @property
    def available(self):
        return self.fields.get("available")

    def __eq__(self, other):
        return (isinstance(other, CudaError) and self.status == other.status
                and self.fields == other.fields)

    def __hash__(self):
        return hash((self.status, tuple(sorted(self.fields.items()))))


# ------------------------------------------------------------- library

_lib_handle = None


def _preload_nccl():
    """Use the NCCL that torch ships, when present, so a process that also
    imports torch loads one NCCL only."""
    try:
        spec = importlib.util.find_spec("nvidia.nccl")
    except (ImportError, ValueError):
        spec = None
    if spec and spec.submodule_search_locations:
        p = os.path.join(list(spec.submodule_search_locations)[0], "lib", "libnccl.so.2")
        if os.path.exists(p):
            ctypes.CDLL(p, mode=ctypes.RTLD_GLOBAL)


def lib() -> ctypes.CDLL:
    global _lib_handle
    if _lib_handle is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(
                f"libvrs.so not found at {LIB_PATH}; build it with "
                "`python vector-rs_b200/build.py` (there is no CPU fallback)")
        _preload_nccl()
        L = ctypes.CDLL(LIB_PATH)
        c = ctypes
        P = c.POINTER
        L.vrs_last_error.restype = c.c_char_p
        L.vrs_device_count.argtypes = [P(c.c_int32)]
        L.vrs_metric_higher_is_better.argtypes = [c.c_int32]
        L.vrs_knn_create.argtypes = [c.c_void_p, c.c_int64, c.c_int32, c.c_int32, c.c_int32,
                                     c.c_int32, P(c.c_void_p)]
        L.vrs_knn_search.argtypes = [c.c_void_p, c.c_void_p, c.c_int64, c.c_int32, c.c_void_p,
                                     c.c_void_p, P(c.c_int32)]
        L.vrs_knn_search_ex.argtypes = [c.c_void_p, c.c_void_p, c.c_int64, c.c_int32, c.c_void_p,
                                        c.c_void_p, P(c.c_int32), c.c_int32]
        L.vrs_knn_info.argtypes = [c.c_void_p, P(c.c_int64), P(c.c_int32), P(c.c_int32),
                                   P(c.c_int32), P(c.c_int32)]
        L.vrs_knn_destroy.argtypes = [c.c_void_p]
        L.vrs_knn_destroy.restype = None
        L.vrs_kmeans_fit.argtypes = [c.c_void_p, c.c_int64, c.c_int32, c.c_int32, c.c_void_p,
                                     c.c_int32, c.c_float, c.c_int32, c.c_int32, c.c_void_p,
                                     c.c_void_p, P(c.c_int32), P(c.c_int32), P(c.c_double)]
        L.vrs_comm_unique_id.argtypes = [c.c_void_p]
        L.vrs_comm_init.argtypes = [c.c_void_p, c.c_int32, c.c_int32, c.c_int32, P(c.c_void_p)]
        L.vrs_comm_destroy.argtypes = [c.c_void_p]
        L.vrs_comm_destroy.restype = None
        L.vrs_knn_create_rank.argtypes = [c.c_void_p, c.c_void_p, c.c_int64, c.c_int64, c.c_int64,
                                          c.c_int32, c.c_int32, c.c_int32, c.c_int32, P(c.c_void_p)]
        L.vrs_kmeans_fit_rank.argtypes = [c.c_void_p, c.c_void_p, c.c_int64, c.c_int64, c.c_int32,
                                          c.c_int32, c.c_void_p, c.c_int32, c.c_float, c.c_int32,
                                          c.c_int32, c.c_void_p, c.c_void_p, P(c.c_int32),
                                          P(c.c_int32), P(c.c_double)]
        L.vrs_ivf_find_top_centroids.argtypes = [c.c_void_p, c.c_void_p, c.c_int64, c.c_int32,
                                                 c.c_void_p, c.c_void_p, P(c.c_int32)]
        L.vrs_ivf_assign.argtypes = [c.c_void_p, c.c_void_p, c.c_int64, c.c_void_p, c.c_void_p]
        L.vrs_vecrstor_info.argtypes = [c.c_char_p, P(c.c_int64), P(c.c_int64)]
        L.vrs_vecrstor_write.argtypes = [c.c_char_p, c.c_void_p, c.c_int64, c.c_int64]
        L.vrs_knn_create_from_file.argtypes = [c.c_char_p, c.c_int32, c.c_int32, c.c_int32,
                                               P(c.c_void_p)]
        L.vrs_centroid_file_write.argtypes = [c.c_char_p, c.c_void_p, c.c_int64, c.c_int64,
                                              c.c_int32, c.c_int64, c.c_float]
        L.vrs_centroid_file_read.argtypes = [c.c_char_p, c.c_void_p, c.c_int64, P(c.c_int32),
                                             P(c.c_int64), P(c.c_int64), P(c.c_int64),
                                             P(c.c_float)]
        L.vrs_knn_set_stream.argtypes = [c.c_void_p, c.c_void_p]
        L.vrs_profile_enable.argtypes = [c.c_int32]
        L.vrs_profile_read.argtypes = [c.c_char_p, P(c.c_double), P(c.c_int64)]
        L.vrs_gen_rows_host.argtypes = [c.c_int32, c.c_uint64, c.c_uint32, c.c_int64, c.c_int64,
                                        c.c_int32, c.c_int64, c.c_void_p, c.c_void_p, c.c_uint32,
                                        c.c_double]
        L.vrs_gen_rows_device.argtypes = [c.c_int32, c.c_uint64, c.c_uint32, c.c_int64, c.c_int64,
                                          c.c_int32, c.c_int64, c.c_void_p, c.c_void_p, c.c_uint32,
                                          c.c_double, c.c_void_p]
        L.vrs_selftest_bounded_wait.argtypes = [c.c_int64]
        L.vrs_ivfpq_create.argtypes = [c.c_void_p, c.c_int64, c.c_int32, c.c_void_p, c.c_int32, c.c_int32,
                                       c.c_void_p, c.c_void_p, c.c_void_p, c.c_int32, P(c.c_void_p)]
        L.vrs_ivfpq_search.argtypes = [c.c_void_p, c.c_void_p, c.c_int64, c.c_int32, c.c_int32, c.c_void_p,
                                       c.c_void_p, c.c_void_p]
        L.vrs_ivfpq_destroy.argtypes = [c.c_void_p]
        L.vrs_ivfpq_destroy.restype = None
        _lib_handle = L
    return _lib_handle


def _check(status: int, **fields):
    if status != VRS_OK:
        msg = lib().vrs_last_error().decode(errors="replace")
        raise CudaError(status, msg, **fields)


def _f32(a) -> np.ndarray:
    return np.ascontiguousarray(np.asarray(a, dtype=np.float32))


def _ptr(a: Optional[np.ndarray]):
    return None if a is None else a.ctypes.data


# ------------------------------------------------------------- results


@dataclass
class SearchResult:
    """crates/vector-index/src/types.rs:13-28."""

    id: int
    distance: float


class CudaDeviceContext:
    """Device queries of crates/vector-cuda/src/device.rs:110-118."""

    @staticmethod
    def device_count() -> int:
        n = ctypes.c_int32(0)
        _check(lib().vrs_device_count(ctypes.byref(n)))
        return int(n.value)


# ----------------------------------------------------------------- kNN


class DistributedKnnEngine:
    """crates/vector-cuda/src/ddp/distributed_knn.rs:26-261 over vrs_knn_*."""

    def __init__(self, handle, dimension: int):
        self._h = handle
        self._dim = dimension

    @classmethod
    def try_new(cls, dataset, dimension: int, num_gpus: int, mode: GpuShardMode,
                metric: DistanceMetric) -> "DistributedKnnEngine":
        if num_gpus < 1:
            raise ValueError("num_gpus must be at least 1")
        data = _f32(dataset).reshape(-1)
        if dimension < 1 or data.size % dimension:
            raise ValueError("dataset length must be a multiple of dimension")
        n = data.size // dimension
        h = ctypes.c_void_p()
        st = lib().vrs_knn_create(_ptr(data), n, dimension, num_gpus, int(mode), int(metric),
                                  ctypes.byref(h))
        fields = {}
        if st == 1:
            fields = {"requested": num_gpus, "available": CudaDeviceContext.device_count()}
        _check(st, **fields)
        return cls(h, dimension)

    new = try_new

    @classmethod
    def from_file(cls, path, num_gpus: int, mode: GpuShardMode,
                  metric: DistanceMetric) -> "DistributedKnnEngine":
        """try_new over an MmapStorage's rows (crates/vector-index/src/storage/mmap.rs):
        the VECRSTOR file is validated, mapped and uploaded shard by shard
        with no host copy of the base."""
        if num_gpus < 1:
            raise ValueError("num_gpus must be at least 1")
        h = ctypes.c_void_p()
        st = lib().vrs_knn_create_from_file(os.fsencode(path), num_gpus, int(mode), int(metric),
                                            ctypes.byref(h))
        fields = {}
        if st == 1:
            fields = {"requested": num_gpus, "available": CudaDeviceContext.device_count()}
        _check(st, **fields)
        d = ctypes.c_int32(0)
        _check(lib().vrs_knn_info(h, None, ctypes.byref(d), None, None, None))
        return cls(h, d.value)

    @classmethod
    def create_rank(cls, comm: "Comm", shard, dimension: int, global_offset: int, n_global: int,
                    mode: GpuShardMode, metric: DistanceMetric,
                    device_ptr: Optional[int] = None, n_local: Optional[int] = None):
        """Rank-mode engine (one process per GPU). `shard` is a host array, or
        pass device_ptr/n_local for rows already resident on this rank's GPU."""
        h = ctypes.c_void_p()
        if device_ptr is not None:
            st = lib().vrs_knn_create_rank(comm._c, ctypes.c_void_p(device_ptr), int(n_local),
                                           global_offset, n_global, dimension, int(mode),
                                           int(metric), 1, ctypes.byref(h))
        else:
            data = _f32(shard).reshape(-1)
            st = lib().vrs_knn_create_rank(comm._c, _ptr(data), data.size // dimension,
                                           global_offset, n_global, dimension, int(mode),
                                           int(metric), 0, ctypes.byref(h))
        _check(st)
        return cls(h, dimension)

    def close(self):
        if self._h:
            lib().vrs_knn_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def search_arrays(self, queries, k: int):
        """Fast path: returns (dist[nq, k'], ids[nq, k']) as numpy arrays."""
        q = _f32(queries).reshape(-1)
        if q.size % self._dim:
            raise ValueError("queries length must be a multiple of dimension")
        nq = q.size // self._dim
        cap = max(nq * max(k, 0), 1)
        dist = np.empty(cap, np.float32)
        ids = np.empty(cap, np.uint32)
        kk = ctypes.c_int32(0)
        _check(lib().vrs_knn_search(self._h, _ptr(q), nq, int(k), _ptr(dist), _ptr(ids),
                                    ctypes.byref(kk)))
        kk = kk.value
        return dist[:nq * kk].reshape(nq, kk), ids[:nq * kk].reshape(nq, kk)

    def search_root(self, queries, k: int, nq: Optional[int] = None):
        """Rank mode, root I/O (VRS_MEM_ROOT): rank 0 passes the queries and
        receives (dist[nq, k'], ids[nq, k']); every other rank passes None
        with the same nq and receives None. The queries reach the other
        ranks by NCCL broadcast and only rank 0's buffers are written."""
        kk = ctypes.c_int32(0)
        if queries is not None:
            q = _f32(queries).reshape(-1)
            nq = q.size // self._dim
            cap = max(nq * max(k, 0), 1)
            dist = np.empty(cap, np.float32)
            ids = np.empty(cap, np.uint32)
            _check(lib().vrs_knn_search_ex(self._h, _ptr(q), nq, int(k), _ptr(dist), _ptr(ids),
                                           ctypes.byref(kk), MEM_ROOT))
            kk = kk.value
            return dist[:nq * kk].reshape(nq, kk), ids[:nq * kk].reshape(nq, kk)
        _check(lib().vrs_knn_search_ex(self._h, None, int(nq), int(k), None, None, ctypes.byref(kk), MEM_ROOT))
        return None

    def search_device(self, q_ptr: int, nq: int, k: int, dist_ptr: int, id_ptr: int,
                      root: bool = False) -> int:
        """Device-resident queries and outputs (raw device pointers)."""
        kk = ctypes.c_int32(0)
        _check(lib().vrs_knn_search_ex(self._h, ctypes.c_void_p(q_ptr) if q_ptr else None, nq, int(k),
                                       ctypes.c_void_p(dist_ptr) if dist_ptr else None,
                                       ctypes.c_void_p(id_ptr) if id_ptr else None,
                                       ctypes.byref(kk), 1 | (MEM_ROOT if root else 0)))
        return kk.value

    def set_stream(self, cuda_stream: Optional[int]):
        """Issue this handle's work on a caller stream (cudaStream_t as int)."""
        _check(lib().vrs_knn_set_stream(self._h, None if not cuda_stream else
                                        ctypes.c_void_p(cuda_stream)))

    def search_batch(self, queries, k: int) -> List[List[SearchResult]]:
        """distributed_knn.rs:155-231."""
        q = _f32(queries).reshape(-1)
        nq = q.size // self._dim
        if nq == 0:
            return []
        if k == 0 or self.num_vectors() == 0:
            return [[] for _ in range(nq)]
        dist, ids = self.search_arrays(q, k)
        return [[SearchResult(int(i), float(d)) for d, i in zip(dr, ir) if i != 0xFFFFFFFF]
                for dr, ir in zip(dist, ids)]

    def search(self, query, k: int) -> List[SearchResult]:
        """distributed_knn.rs:149-153."""
        res = self.search_batch(query, k)
        return res[0] if res else []

    def _info(self):
        n = ctypes.c_int64()
        d, g, m, mt = (ctypes.c_int32() for _ in range(4))
        _check(lib().vrs_knn_info(self._h, ctypes.byref(n), ctypes.byref(d), ctypes.byref(g),
                                  ctypes.byref(m), ctypes.byref(mt)))
        return n.value, d.value, g.value, m.value, mt.value

    def num_gpus(self) -> int:
        return self._info()[2]

    def mode(self) -> GpuShardMode:
        return GpuShardMode(self._info()[3])

    def dimension(self) -> int:
        return self._info()[1]

    def num_vectors(self) -> int:
        return self._info()[0]

    def metric(self) -> DistanceMetric:
        return DistanceMetric(self._info()[4])


class CudaKnnEngine(DistributedKnnEngine):
    """crates/vector-cuda/src/knn.rs:83-169: the single-GPU engine (GPU 0)."""

    @classmethod
    def new(cls, dataset, dimension: int, metric: DistanceMetric) -> "CudaKnnEngine":
        return cls.try_new(dataset, dimension, 1, GpuShardMode.Sharded, metric)


# ------------------------------------------------------------- k-means


@dataclass
class CudaKMeansResult:
    """crates/vector-cuda/src/kmeans.rs:15-35 (+ the last assignments)."""

    centroids: np.ndarray
    dimension: int
    k: int
    iterations: int
    inertia: float
    assignments: Optional[np.ndarray] = field(default=None, repr=False)

    def centroid(self, i: int) -> np.ndarray:
        return self.centroids[i]


def _empty_result(dimension: int) -> CudaKMeansResult:
    return CudaKMeansResult(np.zeros((0, dimension), np.float32), dimension, 0, 0, 0.0, None)


class DistributedKMeansEngine:
    """crates/vector-cuda/src/ddp/distributed_kmeans.rs:19-106."""

    def __init__(self, num_gpus: int):
        self._g = num_gpus

    @classmethod
    def try_new(cls, num_gpus: int) -> "DistributedKMeansEngine":
        if num_gpus < 1:
            raise ValueError("num_gpus must be at least 1")
        avail = CudaDeviceContext.device_count()
        if num_gpus > avail:
            raise CudaError(1, f"Insufficient hardware GPUs: requested {num_gpus} device(s), "
                               f"but only {avail} physical GPU(s) found",
                            requested=num_gpus, available=avail)
        return cls(num_gpus)

    new = try_new

    def num_gpus(self) -> int:
        return self._g

    def fit(self, data, dimension: int, k: int, max_iters: int, tolerance: float,
            metric: DistanceMetric, init=None, return_assignments: bool = True) -> CudaKMeansResult:
        x = _f32(data).reshape(-1)
        n = x.size // dimension if dimension else 0
        if n == 0 or k == 0:
            return _empty_result(dimension)
        kk = min(k, n)
        init_arr = None if init is None else _f32(init).reshape(-1)
        if init_arr is not None and init_arr.size != kk * dimension:
            raise ValueError("init must hold min(k, n) x dimension values")
        cent = np.empty(kk * dimension, np.float32)
        assign = np.empty(n, np.int32) if return_assignments else None
        ok, it, inertia = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_double()
        _check(lib().vrs_kmeans_fit(_ptr(x), n, dimension, k, _ptr(init_arr), max_iters,
                                    float(tolerance), int(metric), self._g, _ptr(cent),
                                    _ptr(assign), ctypes.byref(ok), ctypes.byref(it),
                                    ctypes.byref(inertia)))
        return CudaKMeansResult(cent.reshape(kk, dimension), dimension, ok.value, it.value,
                                inertia.value, assign)


class CudaKMeansEngine(DistributedKMeansEngine):
    """crates/vector-cuda/src/kmeans.rs:38-97: single GPU."""

    def __init__(self):
        super().__init__(1)

    @classmethod
    def new(cls) -> "CudaKMeansEngine":
        return cls()


# ------------------------------------------------- VECRSTOR vector files


class MmapStorage:
    """crates/vector-index/src/storage/mmap.rs: read-only VECRSTOR vectors.
    The header is validated by libvrs (vrs_vecrstor_info, the checks of
    MmapStorage::open); the rows are a numpy memmap, so nothing is copied."""

    HEADER_SIZE = 24

    def __init__(self, path, num_vectors: int, dimension: int):
        self.path = os.fspath(path)
        self._n = num_vectors
        self._d = dimension
        self._rows = (np.memmap(self.path, np.dtype("<f4"), "r", self.HEADER_SIZE,
                                (num_vectors, dimension)) if num_vectors * dimension
                      else np.zeros((num_vectors, dimension), np.float32))

    @classmethod
    def open(cls, path) -> "MmapStorage":
        """mmap.rs:171-223."""
        n, d = ctypes.c_int64(0), ctypes.c_int64(0)
        _check(lib().vrs_vecrstor_info(os.fsencode(path), ctypes.byref(n), ctypes.byref(d)))
        return cls(path, n.value, d.value)

    @staticmethod
    def create(path, dimension: int, vectors: Sequence) -> None:
        """mmap.rs:90-121: every vector must have `dimension` entries."""
        for v in vectors:
            if len(v) != dimension:
                raise ValueError(f"dimension mismatch: expected {dimension}, got {len(v)}")
        flat = (np.asarray(vectors, np.float32).reshape(-1) if len(vectors)
                else np.zeros(0, np.float32))
        MmapStorage.create_from_flat(path, dimension, flat)

    @staticmethod
    def create_from_flat(path, dimension: int, flat_data) -> None:
        """mmap.rs:131-160."""
        flat = _f32(flat_data).reshape(-1)
        if dimension < 1 and flat.size:
            raise ValueError("dimension must be positive")
        if dimension and flat.size % dimension:
            raise ValueError(f"dimension mismatch: expected {dimension}, got {flat.size % dimension}")
        n = flat.size // dimension if dimension else 0
        _check(lib().vrs_vecrstor_write(os.fsencode(path), _ptr(flat) if flat.size else None,
                                        n, dimension))

    def __len__(self) -> int:
        return self._n

    def len(self) -> int:
        return self._n

    def is_empty(self) -> bool:
        return self._n == 0

    def dimension(self) -> int:
        return self._d

    def get(self, i: int) -> np.ndarray:
        """mmap.rs:237-249: out-of-range ids raise (the reference panics)."""
        if not 0 <= i < self._n:
            raise IndexError(f"vector id {i} out of bounds (len={self._n})")
        return self._rows[i]

    def as_raw_slice(self) -> np.ndarray:
        return self._rows.reshape(-1)


@dataclass
class CentroidFileData:
    """crates/vector-index/src/ivf/serializer.rs:378-395."""

    centroids: np.ndarray
    dimension: int
    k: int
    metric: DistanceMetric
    iterations: int
    inertia: float


class IvfPqSerializer:
    """The standalone centroid file of crates/vector-index/src/ivf/serializer.rs:255-370,
    written and read by libvrs (vrs_centroid_file_write / _read)."""

    @staticmethod
    def save_centroid_file(path, centroids, dimension: int, k: int, metric: DistanceMetric,
                           iterations: int, inertia: float) -> None:
        c = _f32(centroids).reshape(-1)
        if c.size != dimension * k:
            raise ValueError(f"centroids hold {c.size} values, expected k x dimension = {k * dimension}")
        _check(lib().vrs_centroid_file_write(os.fsencode(path), _ptr(c) if c.size else None,
                                             dimension, k, int(metric), iterations, inertia))

    @staticmethod
    def load_centroid_file(path) -> CentroidFileData:
        m, d, k, it = ctypes.c_int32(0), ctypes.c_int64(0), ctypes.c_int64(0), ctypes.c_int64(0)
        inertia = ctypes.c_float(0.0)
        L, fp = lib(), os.fsencode(path)
        _check(L.vrs_centroid_file_read(fp, None, 0, ctypes.byref(m), ctypes.byref(d),
                                        ctypes.byref(k), ctypes.byref(it), ctypes.byref(inertia)))
        out = np.empty(max(d.value * k.value, 1), np.float32)
        _check(L.vrs_centroid_file_read(fp, _ptr(out), out.size, None, None, None, None, None))
        return CentroidFileData(out[:d.value * k.value].reshape(k.value, d.value), d.value, k.value,
                                DistanceMetric(m.value), it.value, float(inertia.value))


# ------------------------------------------------ IVF coarse quantiser


class CoarseQuantizer:
    """The K coarse centroids of an IVF index held on the GPU, answering the
    two questions the reference's IvfPqIndex asks its k-means quantiser:
    `find_top_centroids` (crates/vector-index/src/ivf/kmeans.rs:312-356, per
    query in IvfPqIndex::search, ivf/mod.rs:277-284) and `assign`
    (kmeans.rs:264-309 per base vector in IvfPqIndex::build, mod.rs:119-125),
    each as one batched GPU search over the centroids."""

    def __init__(self, centroids, dimension: int, metric: DistanceMetric, num_gpus: int = 1):
        self._engine = DistributedKnnEngine.try_new(centroids, dimension, num_gpus,
                                                    GpuShardMode.Sharded, metric)
        self._dim = dimension
        self.metric = DistanceMetric(metric)

    @property
    def nlist(self) -> int:
        return self._engine.num_vectors()

    def close(self):
        self._engine.close()

    def _rows(self, x) -> Tuple[np.ndarray, int]:
        q = _f32(x).reshape(-1)
        if q.size % self._dim:
            raise ValueError("input length must be a multiple of dimension")
        return q, q.size // self._dim

    def find_top_centroids(self, queries, nprobe: int) -> Tuple[np.ndarray, np.ndarray]:
        """(scores[nq, P] f32, indices[nq, P] int64), P = min(nprobe, K),
        best first; equal scores keep index order."""
        q, nq = self._rows(queries)
        if nprobe < 0:
            raise ValueError("nprobe must be non-negative")
        cap = max(nq * min(nprobe, self.nlist), 1)
        sc = np.empty(cap, np.float32)
        ix = np.empty(cap, np.int64)
        p = ctypes.c_int32(0)
        _check(lib().vrs_ivf_find_top_centroids(self._engine._h, _ptr(q), nq, int(nprobe),
                                                _ptr(sc), _ptr(ix), ctypes.byref(p)))
        p = p.value
        return sc[:nq * p].reshape(nq, p), ix[:nq * p].reshape(nq, p)

    def assign(self, x) -> Tuple[np.ndarray, np.ndarray]:
        """(indices[n] int64, scores[n] f32): the nearest centroid of each row."""
        q, n = self._rows(x)
        ix = np.empty(max(n, 1), np.int64)
        sc = np.empty(max(n, 1), np.float32)
        _check(lib().vrs_ivf_assign(self._engine._h, _ptr(q), n, _ptr(ix), _ptr(sc)))
        return ix[:n], sc[:n]


class KMeans:
    """The reference's single-vector helpers (crates/vector-index/src/ivf/kmeans.rs),
    answered on the GPU. Each call uploads the centroids; hold a
    CoarseQuantizer to probe or assign many vectors against the same ones."""

    @staticmethod
    def find_nearest_centroid(vector, centroids, dimension: int,
                              metric: DistanceMetric) -> Tuple[int, float]:
        """kmeans.rs:264-309."""
        cq = CoarseQuantizer(centroids, dimension, metric)
        try:
            ix, sc = cq.assign(vector)
            return int(ix[0]), float(sc[0])
        finally:
            cq.close()

    @staticmethod
    def find_top_centroids(query, centroids, dimension: int, nprobe: int,
                           metric: DistanceMetric) -> List[Tuple[int, float]]:
        """kmeans.rs:312-356."""
        cq = CoarseQuantizer(centroids, dimension, metric)
        try:
            sc, ix = cq.find_top_centroids(query, nprobe)
            return [(int(i), float(s)) for i, s in zip(ix[0], sc[0])] if len(sc) else []
        finally:
            cq.close()


# ---------------------------------------------------- rank mode (NCCL)


class IvfPqIndex:
    """A trained IVF-PQ index on the GPU (IvfPqIndex of
    crates/vector-index/src/ivf/mod.rs): coarse centroids, product-quantizer
    codebooks and inverted lists (ids, u8 codes) uploaded once;
    search_batch is search_with_nprobe for many queries."""

    def __init__(self, coarse_centroids, dimension: int, codebooks, num_subvectors: int, sub_clusters: int,
                 lists, metric: DistanceMetric):
        """lists: sequence of (ids, codes[len, num_subvectors]) per coarse centroid."""
        cc = _f32(coarse_centroids).reshape(-1)
        nlist = cc.size // dimension
        off = np.zeros(nlist + 1, np.int64)
        for c in range(nlist):
            off[c + 1] = off[c] + len(lists[c][0])
        ids = np.ascontiguousarray(np.concatenate([np.asarray(l[0], np.uint32) for l in lists])
                                   if nlist else np.zeros(0, np.uint32), dtype=np.uint32)
        codes = np.ascontiguousarray(
            np.concatenate([np.asarray(l[1], np.uint8).reshape(-1, num_subvectors) for l in lists])
            if nlist else np.zeros((0, num_subvectors), np.uint8), dtype=np.uint8)
        cb = _f32(codebooks).reshape(-1)
        h = ctypes.c_void_p()
        _check(lib().vrs_ivfpq_create(_ptr(cc) if nlist else None, nlist, dimension, _ptr(cb), num_subvectors,
                                      sub_clusters, _ptr(off), _ptr(ids) if ids.size else None,
                                      _ptr(codes) if codes.size else None, int(metric), ctypes.byref(h)))
        self._h, self._dim = h, dimension

    def close(self):
        if getattr(self, "_h", None):
            lib().vrs_ivfpq_destroy(self._h)
            self._h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def search_batch(self, queries, k: int, nprobe: int):
        """Returns (dist[nq, k], ids[nq, k], count[nq]): row q holds count[q]
        results best first."""
        q = _f32(queries).reshape(-1)
        nq = q.size // self._dim
        dist = np.zeros(max(nq * k, 1), np.float32)
        ids = np.zeros(max(nq * k, 1), np.uint32)
        cnt = np.zeros(max(nq, 1), np.int32)
        _check(lib().vrs_ivfpq_search(self._h, _ptr(q), nq, int(k), int(nprobe), _ptr(dist), _ptr(ids), _ptr(cnt)))
        return dist[:nq * k].reshape(nq, k), ids[:nq * k].reshape(nq, k), cnt[:nq]

    def search_with_nprobe(self, query, k: int, nprobe: int) -> List[SearchResult]:
        d, i, c = self.search_batch(query, k, nprobe)
        return [SearchResult(int(i[0, r]), float(d[0, r])) for r in range(int(c[0]))]


class Comm:
    """One process per GPU: wraps vrs_comm_* (NCCL communicator)."""

    def __init__(self, c):
        self._c = c

    @staticmethod
    def unique_id() -> bytes:
        buf = (ctypes.c_uint8 * 128)()
        _check(lib().vrs_comm_unique_id(buf))
        return bytes(buf)

    @classmethod
    def init(cls, uid: bytes, nranks: int, rank: int, device: int) -> "Comm":
        buf = (ctypes.c_uint8 * 128).from_buffer_copy(uid)
        c = ctypes.c_void_p()
        _check(lib().vrs_comm_init(buf, nranks, rank, device, ctypes.byref(c)))
        return cls(c)

    def close(self):
        if self._c:
            lib().vrs_comm_destroy(self._c)
            self._c = None


def kmeans_fit_rank(comm: Comm, x_local, n_global: int, dimension: int, k: int, init,
                    max_iters: int, tolerance: float, metric: DistanceMetric,
                    device_ptr: Optional[int] = None, n_local: Optional[int] = None):
    """Rank-mode Lloyd k-means (vrs_kmeans_fit_rank). Returns
    (CudaKMeansResult, local assignments)."""
    kk = min(k, n_global)
    init_arr = None if init is None else _f32(init).reshape(-1)
    cent = np.empty(max(kk * dimension, 1), np.float32)
    ok, it, inertia = ctypes.c_int32(), ctypes.c_int32(), ctypes.c_double()
    if device_ptr is not None:
        nl = int(n_local)
        xp, mem = ctypes.c_void_p(device_ptr), 1
    else:
        xl = _f32(x_local).reshape(-1)
        nl = xl.size // dimension
        xp, mem = _ptr(xl), 0
    assign = np.empty(max(nl, 1), np.int32)
    _check(lib().vrs_kmeans_fit_rank(comm._c, xp, nl, n_global, dimension, k, _ptr(init_arr),
                                     max_iters, float(tolerance), int(metric), mem, _ptr(cent),
                                     _ptr(assign), ctypes.byref(ok), ctypes.byref(it),
                                     ctypes.byref(inertia)))
    res = CudaKMeansResult(cent[:ok.value * dimension].reshape(ok.value, dimension), dimension,
                           ok.value, it.value, inertia.value, assign[:nl])
    return res


# ------------------------------------------------------------ profiling


def profile_enable(on=True):
    """True/1: time every named stage; 2: only whole loops ("kmeans_loop");
    False/0: off."""
    _check(lib().vrs_profile_enable(int(on)))


def profile_reset():
    _check(lib().vrs_profile_reset())


def profile_read(name: str):
    """(total device ms, launches) of a named kernel since the last reset."""
    ms, n = ctypes.c_double(), ctypes.c_int64()
    _check(lib().vrs_profile_read(name.encode(), ctypes.byref(ms), ctypes.byref(n)))
    return ms.value, n.value


# ------------------------------------------------------ synthetic data

GEN_NORMAL, GEN_NORMAL_UNIT, GEN_UNIFORM, GEN_UNIFORM_SUM1, GEN_MIXTURE = range(5)
SEED_BASE = 0x5652535F42303031  # "VRS_B001"


def shard_rows(n: int, world: int, rank: int) -> Tuple[int, int]:
    """Rows [r0, r1) held by `rank` of `world` under GpuShardMode::Sharded:
    contiguous chunks of ceil(n / world), the last ones possibly short or
    empty (ddp/distributed_knn.rs:106-111, ddp/distributed_kmeans.rs:137-142).
    Global row ids are r0 + local id."""
    chunk = -(-n // world) if world > 0 else 0
    r0 = min(n, rank * chunk)
    return r0, min(n, r0 + chunk)


def query_chunk(nq: int, world: int, rank: int) -> Tuple[int, int]:
    """Queries [q0, q1) answered by `rank` under GpuShardMode::Replicated:
    chunks of ceil(nq / world) in query order (ddp/distributed_knn.rs:203-229)."""
    return shard_rows(nq, world, rank)


MEM_ROOT = 2  # VRS_MEM_ROOT


def config_seed(index: int) -> int:
    return (SEED_BASE + index) & 0xFFFFFFFFFFFFFFFF


def gen_rows_host(kind: int, seed: int, stream: int, row0: int, rows: int, d: int,
                  centres: Optional[np.ndarray] = None, K: int = 0, sigma: float = 0.0) -> np.ndarray:
    out = np.empty((rows, d), np.float32)
    c = None if centres is None else _f32(centres)
    _check(lib().vrs_gen_rows_host(kind, seed, stream, row0, rows, d, d, _ptr(out), _ptr(c), K,
                                   sigma))
    return out


def gen_rows_device(kind: int, seed: int, stream: int, row0: int, rows: int, d: int,
                    out_ptr: int, centres_ptr: Optional[int] = None, K: int = 0,
                    sigma: float = 0.0, cuda_stream: Optional[int] = None):
    _check(lib().vrs_gen_rows_device(kind, seed, stream, row0, rows, d, d,
                                     ctypes.c_void_p(out_ptr),
                                     None if centres_ptr is None else ctypes.c_void_p(centres_ptr),
                                     K, sigma,
                                     None if cuda_stream is None else ctypes.c_void_p(cuda_stream)))


__all__ = [
    "DistanceMetric", "GpuShardMode", "CudaError", "SearchResult", "CudaDeviceContext",
    "DistributedKnnEngine", "CudaKnnEngine", "CudaKMeansResult", "CudaKMeansEngine",
    "DistributedKMeansEngine", "Comm", "kmeans_fit_rank", "gen_rows_host", "gen_rows_device",
    "config_seed", "shard_rows", "query_chunk", "lib", "LIB_PATH", "profile_enable", "profile_reset", "profile_read",
]
