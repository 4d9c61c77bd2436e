"""CPU restatement of VectorRS's IVF-PQ ADC search (TEST INFRASTRUCTURE ONLY).

Only ``tests/`` may import this module; the product never does. Pure Python
over the pinned pair arithmetic of ``oracle.distance`` (the AVX-512
restatement), for small cases:

* ``pq_encode``        -- ProductQuantizer::encode (crates/vector-index/src/ivf/pq.rs:178-201)
* ``pq_adc_lut``       -- ProductQuantizer::compute_adc_lut (pq.rs:233-268)
* ``pq_distance_with_lut`` -- ProductQuantizer::compute_distance_with_lut (pq.rs:270-296):
  4-way chunks summed as (d0 + d1) + (d2 + d3), then the remainder, in f32
* ``ivf_pq_search``    -- IvfPqIndex::search (crates/vector-index/src/ivf/mod.rs:265-345)
  given trained coarse centroids, codebooks and inverted lists;
  ``ivf_pq_search_c`` is the same search in C (``orc_ivfpq_search``) for
  larger cases, cross-checked against this one.

The search keeps its k best candidates in Rust's ``std::collections::BinaryHeap``
ordered by heap score alone (mod.rs:28-54: equal scores compare Equal, no id
tie-break), so which of several equal-score candidates survive, and their
output order, follow that heap's algorithm. ``RustMaxHeap`` restates the
published std algorithm: push = append + sift_up; pop = take the last element,
swap it into the root, sift_down_to_bottom (always towards the larger child,
the right one when left <= right), then sift_up; sift_up stops at the first
parent that is >= the element.

Training (PQ sub-space k-means with random initialisation, pq.rs:53-169) is
not restated: it is not deterministic in the reference.
"""
from __future__ import annotations

import numpy as np

import oracle

HIGHER_IS_BETTER = oracle.HIGHER_IS_BETTER


def _cmp(a: float, b: float) -> int:
    """f32::partial_cmp(..).unwrap_or(Equal) as -1 / 0 / 1."""
    if a < b:
        return -1
    if a > b:
        return 1
    return 0


class RustMaxHeap:
    """std::collections::BinaryHeap over (heap_score, id, distance) entries,
    compared on heap_score only."""

    def __init__(self):
        self.data = []

    def __len__(self):
        return len(self.data)

    def peek(self):
        return self.data[0] if self.data else None

    def push(self, item):
        self.data.append(item)
        self._sift_up(0, len(self.data) - 1)

    def pop(self):
        if not self.data:
            return None
        item = self.data.pop()
        if self.data:
            item, self.data[0] = self.data[0], item
            self._sift_down_to_bottom(0)
        return item

    def _sift_up(self, start: int, pos: int) -> int:
        elem = self.data[pos]
        while pos > start:
            parent = (pos - 1) // 2
            if _cmp(elem[0], self.data[parent][0]) <= 0:  # elem <= parent: stop
                break
            self.data[pos] = self.data[parent]
            pos = parent
        self.data[pos] = elem
        return pos

    def _sift_down_to_bottom(self, pos: int):
        end = len(self.data)
        start = pos
        elem = self.data[pos]
        child = 2 * pos + 1
        while child <= end - 2:
            if _cmp(self.data[child][0], self.data[child + 1][0]) <= 0:  # left <= right
                child += 1
            self.data[pos] = self.data[child]
            pos = child
            child = 2 * pos + 1
        if child == end - 1:
            self.data[pos] = self.data[child]
            pos = child
        self.data[pos] = elem
        self._sift_up(start, pos)


def pq_encode(vector, codebooks, num_subvectors: int, sub_clusters: int, metric: int) -> np.ndarray:
    """pq.rs:178-201: per sub-space, the nearest sub-centroid (kmeans.rs:264-309)."""
    v = np.asarray(vector, np.float32)
    ds = v.size // num_subvectors
    cb = np.asarray(codebooks, np.float32).reshape(num_subvectors, sub_clusters, ds)
    return np.array([oracle.find_nearest_centroid(v[m * ds:(m + 1) * ds], cb[m], metric)[0]
                     for m in range(num_subvectors)], np.uint8)


def pq_adc_lut(query, codebooks, num_subvectors: int, sub_clusters: int, metric: int) -> np.ndarray:
    """pq.rs:233-268: lut[m * sub_clusters + k] = metric(q_m, c_{m,k})."""
    q = np.asarray(query, np.float32)
    ds = q.size // num_subvectors
    cb = np.asarray(codebooks, np.float32).reshape(num_subvectors, sub_clusters, ds)
    lut = np.empty(num_subvectors * sub_clusters, np.float32)
    for m in range(num_subvectors):
        for k in range(sub_clusters):
            lut[m * sub_clusters + k] = oracle.distance(metric, q[m * ds:(m + 1) * ds], cb[m, k])
    return lut


def pq_distance_with_lut(code, lut, sub_clusters: int) -> np.float32:
    """pq.rs:270-296, in f32: total += (d0 + d1) + (d2 + d3) per 4 codes, then
    the remaining codes one by one."""
    code = [int(c) for c in code]
    lut = np.asarray(lut, np.float32)
    total = np.float32(0.0)
    m = 0
    full = len(code) - len(code) % 4
    while m < full:
        d0 = lut[m * sub_clusters + code[m]]
        d1 = lut[(m + 1) * sub_clusters + code[m + 1]]
        d2 = lut[(m + 2) * sub_clusters + code[m + 2]]
        d3 = lut[(m + 3) * sub_clusters + code[m + 3]]
        total = np.float32(total + np.float32(np.float32(d0 + d1) + np.float32(d2 + d3)))
        m += 4
    while m < len(code):
        total = np.float32(total + lut[m * sub_clusters + code[m]])
        m += 1
    return total


def ivf_pq_search(query, k: int, nprobe: int, coarse_centroids, lists, codebooks,
                  num_subvectors: int, sub_clusters: int, metric: int):
    """mod.rs:265-345 on a trained index. ``lists[c]`` = (ids, codes[len, M]).
    Returns [(id, distance)] best first, at most k entries."""
    cc = np.asarray(coarse_centroids, np.float32)
    nlist = cc.shape[0]
    if k == 0 or nlist == 0:
        return []
    eff = max(min(nprobe, nlist), 1)
    top = oracle.find_top_centroids(query, cc, eff, metric)
    q = np.asarray(query, np.float32)
    hib = metric in HIGHER_IS_BETTER
    heap = RustMaxHeap()
    for cid, _ in top:
        ids, codes = lists[cid]
        if len(ids) == 0:
            continue
        resid = (q - cc[cid]).astype(np.float32)  # f32 subtraction per element
        lut = pq_adc_lut(resid, codebooks, num_subvectors, sub_clusters, metric)
        for i, vid in enumerate(ids):
            dist = pq_distance_with_lut(codes[i], lut, sub_clusters)
            hs = np.float32(-dist) if hib else dist
            if len(heap) < k:
                heap.push((hs, int(vid), dist))
            elif _cmp(hs, heap.peek()[0]) < 0:
                heap.pop()
                heap.push((hs, int(vid), dist))
    out = []
    while len(heap):
        hs, vid, dist = heap.pop()
        out.append((vid, dist))
    out.reverse()
    return out


def flatten_lists(lists, num_subvectors: int):
    """(offsets[nlist + 1] i64, ids u32, codes [total][M] u8) of per-list (ids, codes)."""
    nlist = len(lists)
    off = np.zeros(nlist + 1, np.int64)
    for c in range(nlist):
        off[c + 1] = off[c] + len(lists[c][0])
    ids = np.ascontiguousarray(np.concatenate([np.asarray(l[0], np.uint32) for l in lists])
                               if nlist else np.zeros(0, np.uint32), dtype=np.uint32)
    codes = np.ascontiguousarray(
        np.concatenate([np.asarray(l[1], np.uint8).reshape(-1, num_subvectors) for l in lists])
        if nlist else np.zeros((0, num_subvectors), np.uint8), dtype=np.uint8)
    return off, ids, codes


def ivf_pq_search_c(query, k: int, nprobe: int, coarse_centroids, lists, codebooks,
                    num_subvectors: int, sub_clusters: int, metric: int, use_simd: int = -1):
    """The same search in C (``orc_ivfpq_search`` in vrs_oracle.c), for sizes the
    Python loops cannot reach. Returns (distances f32[c], ids u32[c])."""
    off, ids, codes = flatten_lists(lists, num_subvectors)
    return ivf_pq_search_c_flat(query, k, nprobe, coarse_centroids, off, ids, codes, codebooks,
                                num_subvectors, sub_clusters, metric, use_simd)


def ivf_pq_search_c_flat(query, k: int, nprobe: int, coarse_centroids, off, ids, codes, codebooks,
                         num_subvectors: int, sub_clusters: int, metric: int, use_simd: int = -1):
    """ivf_pq_search_c on lists already flattened by flatten_lists (arrays
    C-contiguous: offsets i64, ids u32, codes u8)."""
    import ctypes
    L = oracle.lib()
    q = np.ascontiguousarray(query, np.float32)
    cc = np.ascontiguousarray(coarse_centroids, np.float32)
    nlist = cc.shape[0] if cc.ndim == 2 else 0
    cb = np.ascontiguousarray(codebooks, np.float32)
    out_d = np.zeros(max(k, 1), np.float32)
    out_i = np.zeros(max(k, 1), np.uint32)
    P = ctypes.c_void_p
    fn = L.orc_ivfpq_search
    fn.restype = ctypes.c_int
    fn.argtypes = [P, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, ctypes.c_int, P, P, P, P,
                   ctypes.c_int, ctypes.c_int, ctypes.c_int, ctypes.c_int, P, P]
    n = fn(q.ctypes.data, q.size, int(k), int(nprobe), cc.ctypes.data if nlist else None, nlist,
           off.ctypes.data, ids.ctypes.data, codes.ctypes.data, cb.ctypes.data, num_subvectors,
           sub_clusters, int(metric), use_simd, out_d.ctypes.data, out_i.ctypes.data)
    return out_d[:n], out_i[:n]
