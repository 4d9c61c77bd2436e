/*
 * vrs.h -- C ABI of libvrs, the B200 (sm_100a) implementation of VectorRS's
 * two GPU hot paths: exact batch flat kNN and Lloyd k-means.
 *
 * This is the boundary the reference's Rust crate `vector-cuda` would bind
 * (one `extern "C"` block). Plain pointers and sizes
 * only. Every function returns a vrs_status; on failure a thread-local
 * message is available from vrs_last_error(). There is no CPU fallback:
 * a missing or failing GPU is an error, never a silent slow path (the
 * reference instead falls back to the CPU, crates/vector-cuda/src/knn.rs:161-168).
 *
 * Thread safety: a handle must not be used by two calls at once; distinct
 * handles may be used from distinct threads.
 */
#ifndef VRS_H
#define VRS_H

#include <stdint.h>

#if defined(__GNUC__)
#define VRS_API __attribute__((visibility("default")))
#else
#define VRS_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. 1..5 mirror CudaError, crates/vector-cuda/src/error.rs:7-29. */
typedef enum vrs_status {
  VRS_OK = 0,
  VRS_ERR_INSUFFICIENT_DEVICES = 1, /* CudaError::InsufficientDevices (error.rs:9-13) */
  VRS_ERR_DEVICE_NOT_FOUND = 2,     /* CudaError::DeviceNotFound (error.rs:15-17) */
  VRS_ERR_DRIVER = 3,               /* CudaError::DriverError (error.rs:19-21) */
  VRS_ERR_HARDWARE_NOT_AVAILABLE = 4, /* CudaError::HardwareNotAvailable (error.rs:23-25) */
  VRS_ERR_INVALID_CONFIG = 5,       /* CudaError::InvalidConfig (error.rs:27-29) */
  VRS_ERR_NCCL = 6,                 /* NCCL failure (no reference counterpart: it has no NCCL) */
  VRS_ERR_TIMEOUT = 7,              /* a bounded device or collective wait gave up */
  VRS_ERR_OOM = 8,                  /* device allocation failed */
  VRS_ERR_INVALID_FILE = 9          /* VECRSTOR file: VectorIndexError::{Io, InvalidHeader,
                                       FileSizeMismatch}, crates/vector-index/src/types.rs:60-85 */
} vrs_status;

/* DistanceMetric codes: the reference's launch codes,
 * crates/vector-cuda/src/knn.rs:235-246 (enum at crates/vector-index/src/lib.rs:49-83). */
typedef enum vrs_metric {
  VRS_L2_SQUARED = 0,
  VRS_DOT_PRODUCT = 1,
  VRS_COSINE_SIMILARITY = 2,
  VRS_MANHATTAN = 3,
  VRS_MINKOWSKI = 4, /* p = 3 */
  VRS_CHEBYSHEV = 5,
  VRS_HAMMING = 6,
  VRS_MAHALANOBIS = 7, /* unit covariance: sqrt(L2^2) */
  VRS_JACCARD = 8,
  VRS_HELLINGER = 9
} vrs_metric;

/* GpuShardMode, crates/vector-cuda/src/ddp/distributed_knn.rs:14-19. */
typedef enum vrs_shard_mode { VRS_SHARDED = 0, VRS_REPLICATED = 1 } vrs_shard_mode;

/* Buffer location flags for the *_ex calls. */
#define VRS_MEM_HOST 0
#define VRS_MEM_DEVICE 1
/* vrs_knn_search_ex only, OR'ed with one of the above: in rank mode, only
 * rank 0's query and output pointers are used (the others may be NULL);
 * the queries travel to the other ranks by NCCL broadcast and the merged
 * results come back to rank 0 alone, as to the one caller of
 * search_batch (crates/vector-cuda/src/ddp/distributed_knn.rs:155-231).
 * Without it every rank passes the same queries and receives all results.
 * Ignored by single-process handles (their caller is the root). */
#define VRS_MEM_ROOT 2

/* Replaces CudaDeviceContext::device_count (crates/vector-cuda/src/device.rs:110-118).
 * Writes 0 (and returns VRS_OK) when no driver or GPU is present. */
VRS_API int vrs_device_count(int32_t* out_count);

/* Thread-local message of the last failing call on this thread ("" if none). */
VRS_API const char* vrs_last_error(void);

/* DistanceMetric::higher_is_better (crates/vector-index/src/lib.rs:85-94). */
VRS_API int vrs_metric_higher_is_better(int32_t metric);

/* ------------------------------------------------------------------ kNN */
typedef struct vrs_knn vrs_knn;

/* Replaces DistributedKnnEngine::try_new (crates/vector-cuda/src/ddp/distributed_knn.rs:40-61)
 * and, with num_gpus == 1, CudaKnnEngine::with_ordinal (crates/vector-cuda/src/knn.rs:90-140).
 * base: n x d row-major f32 on the host (copied; the caller keeps ownership).
 * num_gpus > available -> VRS_ERR_INSUFFICIENT_DEVICES. The GPU count is
 * clamped to min(num_gpus, n) as init_engine does (distributed_knn.rs:98).
 * Sharded: GPU r holds rows [r*ceil(n/g), ...) (distributed_knn.rs:104-128).
 * Replicated: every GPU holds all rows (distributed_knn.rs:129-134). */
VRS_API int vrs_knn_create(const float* base, int64_t n, int32_t d, int32_t num_gpus, int32_t mode,
                   int32_t metric, vrs_knn** out);

/* Replaces DistributedKnnEngine::search_batch (distributed_knn.rs:155-231) and
 * CudaKnnEngine::search_batch (knn.rs:151-169). queries: nq x d host f32.
 * Writes k' = min(k, n) results per query, packed with row stride k':
 * out_dist[nq*k'], out_id[nq*k'] (caller provides room for nq*k), best
 * first: ascending distance, or descending similarity for dot/cosine;
 * exactly equal scores are ordered by lower id. Distances are computed in
 * the arithmetic order of the reference's AVX-512 CPU kernels
 * (crates/vector-simd/src/avx512.rs). nq == 0 or k == 0 -> *out_k = 0. */
VRS_API int vrs_knn_search(vrs_knn* h, const float* queries, int64_t nq, int32_t k, float* out_dist,
                   uint32_t* out_id, int32_t* out_k);

/* As vrs_knn_search; mem = VRS_MEM_DEVICE means queries/out_* are device
 * pointers on the handle's first GPU (rank mode: the rank's GPU);
 * VRS_MEM_ROOT (rank mode) reads queries and writes results on rank 0 only. */
VRS_API int vrs_knn_search_ex(vrs_knn* h, const float* queries, int64_t nq, int32_t k, float* out_dist,
                      uint32_t* out_id, int32_t* out_k, int32_t mem);

/* Getters of DistributedKnnEngine (distributed_knn.rs:233-261). */
VRS_API int vrs_knn_info(const vrs_knn* h, int64_t* num_vectors, int32_t* dimension, int32_t* num_gpus,
                 int32_t* mode, int32_t* metric);

VRS_API void vrs_knn_destroy(vrs_knn* h);

/* -------------------------------------------------------------- k-means */

/* Replaces CudaKMeansEngine::fit (crates/vector-cuda/src/kmeans.rs:58-97) for
 * num_gpus == 1 and DistributedKMeansEngine::fit
 * (crates/vector-cuda/src/ddp/distributed_kmeans.rs:55-106) for num_gpus > 1.
 * x: n x d host f32. init: k' x d initial centroids, or NULL for the first k'
 * points (k' = min(k, n)). Lloyd iterations stop after max_iters or when
 * the largest squared centroid shift is <= tol (kmeans.rs:218-223).
 * Outputs: out_centroids (k' x d), out_assign (n, nullable), *out_k = k',
 * *out_iters, *out_inertia = sum over points of the metric value to the
 * assigned centroid in the last assignment step (kmeans.rs:293-297).
 * Empty clusters keep their centroid (kernels/kmeans.cu:350-356). */
VRS_API int vrs_kmeans_fit(const float* x, int64_t n, int32_t d, int32_t k, const float* init,
                   int32_t max_iters, float tol, int32_t metric, int32_t num_gpus,
                   float* out_centroids, int32_t* out_assign, int32_t* out_k, int32_t* out_iters,
                   double* out_inertia);

/* ------------------------------------------- IVF coarse quantiser probing */
/* Both take a vrs_knn handle created over the K coarse centroids (K x d,
 * vrs_knn_create with the index's metric) and run one batched kNN search;
 * scores are the metric's raw values (similarities not negated) in the
 * AVX-512 DistanceEngine's arithmetic, indices are centroid rows. */

/* Replaces KMeans::find_top_centroids (crates/vector-index/src/ivf/kmeans.rs:312-356),
 * batched over nq queries as IvfPqIndex::search calls it per query
 * (crates/vector-index/src/ivf/mod.rs:277-284). Writes P = min(nprobe, K)
 * entries per query, row stride P: out_score[nq*P], out_idx[nq*P], best
 * first (ascending distance, descending similarity); exactly equal values
 * keep index order, as the reference's stable sort does (kmeans.rs:345-350).
 * nprobe == 0 or K == 0 -> *out_p = 0. P > 2048 is rejected, and for
 * Minkowski, Mahalanobis and Hellinger P = 2048 < K as well (the entry after
 * the boundary must be fetched to order equal roots by index). */
VRS_API int vrs_ivf_find_top_centroids(vrs_knn* centroids, const float* queries, int64_t nq,
                                       int32_t nprobe, float* out_score, int64_t* out_idx,
                                       int32_t* out_p);

/* Replaces KMeans::find_nearest_centroid (kmeans.rs:264-309) over n vectors,
 * as IvfPqIndex::build calls it per base vector (mod.rs:119-125, 203-210):
 * out_idx[n] the nearest centroid (lowest index among equal best values, the
 * reference's strict comparison, kmeans.rs:297-305), out_score[n] (nullable)
 * its value. K == 0 -> index 0 and +inf (-inf for dot/cosine), the initial
 * values of the reference's loop (kmeans.rs:272-277). */
VRS_API int vrs_ivf_assign(vrs_knn* centroids, const float* x, int64_t n, int64_t* out_idx,
                           float* out_score);

/* ------------------------------------------------------ IVF-PQ ADC search */
/* A trained IVF-PQ index held on the current device: nlist coarse centroids
 * (nlist x d), the product quantizer's codebooks (num_subvectors x
 * sub_clusters sub-centroids of d / num_subvectors floats, the layout of
 * ProductQuantizer, crates/vector-index/src/ivf/pq.rs), and the inverted
 * lists back to back: list c holds entries [list_offsets[c],
 * list_offsets[c+1]) of ids (u32) and codes (num_subvectors bytes each, as
 * InvertedList, crates/vector-index/src/ivf/inverted_list.rs:9-15).
 * sub_clusters <= 256; num_subvectors * sub_clusters <= 16384; d <= 4096
 * and a multiple of num_subvectors. Copies everything; the caller keeps its
 * buffers. */
typedef struct vrs_ivfpq vrs_ivfpq;
VRS_API int vrs_ivfpq_create(const float* coarse_centroids, int64_t nlist, int32_t d, const float* codebooks,
                             int32_t num_subvectors, int32_t sub_clusters, const int64_t* list_offsets,
                             const uint32_t* ids, const uint8_t* codes, int32_t metric, vrs_ivfpq** out);

/* Replaces IvfPqIndex::search_with_nprobe (crates/vector-index/src/ivf/mod.rs:
 * 265-345) for nq queries (host buffers): coarse probe of nprobe' =
 * max(1, min(nprobe, nlist)) lists (find_top_centroids order), per list the
 * residual's ADC table (pq.rs:233-268) and the four-way f32 sums of
 * compute_distance_with_lut (pq.rs:270-296), the k best kept exactly as the
 * reference's BinaryHeap keeps them (equal scores included). Row q of
 * out_dist/out_id (stride k) holds out_count[q] <= k results, best first;
 * k == 0 or an empty index gives counts of 0. k <= 2048. */
VRS_API int vrs_ivfpq_search(vrs_ivfpq* h, const float* queries, int64_t nq, int32_t k, int32_t nprobe,
                             float* out_dist, uint32_t* out_id, int32_t* out_count);
VRS_API void vrs_ivfpq_destroy(vrs_ivfpq* h);

/* --------------------------------------------------- VECRSTOR vector files */
/* Format of crates/vector-index/src/storage/mmap.rs:7-16: three little-endian
 * u64 (magic 0x5645435253544F52 "VECRSTOR", N, D), then N x D f32 rows. */

/* The header checks of MmapStorage::open (mmap.rs:171-223): shorter than 24
 * bytes or another magic -> VRS_ERR_INVALID_FILE (InvalidHeader); shorter
 * than 24 + N*D*4 bytes -> VRS_ERR_INVALID_FILE (FileSizeMismatch); longer
 * files are accepted. Writes N and D. */
VRS_API int vrs_vecrstor_info(const char* path, int64_t* num_vectors, int64_t* dimension);

/* MmapStorage::create_from_flat (mmap.rs:131-160): header + n x d rows. */
VRS_API int vrs_vecrstor_write(const char* path, const float* data, int64_t n, int64_t d);

/* vrs_knn_create over the rows of a VECRSTOR file, in place of
 * DistributedKnnEngine::try_new(storage.as_raw_slice(), ...) with an
 * MmapStorage: the file is validated as vrs_vecrstor_info does, mapped
 * read-only and each GPU's row range is uploaded from the mapping (no host
 * copy of the base). D must be in 1..2^31-1. */
VRS_API int vrs_knn_create_from_file(const char* path, int32_t num_gpus, int32_t mode,
                                     int32_t metric, vrs_knn** out);

/* IvfPqSerializer::save_centroid_file (crates/vector-index/src/ivf/serializer.rs:255-307):
 * the k-means output (e.g. out_centroids/out_k/out_iters/out_inertia of
 * vrs_kmeans_fit) as a standalone file: packed little-endian header of 29
 * bytes -- magic u64 "VRSKMEAN" (0x5652534B4D45414E), version u32 = 1,
 * metric u8 (vrs_metric codes, serializer.rs:397-410), D u32, K u32,
 * iterations u32, inertia f32 -- then K x D f32. */
VRS_API int vrs_centroid_file_write(const char* path, const float* centroids, int64_t d, int64_t k,
                                    int32_t metric, int64_t iterations, float inertia);

/* IvfPqSerializer::load_centroid_file (serializer.rs:309-370). With
 * out_centroids NULL only the header is read (to size the buffer); else
 * K x D floats are read into it (capacity in floats). Wrong magic, version or
 * metric code (serializer.rs:318-339, 413-430) and short files ->
 * VRS_ERR_INVALID_FILE with the reference's messages. */
VRS_API int vrs_centroid_file_read(const char* path, float* out_centroids, int64_t capacity,
                                   int32_t* metric, int64_t* d, int64_t* k, int64_t* iterations,
                                   float* inertia);

/* ---------------------------------------- one process per GPU (rank mode) */
/* The multi-process form of the engines above: each process drives one GPU
 * and owns one row shard; the ranks exchange through NCCL. Replaces the
 * per-iteration MPI_Allreduce of crates/vector-mpi/src/distributed_kmeans.rs:173-260
 * and the host merge of crates/vector-cuda/src/ddp/collective.rs:115-159. */
typedef struct vrs_comm vrs_comm;

/* 128-byte NCCL unique id, created on one rank and shared out of band. */
VRS_API int vrs_comm_unique_id(uint8_t out_id[128]);
VRS_API int vrs_comm_init(const uint8_t id[128], int32_t nranks, int32_t rank, int32_t device,
                  vrs_comm** out);
VRS_API void vrs_comm_destroy(vrs_comm* c);

/* Rank-local shard of a Sharded (or full copy of a Replicated) index.
 * shard: n_local x d, host or device (mem). global_offset: global id of
 * shard row 0; n_global: rows over all ranks. For a Sharded handle over more
 * than one rank this is a collective (all ranks call it): the ranks agree on
 * the search path and the largest row norm, which the pooled pivot bounds
 * of vrs_knn_search need. */
VRS_API int vrs_knn_create_rank(vrs_comm* comm, const float* shard, int64_t n_local,
                        int64_t global_offset, int64_t n_global, int32_t d, int32_t mode,
                        int32_t metric, int32_t mem, vrs_knn** out);

/* Rank-mode k-means: every rank passes its own rows (host or device) and
 * the same init (k' x d, host; NULL -> the first k' global rows, which must
 * lie on rank 0). Outputs are identical on all ranks; out_assign (nullable)
 * receives this rank's n_local assignments. */
VRS_API int vrs_kmeans_fit_rank(vrs_comm* comm, const float* x_local, int64_t n_local, int64_t n_global,
                        int32_t d, int32_t k, const float* init, int32_t max_iters, float tol,
                        int32_t metric, int32_t mem, float* out_centroids, int32_t* out_assign,
                        int32_t* out_k, int32_t* out_iters, double* out_inertia);

/* No counterpart in the reference. Exact kNN for callers that cannot
 * allocate device memory during a search (inside a captured or
 * allocation-free region, behind a plugin host or caching pool that owns
 * all device memory, or in latency-critical loops): nothing is allocated;
 * base (n x d), queries (nq x d), out_dist and out_id (nq x k', k' =
 * min(k, n), packed) are caller-provided device pointers on the current
 * device, and work is queued on cuda_stream (NULL = default stream); the
 * call returns without waiting. Scratch is one fixed 8 MiB device array per
 * device, held until exit; a batch whose candidate lists do not fit is
 * rejected with VRS_ERR_INVALID_CONFIG (split it). The first call on a
 * device looks up that array's address, so make it before any stream
 * capture. That address is cached for the life of the process, so do not
 * use this entry point across a cudaDeviceReset (or any other teardown of
 * the device's primary context). Calls that overlap on the GPU share the
 * array and race. Cosine and Hellinger are rejected (they need per-row
 * norms or roots). */
VRS_API int vrs_knn_search_noalloc(const float* base, int64_t n, int32_t d, const float* queries,
                                   int64_t nq, int32_t k, int32_t metric, float* out_dist,
                                   uint32_t* out_id, int32_t* out_k, void* cuda_stream);

/* No counterpart in the reference (its kernels have no bounded waits).
 * Self-test of the device-side bounded wait every tensor-core pipeline
 * uses: one thread on the current device waits on an mbarrier that nothing
 * arrives on, through the same helper, for limit_ns (1 us .. 1 s). Returns
 * VRS_ERR_TIMEOUT with the stage code in vrs_last_error() when the wait gave
 * up as designed, and leaves the device usable. */
VRS_API int vrs_selftest_bounded_wait(int64_t limit_ns);

/* ------------------------------------------------------ streams, profiling */
/* Makes a single-GPU or rank-mode handle issue its work on `cuda_stream`
 * (a cudaStream_t of the handle's device; NULL restores the handle's own).
 * Calls still return only after their results are ready. */
VRS_API int vrs_knn_set_stream(vrs_knn* h, void* cuda_stream);

/* Kernel timing with CUDA events (off by default). When on (1), every
 * launch of the named stages below is bracketed by events on its stream and
 * the elapsed device time is accumulated per name: "knn_prep", "knn_pivot",
 * "knn_scan", "knn_select", "knn_gather", "knn_merge", "knn_fallback",
 * "kmeans_assign", "kmeans_finalize", "kmeans_sums", "kmeans_update",
 * "kmeans_loop" (a whole Lloyd loop). With on = 2 only the whole-loop stage
 * ("kmeans_loop") is timed, so the per-iteration host work stays as with
 * profiling off. "*" reads the count of kernel launches since the reset;
 * "knn_fallback_queries" (with on = 1) counts, in `launches`, the queries
 * that took the exact re-search (total_ms stays 0). */
VRS_API int vrs_profile_enable(int32_t on);
VRS_API int vrs_profile_reset(void);
VRS_API int vrs_profile_read(const char* name, double* total_ms, int64_t* launches);

/* ------------------------------------------------ seeded synthetic inputs */
/* Counter-based Philox4x32-10 generator; identical bits on host and device.
 * kind: 0 N(0,1); 1 N(0,1) rows L2-normalised (f64); 2 U[0,1); 3 U[0,1)
 * rows rescaled to sum 1 (f64); 4 Gaussian mixture: centre (K x d, given)
 * chosen per row + sigma * N(0,1). Writes rows [row0, row0+rows) of the
 * conceptual matrix, ld floats apart. */
#define VRS_GEN_NORMAL 0
#define VRS_GEN_NORMAL_UNIT 1
#define VRS_GEN_UNIFORM 2
#define VRS_GEN_UNIFORM_SUM1 3
#define VRS_GEN_MIXTURE 4
VRS_API int vrs_gen_rows_host(int32_t kind, uint64_t seed, uint32_t stream, int64_t row0, int64_t rows,
                      int32_t d, int64_t ld, float* out, const float* centres, uint32_t K,
                      double sigma);
/* Same rows generated on the current device into device memory (out and
 * centres are device pointers); stream is a cudaStream_t or NULL. */
VRS_API int vrs_gen_rows_device(int32_t kind, uint64_t seed, uint32_t stream_id, int64_t row0,
                        int64_t rows, int32_t d, int64_t ld, float* out, const float* centres,
                        uint32_t K, double sigma, void* cuda_stream);

#ifdef __cplusplus
}
#endif

#endif /* VRS_H */
