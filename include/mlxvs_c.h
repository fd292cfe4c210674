/*
 * mlxvs_b200 C API: exact k-nearest-neighbor search on NVIDIA B200 (sm_100a).
 *
 * Drop-in for the brute-force part of mlxVS's C API
 * (include/mlxvs/mlxvs_c.h in the reference).  Conventions follow it:
 *   - every function returns MLXVS_OK (0) or an error code, and
 *     mlxvs_last_error() then describes the failure (per thread; "" after a
 *     success)                                   ref: src/c_api.cpp:28-47
 *   - host-memory entry points take row-major host arrays, copy the inputs
 *     and write the outputs into buffers the caller owns
 *   - ids are int32 [nq, k], -1 where fewer than k rows exist; distances are
 *     float32 [nq, k]: squared L2 (ascending, +inf where missing), or the
 *     inner product / cosine similarity (descending, -inf where missing)
 *   - ties keep the lower id (ref: src/kernels.h:20-23)
 *
 * Entry points marked "device" take CUDA device pointers and a cudaStream_t
 * (as void*, NULL = the legacy default stream); they enqueue work and return
 * without waiting, except where noted.  Errors found by the kernels
 * themselves are reported by mlxvs_device_synchronize().
 */
#ifndef MLXVS_B200_C_H
#define MLXVS_B200_C_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define MLXVS_C_API __attribute__((visibility("default")))

/** The C API's version: major * 10000 + minor (ref: mlxvs_c.h:25). */
#define MLXVS_C_API_VERSION 100

/* ref: include/mlxvs/mlxvs_c.h:27-35 (same values) */
typedef enum {
  MLXVS_OK = 0,
  /** An argument was out of range (mlxvs_last_error says which). */
  MLXVS_ERROR_INVALID_ARGUMENT = 1,
  /** Kept for value compatibility; the search functions do no file I/O. */
  MLXVS_ERROR_IO = 2,
  /** Anything else: no CUDA device, out of device memory, a kernel error. */
  MLXVS_ERROR_INTERNAL = 3,
} mlxvs_status;

/* ref: include/mlxvs/mlxvs_c.h:37-45 (same values) */
typedef enum {
  /** Dot product, larger is closer. */
  MLXVS_INNER_PRODUCT = 0,
  /** Squared Euclidean distance, smaller is closer. */
  MLXVS_L2 = 1,
  /** Cosine similarity, larger is closer. */
  MLXVS_COSINE = 2,
} mlxvs_metric;

/** Candidate-key lists produced by the *_keys_device functions hold
 * Hamming keys when merged with this kind (not a metric of
 * mlxvs_brute_force_knn). */
#define MLXVS_KIND_HAMMING 3

/** The last error of this thread, or "" after a success.
 * ref: include/mlxvs/mlxvs_c.h:105-106, src/c_api.cpp:190-192 */
MLXVS_C_API const char* mlxvs_last_error(void);

/** The library version, such as "0.16.1-b200".
 * ref: include/mlxvs/mlxvs_c.h:108-109, src/c_api.cpp:194-196 */
MLXVS_C_API const char* mlxvs_version(void);

/**
 * Exact k-nearest neighbors of nq queries among n base rows (float32,
 * row-major, host memory).  1 <= k <= 256; distances may be NULL.
 * Replaces: mlxvs_brute_force_knn, include/mlxvs/mlxvs_c.h:247-256,
 * src/c_api.cpp:468-489 (same signature and semantics).
 */
MLXVS_C_API int mlxvs_brute_force_knn(
    const float* base,
    int64_t n,
    const float* queries,
    int64_t nq,
    int32_t d,
    int32_t k,
    mlxvs_metric metric,
    int32_t* ids,
    float* distances);

/**
 * Exact k-NN by Hamming distance of bit-packed rows uint8 [n, bytes] and
 * queries uint8 [nq, bytes] (host memory).  Distances are the Hamming
 * distances as float32, ascending, +inf where missing; ties keep the lower
 * id.  1 <= k <= 256.
 * Replaces: mlxvs::hamming_knn, include/mlxvs/mlxvs.h:780-784 and
 * src/ivf.cpp:1343-1403 (the reference has no C entry for it).
 */
MLXVS_C_API int mlxvs_hamming_knn(
    const uint8_t* rows,
    int64_t n,
    const uint8_t* queries,
    int64_t nq,
    int32_t bytes,
    int32_t k,
    int32_t* ids,
    float* distances);

/**
 * mlxvs_brute_force_knn on device pointers, enqueued on stream.
 * Replaces: mlxvs::brute_force_knn, include/mlxvs/mlxvs.h:59-65 (the C++
 * entry the Python binding python/bindings.cpp:37-47 calls).  The inputs
 * stay untouched; scratch memory comes from the device's stream-ordered
 * pool.  Waits once on the host for the input-conversion kernels' flags
 * (exact fp16 operands or not); for k <= 16 with L2 or inner product the
 * exact path's kernel is already enqueued behind them while the host waits,
 * and returns at once if the flags call for another path.
 */
MLXVS_C_API int mlxvs_brute_force_knn_device(
    const float* base,
    int64_t n,
    const float* queries,
    int64_t nq,
    int32_t d,
    int32_t k,
    mlxvs_metric metric,
    int32_t* ids,
    float* distances,
    void* stream);

/** mlxvs_hamming_knn on device pointers, enqueued on stream.
 * Replaces: mlxvs::hamming_knn, include/mlxvs/mlxvs.h:780-784. */
MLXVS_C_API int mlxvs_hamming_knn_device(
    const uint8_t* rows,
    int64_t n,
    const uint8_t* queries,
    int64_t nq,
    int32_t bytes,
    int32_t k,
    int32_t* ids,
    float* distances,
    void* stream);

/**
 * One shard of a row-sharded search: the k best candidates of every query
 * among these n base rows, as 64-bit keys [nq, k], best first, whose ids are
 * id_offset + row.  A key is (order_bits(score) << 32) | (uint32)~id, where
 * order_bits maps a float to an unsigned int of the same order (ref:
 * src/kernels.h:16-19) and score is the reference's pre-distance score
 * (L2: 2 q.b - |b|^2, ref src/knn.cpp:111-116; IP: q.b; cosine: the cosine);
 * larger keys are better and 0 is an empty slot.
 * Replaces: the per-tile step of src/knn.cpp:104-121 across devices.
 */
MLXVS_C_API int mlxvs_knn_keys_device(
    const float* base,
    int64_t n,
    const float* queries,
    int64_t nq,
    int32_t d,
    int32_t k,
    mlxvs_metric metric,
    int64_t id_offset,
    uint64_t* keys,
    void* stream);

/**
 * Exact k-nearest-neighbor graph of rows [n, d] (host, row-major float32):
 * for every row, its k nearest OTHER rows, nearest first, ids [n, k] and
 * distances [n, k] as mlxvs_brute_force_knn returns them (-1 / +-inf where
 * fewer than k exist).  Requires 1 <= k <= 255, n >= 2 and d >= 1.
 * Replaces: mlxvs::all_neighbors with algo BruteForce and one cluster
 * (include/mlxvs/mlxvs.h:187-205, src/all_neighbors.cpp:250-263,364-377);
 * the reference has no C entry for it.  The row itself is excluded inside
 * the search instead of searching k + 1 and dropping it
 * (src/all_neighbors.cpp:56-95).
 */
MLXVS_C_API int mlxvs_all_neighbors(
    const float* rows,
    int64_t n,
    int32_t d,
    int32_t k,
    mlxvs_metric metric,
    int32_t* ids,
    float* distances);

/**
 * Device-pointer variant of mlxvs_all_neighbors for the rows
 * query_begin .. query_end - 1 (their lists [query_end - query_begin, k]),
 * so that devices holding all rows can split the graph by rows.
 * Replaces: as mlxvs_all_neighbors.
 */
MLXVS_C_API int mlxvs_all_neighbors_device(
    const float* rows,
    int64_t n,
    int32_t d,
    int32_t k,
    mlxvs_metric metric,
    int64_t query_begin,
    int64_t query_end,
    int32_t* ids,
    float* distances,
    void* stream);

/**
 * One merge step of the exact search, for tests and benchmarks: the best k
 * of each row of scores [nq, t] (host, row-major float32; ids id_offset +
 * column) together with the running lists ids / best [nq, k], which are
 * ignored (may be NULL) when first != 0.  Writes out_ids / out_scores
 * [nq, k], best first (higher score, then lower id as unsigned), -1 / -inf
 * where fewer than k exist.  1 <= k <= 256.
 * Replaces: mlxvs::topk_merge (include/mlxvs/mlxvs.h:898-905,
 * src/knn.cpp:37-69, kernel src/kernels.h:37-229); no C entry in the
 * reference.
 */
MLXVS_C_API int mlxvs_topk_merge(
    const float* scores,
    int64_t nq,
    int32_t t,
    const int32_t* ids,
    const float* best,
    int32_t id_offset,
    int32_t first,
    int32_t k,
    int32_t* out_ids,
    float* out_scores);

/** mlxvs_topk_merge on device pointers, enqueued on stream.
 * Replaces: as mlxvs_topk_merge. */
MLXVS_C_API int mlxvs_topk_merge_device(
    const float* scores,
    int64_t nq,
    int32_t t,
    const int32_t* ids,
    const float* best,
    int32_t id_offset,
    int32_t first,
    int32_t k,
    int32_t* out_ids,
    float* out_scores,
    void* stream);

/**
 * Exact re-ranking: the k nearest of each query's candidate ids
 * candidates [nq, c] (ids into dataset [n, d]; ids outside [0, n) are
 * skipped) by exact distances, nearest first, as mlxvs_brute_force_knn
 * returns them (-1 / +-inf where fewer than k are valid).  Equal distances
 * keep the candidates' order.  Host buffers; only the distinct candidate
 * rows are copied to the device.  1 <= k <= c.
 * Replaces: mlxvs::refine (include/mlxvs/mlxvs.h:853-865,
 * src/ivf.cpp:1642-1708); no C entry in the reference.
 */
MLXVS_C_API int mlxvs_refine(
    const float* dataset,
    int64_t n,
    int32_t d,
    const float* queries,
    int64_t nq,
    const int32_t* candidates,
    int32_t c,
    int32_t k,
    mlxvs_metric metric,
    int32_t* ids,
    float* distances);

/** mlxvs_refine on device pointers (the whole dataset on the device),
 * enqueued on stream.  Replaces: as mlxvs_refine. */
MLXVS_C_API int mlxvs_refine_device(
    const float* dataset,
    int64_t n,
    int32_t d,
    const float* queries,
    int64_t nq,
    const int32_t* candidates,
    int32_t c,
    int32_t k,
    mlxvs_metric metric,
    int32_t* ids,
    float* distances,
    void* stream);

/** Hamming shard: keys of score -distance (see mlxvs_knn_keys_device).
 * Replaces: the tile step of src/ivf.cpp:1370-1387 across devices. */
MLXVS_C_API int mlxvs_hamming_keys_device(
    const uint8_t* rows,
    int64_t n,
    const uint8_t* queries,
    int64_t nq,
    int32_t bytes,
    int32_t k,
    int64_t id_offset,
    uint64_t* keys,
    void* stream);

/**
 * Merges num_lists key lists laid out [num_lists][nq][k] into the k best
 * distinct keys per query (ties keep the lower id; a key present in several
 * lists is taken once; the lists may come in any order, sorted ones merge
 * fastest) and converts them to ids and distances of
 * the given kind (an mlxvs_metric, or MLXVS_KIND_HAMMING).  For MLXVS_L2 the
 * distance is max(|q|^2 - score, 0) (ref: src/knn.cpp:122-131), so queries
 * [nq, d] must be given; otherwise queries may be NULL.
 * Replaces: the cross-tile merge of src/knn.cpp:117 / src/ivf.cpp:1388-1402,
 * here also across devices.
 */
MLXVS_C_API int mlxvs_merge_keys_device(
    const uint64_t* lists,
    int32_t num_lists,
    int64_t nq,
    int32_t k,
    int32_t kind,
    const float* queries,
    int32_t d,
    int32_t* ids,
    float* distances,
    void* stream);

/**
 * Exchange of the row shards' key lists between the GPUs of one node (one
 * process per GPU), replacing an all-gather of the lists followed by
 * mlxvs_merge_keys_device: each GPU writes its [nq, k] keys of a step
 * (mlxvs_knn_keys_device / mlxvs_hamming_keys_device) into its slot of the
 * step's epoch (mlxvs_exchange_keys), then mlxvs_exchange_merge_device
 * publishes them, waits until every GPU has published the same epoch
 * (bounded; a wait that gives up makes that step's results missing and is
 * reported by mlxvs_device_synchronize) and merges the world's lists,
 * reading the peers' slots over NVLink.  Epochs start at 1 and rise by one
 * per step, the same on every GPU.  Set-up: mlxvs_exchange_create on every
 * GPU (world <= 8, capacity >= nq * k keys), exchange the 64-byte handles
 * (mlxvs_exchange_handle) between the processes, mlxvs_exchange_open each
 * peer's.  The merge needs k <= 32 and world * k <= 768.
 * Replaces: the cross-tile merge of src/knn.cpp:117 across devices (no
 * counterpart in the reference, which runs on one device).
 */
MLXVS_C_API int mlxvs_exchange_create(int32_t world, int32_t rank, int64_t capacity_keys,
                                      void** exchange);
MLXVS_C_API int mlxvs_exchange_handle(void* exchange, uint8_t* handle);
MLXVS_C_API int mlxvs_exchange_open(void* exchange, int32_t peer, const uint8_t* handle);
MLXVS_C_API int mlxvs_exchange_keys(void* exchange, uint32_t epoch, uint64_t** keys);
MLXVS_C_API int mlxvs_exchange_merge_device(
    void* exchange,
    uint32_t epoch,
    int64_t nq,
    int32_t k,
    int32_t kind,
    const float* queries,
    int32_t d,
    int32_t* ids,
    float* distances,
    void* stream);
MLXVS_C_API int mlxvs_exchange_destroy(void* exchange);

/**
 * Waits for stream and reports any error the library's kernels recorded on
 * the current device since the last call (a bounded wait that gave up).
 * Not in the reference (MLX reports errors at mx::eval).
 */
MLXVS_C_API int mlxvs_device_synchronize(void* stream);

/**
 * Hamming k-NN for callers that cannot allocate device memory.  No
 * counterpart in the reference: it is mlxvs_hamming_knn_device with every
 * scratch buffer placed in one 16 MiB array that the library reserves
 * statically on each GPU that loads it (held until the process exits), so
 * the call itself never calls cudaMalloc, cudaFree or any allocating
 * routine.  Some callers cannot allocate: a serving loop that may not stall
 * other streams (cudaMalloc and cudaFree synchronize the device), a host
 * framework that has already reserved the device's memory for its own
 * allocator, or code that promises a fixed memory footprint after start-up.
 *
 * Limits: bytes must be 16, 32, 64, 128, 256 or 512 (codes are read in
 * place, so no padded copy is made) and rows / queries 16-byte aligned; the
 * lists for nq * k must fit the array (about (k + 1) * nq * 8 bytes per base
 * range; requests that do not fit even one range fail with
 * MLXVS_ERROR_INVALID_ARGUMENT).  rows, queries, ids and distances are
 * device pointers the caller owns.  The first call on a device looks the
 * array up with cudaGetSymbolAddress and should come before any stream
 * capture.  Every call reuses the same array, so calls that overlap on the
 * GPU (other streams, other host threads, the same device) race; the call
 * waits for its stream before returning and reports a kernel that gave up.
 */
MLXVS_C_API int mlxvs_hamming_knn_noalloc(
    const uint8_t* rows,
    int64_t n,
    const uint8_t* queries,
    int64_t nq,
    int32_t bytes,
    int32_t k,
    int32_t* ids,
    float* distances,
    void* stream);

/**
 * Benchmark support (not in the reference): when on, every launch of this
 * library's kernels is bracketed by CUDA events on its stream.  Turning it
 * on or off clears the records.
 */
MLXVS_C_API int mlxvs_profile_enable(int32_t on);

/**
 * Total device time in ms and launch count of the recorded launches of one
 * kernel ("prep", "gemm_topk", "merge", "hamming_topk", "sumsq", "fill"), or
 * of all of them when kernel is NULL.  Waits for the recorded events.
 */
MLXVS_C_API int mlxvs_profile_read(const char* kernel, double* total_ms, int64_t* launches);

/**
 * Benchmark support (not in the reference): the tensor-core operations
 * (multiply-adds count 2) that the recorded launches of one kernel issued,
 * or of all of them when kernel is NULL -- the MMA shape times the padded
 * query blocks, tiles and K the kernel ran, against which the algorithmic
 * 2*Q*N*D is the useful part.
 */
MLXVS_C_API int mlxvs_profile_issued(const char* kernel, double* tensor_ops);

#ifdef __cplusplus
}
#endif

#endif /* MLXVS_B200_C_H */
