// Internal C++ API of the exact k-NN engine (device pointers, stream
// ordered).  Mirrors the reference's C++ entry points
// (include/mlxvs/mlxvs.h:22-65, :780-784) with mx::array replaced by device
// pointers and sizes.  Errors: std::invalid_argument for bad arguments,
// std::runtime_error for CUDA failures.
#pragma once

#include <cuda_runtime.h>
#include <stdint.h>

namespace mlxvs_b200 {

/** ref: include/mlxvs/mlxvs.h:22-29 */
enum class Metric : int { InnerProduct = 0, L2 = 1, Cosine = 2 };

/** The kind of a key list: a Metric, or Hamming distances. */
constexpr int KIND_HAMMING = 3;

/** ref: include/mlxvs/mlxvs.h:45-51.  tile_rows is accepted for signature
 * compatibility; the kernels pick their own tiles. */
struct KnnOptions {
  int tile_rows = 65536;
};

/** Exact k-NN: ids int32 [nq, k] and distances float32 [nq, k] (dist may be
 * null).  ref: brute_force_knn, src/knn.cpp:71-142. */
void brute_force_knn(const float* base, int64_t n, const float* queries, int64_t nq, int d, int k,
                     Metric metric, int32_t* ids, float* dist, cudaStream_t s,
                     const KnnOptions& options = {});

/** One shard's k best keys per query [nq, k], best first, ids offset. */
void knn_keys(const float* base, int64_t n, const float* queries, int64_t nq, int d, int k,
              Metric metric, int64_t id_offset, uint64_t* keys, cudaStream_t s);

/** Exact k-NN graph of rows [n, d]: for rows query_begin .. query_end - 1,
 * the k nearest other rows, as brute_force_knn returns them (ids, dist
 * [query_end - query_begin, k]).  ref: all_neighbors with algo BruteForce
 * and one cluster, src/all_neighbors.cpp:56-95,250-263,364-377. */
void all_neighbors(const float* rows, int64_t n, int d, int k, Metric metric,
                   int64_t query_begin, int64_t query_end, int32_t* ids, float* dist,
                   cudaStream_t s);

/** One merge step: the best k of each row of scores [nq, t] (ids
 * id_offset + column) together with the running lists ids / best [nq, k]
 * (ignored when first), best first: out_ids, out_scores [nq, k].
 * ref: topk_merge, src/knn.cpp:37-69, include/mlxvs/mlxvs.h:898-905. */
void topk_merge(const float* scores, int64_t nq, int t, const int32_t* ids, const float* best,
                int id_offset, bool first, int k, int32_t* out_ids, float* out_scores,
                cudaStream_t s);

/** Exact re-ranking: the k nearest of each query's candidate ids [nq, c]
 * (ids outside [0, n) skipped) by exact distances, nearest first, as
 * brute_force_knn returns them.  ref: refine, src/ivf.cpp:1642-1708. */
void refine(const float* dataset, int64_t n, int d, const float* queries, int64_t nq,
            const int32_t* candidates, int c, int k, Metric metric, int32_t* ids, float* dist,
            cudaStream_t s);

/** Exact Hamming k-NN.  ref: hamming_knn, src/ivf.cpp:1343-1403. */
void hamming_knn(const uint8_t* rows, int64_t n, const uint8_t* queries, int64_t nq, int bytes,
                 int k, int32_t* ids, float* dist, cudaStream_t s);

void hamming_keys(const uint8_t* rows, int64_t n, const uint8_t* queries, int64_t nq, int bytes,
                  int k, int64_t id_offset, uint64_t* keys, cudaStream_t s);

/** Best k of num_lists key lists [num_lists][nq][k], as ids and distances
 * of the given kind (a Metric value or KIND_HAMMING). */
void merge_keys(const uint64_t* lists, int num_lists, int64_t nq, int k, int kind,
                const float* queries, int d, int32_t* ids, float* dist, cudaStream_t s);

/** Waits for s, then throws if a kernel of this library recorded an error
 * on the current device (and clears it). */
void device_synchronize(cudaStream_t s);

/** Per-kernel device times for benchmarks: when on, launches are bracketed
 * by CUDA events on their stream.  Enabling (or disabling) clears the
 * records. */
void profile_enable(bool on);

/** Sum of the recorded device times (ms) and launch count of the kernels
 * named `name` ("prep", "gemm_topk", "merge", "hamming_topk", "sumsq",
 * "fill"), or of all of them when name is null.  Waits for the events. */
void profile_read(const char* name, double* total_ms, int64_t* launches);
void profile_issued(const char* name, double* ops);

/** Hamming k-NN with no device allocation: its scratch is a 16 MiB static
 * device array shared by all calls (they race if they overlap on the GPU).
 * Codes must be 16, 32, 64, 128, 256 or 512 bytes and 16-byte aligned. The
 * first call on a device looks the array up.  Waits for its stream. */
void hamming_knn_noalloc(const uint8_t* rows, int64_t n, const uint8_t* queries, int64_t nq,
                         int bytes, int k, int32_t* ids, float* dist, cudaStream_t s);

/** A row-sharded search's exchange of key lists between the GPUs of one
 * node, replacing an all-gather followed by a merge: every GPU writes its
 * [nq, k] keys of a step into its own buffer, publishes the step's epoch in
 * a flag there, and merges the world's lists by reading its peers' buffers
 * over NVLink (CUDA IPC mappings, plain loads).  Two key slots alternate by
 * epoch, so a GPU never overwrites keys a slower peer may still read.  One
 * object per process and GPU; epochs start at 1 and rise by one per step,
 * in the same order on every GPU. */
struct Exchange;
Exchange* exchange_create(int world, int rank, int64_t capacity_keys);
/** The IPC handle (64 bytes) of this GPU's buffer, for the peers. */
void exchange_handle(Exchange* x, void* handle);
/** Maps a peer's buffer from its handle. */
void exchange_open(Exchange* x, int peer, const void* handle);
/** This GPU's key slot of an epoch: [nq, k] keys, nq * k <= capacity. */
uint64_t* exchange_keys(Exchange* x, uint32_t epoch);
/** Publishes this GPU's keys of the epoch, waits (bounded) for every peer's,
 * and merges the world's lists into ids and distances of the given kind, as
 * merge_keys does; queued on s. */
void exchange_merge(Exchange* x, uint32_t epoch, int64_t nq, int k, int kind,
                    const float* queries, int d, int32_t* ids, float* dist, cudaStream_t s);
void exchange_destroy(Exchange* x);

/** Version string. */
const char* version();

}  // namespace mlxvs_b200
