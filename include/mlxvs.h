/*
 * C++ API of the exact k-NN search, with the reference's names, argument
 * order, defaults and exceptions (include/mlxvs/mlxvs.h:22-65, :780-784,
 * :898-905), over a plain array view instead of an MLX array.
 *
 * An Array is a row-major view of host memory (device == -1) or of one CUDA
 * device's memory (device >= 0).  Inputs may be any real dtype; they are
 * used as float32, as the reference's float_rows does (src/utils.h:18-29).
 * Results are Arrays that own their memory, on the queries' device.  Work
 * is queued on the given CUDA stream (a cudaStream_t; null: the default
 * stream); results on a device are ready once that stream reaches them,
 * results on the host when the call returns.
 *
 * Errors: std::invalid_argument with "[mlxvs::<op>] ..." messages for bad
 * arguments, std::runtime_error for CUDA failures.
 */
#ifndef MLXVS_B200_CPP_H
#define MLXVS_B200_CPP_H

#include <cstdint>
#include <memory>
#include <utility>
#include <vector>

#define MLXVS_CPP_API __attribute__((visibility("default")))

namespace mlxvs {

/** Element types an Array may hold. */
enum class Dtype : int32_t {
  Float32,
  Float16,
  BFloat16,
  Float64,
  Int8,
  UInt8,
  Int16,
  Int32,
  Int64,
  Bool,
};

/** Bytes per element of a Dtype. */
MLXVS_CPP_API int64_t dtype_size(Dtype t);

/**
 * A row-major array: data, shape and element type, on the host (device -1)
 * or a CUDA device (its ordinal).  A view does not own its data; arrays the
 * library returns keep theirs alive through `owner`.
 */
struct Array {
  void* data = nullptr;
  std::vector<int64_t> shape;
  Dtype dtype = Dtype::Float32;
  int device = -1;
  std::shared_ptr<void> owner;

  int ndim() const { return (int)shape.size(); }
  int64_t size() const {
    int64_t s = 1;
    for (int64_t e : shape) s *= e;
    return s;
  }
  template <class T>
  T* ptr() const {
    return static_cast<T*>(data);
  }
};

/** A view of existing memory (no copy, no ownership). */
inline Array view(void* data, std::vector<int64_t> shape, Dtype dtype, int device = -1) {
  Array a;
  a.data = data;
  a.shape = std::move(shape);
  a.dtype = dtype;
  a.device = device;
  return a;
}

/** A CUDA stream (cudaStream_t); null is the default stream. */
using Stream = void*;

/** How two rows compare.  ref: include/mlxvs/mlxvs.h:22-29 */
enum class Metric {
  /** Dot product, larger is closer. */
  InnerProduct,
  /** Squared Euclidean distance, smaller is closer. */
  L2,
  /** Cosine similarity, larger is closer. */
  Cosine,
};

/** The k nearest rows of each query, nearest first.
 * ref: include/mlxvs/mlxvs.h:32-42 */
struct Neighbors {
  /** Row indices, int32 [nq, k]; -1 where fewer exist. */
  Array ids;
  /** float32 [nq, k]: dot product, cosine similarity or squared distance;
   * a missing neighbor has -inf, or +inf for L2. */
  Array distances;
};

/** Options of brute_force_knn.  ref: include/mlxvs/mlxvs.h:45-51.
 * tile_rows is accepted for compatibility: the fused kernels choose their
 * own tiles and never materialize a score matrix. */
struct KnnOptions {
  int tile_rows = 65536;
};

/**
 * Exact k nearest neighbors of every row of queries [nq, d] among the rows
 * of base [n, d] (any real dtype, computed as float32).  1 <= k <= 256.
 * ref: include/mlxvs/mlxvs.h:59-65, src/knn.cpp:71-142.
 */
MLXVS_CPP_API Neighbors brute_force_knn(const Array& base, const Array& queries, int k,
                                        Metric metric, const KnnOptions& options = {},
                                        Stream s = {});

/**
 * Exact k-NN of bit-packed queries uint8 [nq, bytes] among bit-packed rows
 * uint8 [n, bytes] by Hamming distance: ids and distances (exact integers
 * as float32), nearest first, ties to the lower id.  k <= 256.
 * ref: include/mlxvs/mlxvs.h:780-784, src/ivf.cpp:1343-1403.
 */
MLXVS_CPP_API Neighbors hamming_knn(const Array& rows, const Array& queries, int k,
                                    Stream s = {});

/**
 * One merge step of brute_force_knn: the best k of each row of scores
 * float32 [nq, t] (ids id_offset + column) together with the running lists
 * ids int32 / best float32 [nq, k], ignored when first is set.  Returns the
 * merged ids and scores, best first.
 * ref: include/mlxvs/mlxvs.h:898-905, src/knn.cpp:37-69.
 */
MLXVS_CPP_API std::pair<Array, Array> topk_merge(const Array& scores, const Array& ids,
                                                 const Array& best, int id_offset, bool first,
                                                 int k, Stream s = {});

}  // namespace mlxvs

#endif /* MLXVS_B200_CPP_H */
