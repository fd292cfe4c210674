// The C++ API of include/mlxvs.h over the engine (device arrays) and the C
// API's host-memory entries (host arrays).  Argument checks and messages
// restate the reference's (src/utils.h:18-38, src/knn.cpp:78-92,
// src/ivf.cpp:1123-1127,1350-1362).
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "engine.h"
#include "mlxvs.h"
#include "mlxvs_c.h"

namespace {

using mlxvs::Array;
using mlxvs::Dtype;

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    throw std::runtime_error(std::string("[mlxvs_b200] CUDA error: ") + cudaGetErrorString(e) +
                             " (" + what + ")");
  }
}

// A C API status as the exception the C++ API throws.
void check_status(int rc) {
  if (rc == MLXVS_OK) return;
  const std::string msg = mlxvs_last_error();
  if (rc == MLXVS_ERROR_INVALID_ARGUMENT) throw std::invalid_argument(msg);
  throw std::runtime_error(msg);
}

// Makes a device current for the scope (restoring the previous one).
struct DeviceScope {
  int prev = -1;
  explicit DeviceScope(int dev) {
    if (dev < 0) return;
    ck(cudaGetDevice(&prev), "cudaGetDevice");
    if (prev != dev) ck(cudaSetDevice(dev), "cudaSetDevice");
  }
  ~DeviceScope() {
    int cur = -1;
    if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
  }
};

// An owning array: host memory (device -1) or device memory freed when the
// last reference goes.
Array make_array(std::vector<int64_t> shape, Dtype dtype, int device) {
  Array a;
  a.shape = std::move(shape);
  a.dtype = dtype;
  a.device = device;
  const size_t bytes = (size_t)std::max<int64_t>(a.size(), 1) * mlxvs::dtype_size(dtype);
  if (device < 0) {
    auto buf = std::shared_ptr<uint8_t>(new uint8_t[bytes], std::default_delete<uint8_t[]>());
    a.data = buf.get();
    a.owner = buf;
  } else {
    void* p = nullptr;
    ck(cudaMalloc(&p, bytes), "cudaMalloc");
    a.data = p;
    a.owner = std::shared_ptr<void>(p, [](void* q) { cudaFree(q); });
  }
  return a;
}

template <class T>
__global__ void to_float_kernel(const T* x, int64_t count, float* y) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = static_cast<float>(x[i]);
}

template <class T>
__global__ void half_to_float_kernel(const T* x, int64_t count, float* y) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = __half2float(x[i]);
}

__global__ void bf16_to_float_kernel(const __nv_bfloat16* x, int64_t count, float* y) {
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < count;
       i += (int64_t)gridDim.x * blockDim.x)
    y[i] = __bfloat162float(x[i]);
}

template <class T>
void host_to_float(const void* x, int64_t count, float* y) {
  const T* s = static_cast<const T*>(x);
  for (int64_t i = 0; i < count; ++i) y[i] = static_cast<float>(s[i]);
}

std::string op_msg(const char* op, const char* name, const char* what) {
  return std::string("[") + op + "] " + name + " " + what;
}

// float_rows (src/utils.h:18-29): a 2-D array of any real dtype as float32
// rows on the array's own memory.  A float32 array is used in place; others
// are converted into `holder`.
const float* float_rows(const Array& x, const char* op, const char* name, Array& holder,
                        cudaStream_t s) {
  if (x.ndim() != 2) throw std::invalid_argument(op_msg(op, name, "must be 2-D [n, d]."));
  if (x.dtype == Dtype::Bool) throw std::invalid_argument(op_msg(op, name, "must be real numbers."));
  if (x.size() > 0 && x.data == nullptr)
    throw std::invalid_argument(op_msg(op, name, "has no data."));
  if (x.dtype == Dtype::Float32) return x.ptr<float>();
  holder = make_array(x.shape, Dtype::Float32, x.device);
  const int64_t count = x.size();
  float* y = holder.ptr<float>();
  if (count == 0) return y;
  if (x.device < 0) {
    switch (x.dtype) {
      case Dtype::Float16: {
        const __half* h = x.ptr<__half>();
        for (int64_t i = 0; i < count; ++i) y[i] = __half2float(h[i]);
        break;
      }
      case Dtype::BFloat16: {
        const __nv_bfloat16* h = x.ptr<__nv_bfloat16>();
        for (int64_t i = 0; i < count; ++i) y[i] = __bfloat162float(h[i]);
        break;
      }
      case Dtype::Float64: host_to_float<double>(x.data, count, y); break;
      case Dtype::Int8: host_to_float<int8_t>(x.data, count, y); break;
      case Dtype::UInt8: host_to_float<uint8_t>(x.data, count, y); break;
      case Dtype::Int16: host_to_float<int16_t>(x.data, count, y); break;
      case Dtype::Int32: host_to_float<int32_t>(x.data, count, y); break;
      case Dtype::Int64: host_to_float<int64_t>(x.data, count, y); break;
      default: throw std::invalid_argument(op_msg(op, name, "must be real numbers."));
    }
    return y;
  }
  const unsigned grid = (unsigned)std::min<int64_t>((count + 255) / 256, 4096);
  switch (x.dtype) {
    case Dtype::Float16:
      half_to_float_kernel<<<grid, 256, 0, s>>>(x.ptr<__half>(), count, y);
      break;
    case Dtype::BFloat16:
      bf16_to_float_kernel<<<grid, 256, 0, s>>>(x.ptr<__nv_bfloat16>(), count, y);
      break;
    case Dtype::Float64: to_float_kernel<<<grid, 256, 0, s>>>(x.ptr<double>(), count, y); break;
    case Dtype::Int8: to_float_kernel<<<grid, 256, 0, s>>>(x.ptr<int8_t>(), count, y); break;
    case Dtype::UInt8: to_float_kernel<<<grid, 256, 0, s>>>(x.ptr<uint8_t>(), count, y); break;
    case Dtype::Int16: to_float_kernel<<<grid, 256, 0, s>>>(x.ptr<int16_t>(), count, y); break;
    case Dtype::Int32: to_float_kernel<<<grid, 256, 0, s>>>(x.ptr<int32_t>(), count, y); break;
    case Dtype::Int64: to_float_kernel<<<grid, 256, 0, s>>>(x.ptr<int64_t>(), count, y); break;
    default: throw std::invalid_argument(op_msg(op, name, "must be real numbers."));
  }
  ck(cudaGetLastError(), "float_rows conversion");
  return y;
}

// Both arrays on the host, or both on one device (which is returned, -1 for
// the host).
int common_device(const Array& a, const Array& b, const char* op) {
  if (a.device != b.device)
    throw std::invalid_argument(std::string("[") + op +
                                "] the arrays must be on the same device.");
  return a.device;
}

}  // namespace

namespace mlxvs {

int64_t dtype_size(Dtype t) {
  switch (t) {
    case Dtype::Float64:
    case Dtype::Int64: return 8;
    case Dtype::Float32:
    case Dtype::Int32: return 4;
    case Dtype::Float16:
    case Dtype::BFloat16:
    case Dtype::Int16: return 2;
    default: return 1;
  }
}

// ref: mlxvs::brute_force_knn, src/knn.cpp:71-142
Neighbors brute_force_knn(const Array& base, const Array& queries, int k, Metric metric,
                          const KnnOptions& options, Stream stream) {
  const char* op = "mlxvs::brute_force_knn";
  const int dev = common_device(base, queries, op);
  DeviceScope scope(dev);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  Array hb, hq;
  const float* b = float_rows(base, op, "base", hb, s);
  const float* q = float_rows(queries, op, "queries", hq, s);
  if (base.shape[1] != queries.shape[1])
    throw std::invalid_argument(
        "[mlxvs::brute_force_knn] base and queries must have the same number of columns.");
  if (k < 1 || k > 256) throw std::invalid_argument("[mlxvs::brute_force_knn] k must be in [1, 256].");
  const int64_t n = base.shape[0], nq = queries.shape[0];
  const int64_t d = base.shape[1];
  if (d > INT32_MAX) throw std::invalid_argument("[mlxvs::brute_force_knn] d is too large.");
  Neighbors out;
  out.ids = make_array({nq, k}, Dtype::Int32, dev);
  out.distances = make_array({nq, k}, Dtype::Float32, dev);
  if (dev < 0) {
    // the host entry: chunked copies overlapped with the search
    check_status(mlxvs_brute_force_knn(b, n, q, nq, (int32_t)d, k, (mlxvs_metric)metric,
                                       out.ids.ptr<int32_t>(), out.distances.ptr<float>()));
  } else {
    mlxvs_b200::KnnOptions o;
    o.tile_rows = options.tile_rows;
    mlxvs_b200::brute_force_knn(b, n, q, nq, (int)d, k, (mlxvs_b200::Metric)metric,
                                out.ids.ptr<int32_t>(), out.distances.ptr<float>(), s, o);
    // the converted inputs live until the stream has used them
    if (hb.owner || hq.owner) ck(cudaStreamSynchronize(s), "cudaStreamSynchronize");
  }
  return out;
}

// ref: mlxvs::hamming_knn, src/ivf.cpp:1343-1403 (argument checks of
// pack_words, src/ivf.cpp:1123-1127)
Neighbors hamming_knn(const Array& rows, const Array& queries, int k, Stream stream) {
  const char* op = "mlxvs::hamming_knn";
  for (const Array* a : {&rows, &queries})
    if (a->ndim() != 2 || a->dtype != Dtype::UInt8)
      throw std::invalid_argument("[mlxvs::hamming_knn] rows must be bit-packed uint8 [n, bytes].");
  if (queries.shape[1] != rows.shape[1])
    throw std::invalid_argument("[mlxvs::hamming_knn] queries must have the rows' bytes.");
  if (k < 1 || k > 256) throw std::invalid_argument("[mlxvs::hamming_knn] k must be in [1, 256].");
  const int dev = common_device(rows, queries, op);
  DeviceScope scope(dev);
  const int64_t n = rows.shape[0], nq = queries.shape[0], bytes = rows.shape[1];
  if (bytes > INT32_MAX) throw std::invalid_argument("[mlxvs::hamming_knn] too many bytes per row.");
  Neighbors out;
  out.ids = make_array({nq, k}, Dtype::Int32, dev);
  out.distances = make_array({nq, k}, Dtype::Float32, dev);
  if (dev < 0)
    check_status(mlxvs_hamming_knn(rows.ptr<uint8_t>(), n, queries.ptr<uint8_t>(), nq,
                                   (int32_t)bytes, k, out.ids.ptr<int32_t>(),
                                   out.distances.ptr<float>()));
  else
    mlxvs_b200::hamming_knn(rows.ptr<uint8_t>(), n, queries.ptr<uint8_t>(), nq, (int)bytes, k,
                            out.ids.ptr<int32_t>(), out.distances.ptr<float>(),
                            static_cast<cudaStream_t>(stream));
  return out;
}

// ref: mlxvs::topk_merge, src/knn.cpp:37-69
std::pair<Array, Array> topk_merge(const Array& scores, const Array& ids, const Array& best,
                                   int id_offset, bool first, int k, Stream stream) {
  if (scores.ndim() != 2 || scores.dtype != Dtype::Float32)
    throw std::invalid_argument("[mlxvs::topk_merge] scores must be float32 [nq, t]");
  if (k < 1 || k > 256) throw std::invalid_argument("[mlxvs::topk_merge] k must be in [1, 256]");
  const int64_t nq = scores.shape[0], t = scores.shape[1];
  if (t > INT32_MAX) throw std::invalid_argument("[mlxvs::topk_merge] t is too large.");
  const int dev = scores.device;
  if (!first) {
    if (ids.ndim() != 2 || ids.dtype != Dtype::Int32 || ids.shape[0] != nq || ids.shape[1] != k ||
        best.ndim() != 2 || best.dtype != Dtype::Float32 || best.shape[0] != nq ||
        best.shape[1] != k)
      throw std::invalid_argument(
          "[mlxvs::topk_merge] ids and best must be int32 and float32 [nq, k] unless first.");
    common_device(scores, ids, "mlxvs::topk_merge");
    common_device(scores, best, "mlxvs::topk_merge");
  }
  DeviceScope scope(dev);
  Array out_ids = make_array({nq, k}, Dtype::Int32, dev);
  Array out_scores = make_array({nq, k}, Dtype::Float32, dev);
  const int32_t* pi = first ? nullptr : ids.ptr<int32_t>();
  const float* pb = first ? nullptr : best.ptr<float>();
  if (dev < 0)
    check_status(mlxvs_topk_merge(scores.ptr<float>(), nq, (int32_t)t, pi, pb, id_offset,
                                  first ? 1 : 0, k, out_ids.ptr<int32_t>(),
                                  out_scores.ptr<float>()));
  else
    mlxvs_b200::topk_merge(scores.ptr<float>(), nq, (int)t, pi, pb, id_offset, first, k,
                           out_ids.ptr<int32_t>(), out_scores.ptr<float>(),
                           static_cast<cudaStream_t>(stream));
  return {out_ids, out_scores};
}

}  // namespace mlxvs
