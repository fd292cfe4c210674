// The C API (include/mlxvs_c.h) over the engine.  Error handling restates
// the reference's: std::invalid_argument -> MLXVS_ERROR_INVALID_ARGUMENT, any
// other exception -> MLXVS_ERROR_INTERNAL, the message kept per thread and
// cleared on success (ref: src/c_api.cpp:28-47).
#include <cuda_runtime.h>

#include <algorithm>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "engine.h"
#include "mlxvs_c.h"

namespace {

thread_local std::string last_error;

template <typename F>
int guarded(F&& f) {
  try {
    f();
    last_error.clear();
    return MLXVS_OK;
  } catch (const std::invalid_argument& e) {
    last_error = e.what();
    return MLXVS_ERROR_INVALID_ARGUMENT;
  } catch (const std::exception& e) {
    last_error = e.what();
    return MLXVS_ERROR_INTERNAL;
  } catch (...) {
    last_error = "unknown error";
    return MLXVS_ERROR_INTERNAL;
  }
}

void require(bool ok, const char* what) {
  if (!ok) throw std::invalid_argument(std::string("[mlxvs] ") + what);
}

void ck(cudaError_t e, const char* what) {
  if (e != cudaSuccess) {
    cudaGetLastError();
    throw std::runtime_error(std::string("[mlxvs_b200] CUDA error: ") + cudaGetErrorString(e) +
                             " (" + what + ")");
  }
}

mlxvs_b200::Metric to_metric(mlxvs_metric m) {
  switch (m) {
    case MLXVS_INNER_PRODUCT:
      return mlxvs_b200::Metric::InnerProduct;
    case MLXVS_L2:
      return mlxvs_b200::Metric::L2;
    case MLXVS_COSINE:
      return mlxvs_b200::Metric::Cosine;
  }
  throw std::invalid_argument("[mlxvs] unknown metric.");
}

// ref: host_rows, src/c_api.cpp:84-91
void host_rows(const void* rows, int64_t n, int32_t d) {
  require(rows != nullptr || n == 0, "rows must not be NULL.");
  require(n >= 0 && n < (1LL << 31), "the number of rows must be in [0, 2^31).");
  require(d >= 1, "the dimension must be at least 1.");
}

// Device buffers of one host-memory call, freed in stream order.
struct DeviceBuffers {
  cudaStream_t s = nullptr;
  void* ptrs[8] = {};
  int count = 0;
  explicit DeviceBuffers(cudaStream_t st) : s(st) {}
  void* alloc(size_t bytes) {
    void* p = nullptr;
    ck(cudaMallocAsync(&p, bytes > 0 ? bytes : 256, s), "cudaMallocAsync");
    ptrs[count++] = p;
    return p;
  }
  ~DeviceBuffers() {
    for (int i = 0; i < count; ++i) cudaFreeAsync(ptrs[i], s);
  }
};

// One non-blocking stream per host thread for the host-memory entry points.
cudaStream_t thread_stream() {
  thread_local cudaStream_t s = nullptr;
  thread_local int dev = -1;
  int cur = 0;
  ck(cudaGetDevice(&cur), "cudaGetDevice");
  if (s == nullptr || dev != cur) {
    ck(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
    dev = cur;
  }
  return s;
}

// A second stream per thread and device, for host-to-device copies that
// overlap the search.
cudaStream_t thread_copy_stream() {
  thread_local cudaStream_t s = nullptr;
  thread_local int dev = -1;
  int cur = 0;
  ck(cudaGetDevice(&cur), "cudaGetDevice");
  if (s == nullptr || dev != cur) {
    ck(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking), "cudaStreamCreate");
    dev = cur;
  }
  return s;
}

// Base chunks copied and searched one after another (the copies of later
// chunks overlap the searches of earlier ones): 1 below 2^18 rows, else up
// to 8 chunks of at least 2^17 rows.
int copy_chunks(int64_t n) {
  if (n < (1LL << 18)) return 1;
  return (int)std::min<int64_t>(8, n >> 17);
}

// Copies host rows [n][row_elems] to dev_rows in `chunks` pieces on the copy
// stream; search(c, dev_chunk, row0, rows) runs on s as soon as piece c has
// landed, while later pieces are still being copied.
template <class T, class Search>
void copy_and_search(const T* host_rows, T* dev_rows, int64_t n, size_t row_elems, int chunks,
                     cudaStream_t s, Search search) {
  cudaStream_t cs = thread_copy_stream();
  std::vector<cudaEvent_t> ev(chunks + 1, nullptr);
  struct Events {
    std::vector<cudaEvent_t>& e;
    ~Events() {
      for (auto x : e)
        if (x) cudaEventDestroy(x);
    }
  } guard{ev};
  for (auto& e : ev) ck(cudaEventCreateWithFlags(&e, cudaEventDisableTiming), "event");
  ck(cudaEventRecord(ev[chunks], s), "event");  // the device buffers exist
  ck(cudaStreamWaitEvent(cs, ev[chunks], 0), "event");
  auto row = [&](int c) { return n * c / chunks; };
  auto copy = [&](int c) {
    const int64_t r0 = row(c), r1 = row(c + 1);
    ck(cudaMemcpyAsync(dev_rows + r0 * row_elems, host_rows + r0 * row_elems,
                       (size_t)(r1 - r0) * row_elems * sizeof(T), cudaMemcpyHostToDevice, cs),
       "copy rows");
    ck(cudaEventRecord(ev[c], cs), "event");
  };
  copy(0);
  for (int c = 0; c < chunks; ++c) {
    if (c + 1 < chunks) copy(c + 1);
    ck(cudaStreamWaitEvent(s, ev[c], 0), "event");
    search(c, dev_rows + row(c) * row_elems, row(c), row(c + 1) - row(c));
  }
}

}  // namespace

extern "C" {

const char* mlxvs_last_error(void) { return last_error.c_str(); }

const char* mlxvs_version(void) { return mlxvs_b200::version(); }

int mlxvs_brute_force_knn(const float* base, int64_t n, const float* queries, int64_t nq,
                          int32_t d, int32_t k, mlxvs_metric metric, int32_t* ids,
                          float* distances) {
  return guarded([&] {
    require(ids != nullptr, "ids must not be NULL.");
    host_rows(base, n, d);
    host_rows(queries, nq, d);
    mlxvs_b200::Metric m = to_metric(metric);
    require(k >= 1 && k <= 256, "k must be in [1, 256].");
    if (nq == 0) return;
    cudaStream_t s = thread_stream();
    DeviceBuffers buf(s);
    const size_t bbytes = (size_t)n * d * sizeof(float);
    const size_t qbytes = (size_t)nq * d * sizeof(float);
    const size_t count = (size_t)nq * k;
    float* db = static_cast<float*>(buf.alloc(bbytes));
    float* dq = static_cast<float*>(buf.alloc(qbytes));
    int32_t* dids = static_cast<int32_t*>(buf.alloc(count * sizeof(int32_t)));
    float* ddist = distances ? static_cast<float*>(buf.alloc(count * sizeof(float))) : nullptr;
    ck(cudaMemcpyAsync(dq, queries, qbytes, cudaMemcpyHostToDevice, s), "copy queries");
    const int chunks = copy_chunks(n);
    if (chunks == 1) {
      if (bbytes) ck(cudaMemcpyAsync(db, base, bbytes, cudaMemcpyHostToDevice, s), "copy base");
      mlxvs_b200::brute_force_knn(db, n, dq, nq, d, k, m, dids, ddist, s);
    } else {
      // chunk c's rows are searched (keys with global ids) as soon as they
      // have landed, while the next chunks are still being copied; one merge
      // of the chunks' lists gives the result (as for row shards on GPUs)
      uint64_t* lists = static_cast<uint64_t*>(buf.alloc((size_t)chunks * count * 8));
      copy_and_search(base, db, n, (size_t)d, chunks, s,
                      [&](int c, const float* rows, int64_t r0, int64_t nr) {
                        mlxvs_b200::knn_keys(rows, nr, dq, nq, d, k, m, r0,
                                             lists + (size_t)c * count, s);
                      });
      mlxvs_b200::merge_keys(lists, chunks, nq, k, static_cast<int>(m), dq, d, dids, ddist, s);
    }
    ck(cudaMemcpyAsync(ids, dids, count * sizeof(int32_t), cudaMemcpyDeviceToHost, s), "copy ids");
    if (distances)
      ck(cudaMemcpyAsync(distances, ddist, count * sizeof(float), cudaMemcpyDeviceToHost, s),
         "copy distances");
    mlxvs_b200::device_synchronize(s);
  });
}

int mlxvs_all_neighbors(const float* rows, int64_t n, int32_t d, int32_t k, mlxvs_metric metric,
                        int32_t* ids, float* distances) {
  return guarded([&] {
    require(ids != nullptr, "ids must not be NULL.");
    host_rows(rows, n, d);
    mlxvs_b200::Metric m = to_metric(metric);
    require(k >= 1 && k <= 255 && n >= 2,
            "[mlxvs::all_neighbors] 1 <= k <= 255, n >= 2 and d >= 1");
    cudaStream_t s = thread_stream();
    DeviceBuffers buf(s);
    const size_t rbytes = (size_t)n * d * sizeof(float);
    const size_t count = (size_t)n * k;
    float* dr = static_cast<float*>(buf.alloc(rbytes));
    int32_t* dids = static_cast<int32_t*>(buf.alloc(count * sizeof(int32_t)));
    float* ddist = distances ? static_cast<float*>(buf.alloc(count * sizeof(float))) : nullptr;
    ck(cudaMemcpyAsync(dr, rows, rbytes, cudaMemcpyHostToDevice, s), "copy rows");
    mlxvs_b200::all_neighbors(dr, n, d, k, m, 0, n, dids, ddist, s);
    ck(cudaMemcpyAsync(ids, dids, count * sizeof(int32_t), cudaMemcpyDeviceToHost, s), "copy ids");
    if (distances)
      ck(cudaMemcpyAsync(distances, ddist, count * sizeof(float), cudaMemcpyDeviceToHost, s),
         "copy distances");
    mlxvs_b200::device_synchronize(s);
  });
}

int mlxvs_all_neighbors_device(const float* rows, int64_t n, int32_t d, int32_t k,
                               mlxvs_metric metric, int64_t query_begin, int64_t query_end,
                               int32_t* ids, float* distances, void* stream) {
  return guarded([&] {
    host_rows(rows, n, d);
    mlxvs_b200::all_neighbors(rows, n, d, k, to_metric(metric), query_begin, query_end, ids,
                              distances, static_cast<cudaStream_t>(stream));
  });
}

int mlxvs_topk_merge_device(const float* scores, int64_t nq, int32_t t, const int32_t* ids,
                            const float* best, int32_t id_offset, int32_t first, int32_t k,
                            int32_t* out_ids, float* out_scores, void* stream) {
  return guarded([&] {
    mlxvs_b200::topk_merge(scores, nq, t, ids, best, id_offset, first != 0, k, out_ids,
                           out_scores, static_cast<cudaStream_t>(stream));
  });
}

int mlxvs_topk_merge(const float* scores, int64_t nq, int32_t t, const int32_t* ids,
                     const float* best, int32_t id_offset, int32_t first, int32_t k,
                     int32_t* out_ids, float* out_scores) {
  return guarded([&] {
    require(k >= 1 && k <= 256, "[mlxvs::topk_merge] k must be in [1, 256]");
    require(nq >= 0 && t >= 0, "[mlxvs::topk_merge] scores must be float32 [nq, t]");
    require(out_ids != nullptr && out_scores != nullptr,
            "[mlxvs::topk_merge] outputs must not be NULL.");
    require(first || (ids != nullptr && best != nullptr),
            "[mlxvs::topk_merge] ids and best [nq, k] are needed unless first.");
    if (nq == 0) return;
    cudaStream_t s = thread_stream();
    DeviceBuffers buf(s);
    const size_t sbytes = (size_t)nq * t * sizeof(float);
    const size_t count = (size_t)nq * k;
    float* ds = static_cast<float*>(buf.alloc(sbytes));
    int32_t* dprev = first ? nullptr : static_cast<int32_t*>(buf.alloc(count * 4));
    float* dbest = first ? nullptr : static_cast<float*>(buf.alloc(count * 4));
    int32_t* dids = static_cast<int32_t*>(buf.alloc(count * 4));
    float* dout = static_cast<float*>(buf.alloc(count * 4));
    if (sbytes) ck(cudaMemcpyAsync(ds, scores, sbytes, cudaMemcpyHostToDevice, s), "copy scores");
    if (!first) {
      ck(cudaMemcpyAsync(dprev, ids, count * 4, cudaMemcpyHostToDevice, s), "copy ids");
      ck(cudaMemcpyAsync(dbest, best, count * 4, cudaMemcpyHostToDevice, s), "copy best");
    }
    mlxvs_b200::topk_merge(ds, nq, t, dprev, dbest, id_offset, first != 0, k, dids, dout, s);
    ck(cudaMemcpyAsync(out_ids, dids, count * 4, cudaMemcpyDeviceToHost, s), "copy ids");
    ck(cudaMemcpyAsync(out_scores, dout, count * 4, cudaMemcpyDeviceToHost, s), "copy scores");
    mlxvs_b200::device_synchronize(s);
  });
}

int mlxvs_refine_device(const float* dataset, int64_t n, int32_t d, const float* queries,
                        int64_t nq, const int32_t* candidates, int32_t c, int32_t k,
                        mlxvs_metric metric, int32_t* ids, float* distances, void* stream) {
  return guarded([&] {
    mlxvs_b200::refine(dataset, n, d, queries, nq, candidates, c, k, to_metric(metric), ids,
                       distances, static_cast<cudaStream_t>(stream));
  });
}

int mlxvs_refine(const float* dataset, int64_t n, int32_t d, const float* queries, int64_t nq,
                 const int32_t* candidates, int32_t c, int32_t k, mlxvs_metric metric,
                 int32_t* ids, float* distances) {
  return guarded([&] {
    require(ids != nullptr, "ids must not be NULL.");
    host_rows(dataset, n, d);
    host_rows(queries, nq, d);
    mlxvs_b200::Metric m = to_metric(metric);
    require(c >= 0 && k >= 1 && k <= c,
            "[mlxvs::refine] k must be in [1, candidates per query].");
    if (nq == 0) return;
    require(candidates != nullptr, "candidates must not be NULL.");
    // only the distinct candidate rows travel to the device (the dataset
    // may be far larger than the candidates), with the candidates renumbered
    std::vector<int32_t> uniq;
    uniq.reserve((size_t)nq * c);
    for (int64_t i = 0; i < nq * (int64_t)c; ++i)
      if (candidates[i] >= 0 && candidates[i] < n) uniq.push_back(candidates[i]);
    std::sort(uniq.begin(), uniq.end());
    uniq.erase(std::unique(uniq.begin(), uniq.end()), uniq.end());
    std::vector<int32_t> local((size_t)nq * c);
    for (int64_t i = 0; i < nq * (int64_t)c; ++i) {
      const int32_t id = candidates[i];
      local[i] = (id >= 0 && id < n)
                     ? (int32_t)(std::lower_bound(uniq.begin(), uniq.end(), id) - uniq.begin())
                     : -1;
    }
    std::vector<float> rows(uniq.size() * (size_t)d);
    for (size_t r = 0; r < uniq.size(); ++r)
      std::memcpy(rows.data() + r * d, dataset + (size_t)uniq[r] * d, (size_t)d * sizeof(float));
    cudaStream_t s = thread_stream();
    DeviceBuffers buf(s);
    const size_t count = (size_t)nq * k;
    float* drows = static_cast<float*>(buf.alloc(rows.size() * sizeof(float)));
    float* dq = static_cast<float*>(buf.alloc((size_t)nq * d * sizeof(float)));
    int32_t* dc = static_cast<int32_t*>(buf.alloc(local.size() * sizeof(int32_t)));
    int32_t* dids = static_cast<int32_t*>(buf.alloc(count * sizeof(int32_t)));
    float* ddist = static_cast<float*>(buf.alloc(count * sizeof(float)));
    if (!rows.empty())
      ck(cudaMemcpyAsync(drows, rows.data(), rows.size() * sizeof(float), cudaMemcpyHostToDevice,
                         s), "copy rows");
    ck(cudaMemcpyAsync(dq, queries, (size_t)nq * d * sizeof(float), cudaMemcpyHostToDevice, s),
       "copy queries");
    ck(cudaMemcpyAsync(dc, local.data(), local.size() * sizeof(int32_t), cudaMemcpyHostToDevice,
                       s), "copy candidates");
    mlxvs_b200::refine(drows, (int64_t)uniq.size(), d, dq, nq, dc, c, k, m, dids, ddist, s);
    ck(cudaMemcpyAsync(ids, dids, count * sizeof(int32_t), cudaMemcpyDeviceToHost, s),
       "copy ids");
    if (distances)
      ck(cudaMemcpyAsync(distances, ddist, count * sizeof(float), cudaMemcpyDeviceToHost, s),
         "copy distances");
    mlxvs_b200::device_synchronize(s);
    for (size_t i = 0; i < count; ++i)
      if (ids[i] >= 0) ids[i] = uniq[(size_t)ids[i]];
  });
}

int mlxvs_hamming_knn(const uint8_t* rows, int64_t n, const uint8_t* queries, int64_t nq,
                      int32_t bytes, int32_t k, int32_t* ids, float* distances) {
  return guarded([&] {
    require(ids != nullptr, "ids must not be NULL.");
    host_rows(rows, n, bytes);
    host_rows(queries, nq, bytes);
    require(k >= 1 && k <= 256, "k must be in [1, 256].");
    if (nq == 0) return;
    cudaStream_t s = thread_stream();
    DeviceBuffers buf(s);
    const size_t rbytes = (size_t)n * bytes;
    const size_t qbytes = (size_t)nq * bytes;
    const size_t count = (size_t)nq * k;
    uint8_t* dr = static_cast<uint8_t*>(buf.alloc(rbytes));
    uint8_t* dq = static_cast<uint8_t*>(buf.alloc(qbytes));
    int32_t* dids = static_cast<int32_t*>(buf.alloc(count * sizeof(int32_t)));
    float* ddist = distances ? static_cast<float*>(buf.alloc(count * sizeof(float))) : nullptr;
    ck(cudaMemcpyAsync(dq, queries, qbytes, cudaMemcpyHostToDevice, s), "copy queries");
    const int chunks = copy_chunks(n);
    if (chunks == 1) {
      if (rbytes) ck(cudaMemcpyAsync(dr, rows, rbytes, cudaMemcpyHostToDevice, s), "copy rows");
      mlxvs_b200::hamming_knn(dr, n, dq, nq, bytes, k, dids, ddist, s);
    } else {
      // as mlxvs_brute_force_knn: chunks searched as they land, then merged
      uint64_t* lists = static_cast<uint64_t*>(buf.alloc((size_t)chunks * count * 8));
      copy_and_search(rows, dr, n, (size_t)bytes, chunks, s,
                      [&](int c, const uint8_t* part, int64_t r0, int64_t nr) {
                        mlxvs_b200::hamming_keys(part, nr, dq, nq, bytes, k, r0,
                                                 lists + (size_t)c * count, s);
                      });
      mlxvs_b200::merge_keys(lists, chunks, nq, k, mlxvs_b200::KIND_HAMMING, nullptr, bytes, dids,
                             ddist, s);
    }
    ck(cudaMemcpyAsync(ids, dids, count * sizeof(int32_t), cudaMemcpyDeviceToHost, s), "copy ids");
    if (distances)
      ck(cudaMemcpyAsync(distances, ddist, count * sizeof(float), cudaMemcpyDeviceToHost, s),
         "copy distances");
    mlxvs_b200::device_synchronize(s);
  });
}

int mlxvs_brute_force_knn_device(const float* base, int64_t n, const float* queries, int64_t nq,
                                 int32_t d, int32_t k, mlxvs_metric metric, int32_t* ids,
                                 float* distances, void* stream) {
  return guarded([&] {
    require(ids != nullptr || nq == 0, "ids must not be NULL.");
    host_rows(base, n, d);
    host_rows(queries, nq, d);
    mlxvs_b200::brute_force_knn(base, n, queries, nq, d, k, to_metric(metric), ids, distances,
                                static_cast<cudaStream_t>(stream));
  });
}

int mlxvs_hamming_knn_device(const uint8_t* rows, int64_t n, const uint8_t* queries, int64_t nq,
                             int32_t bytes, int32_t k, int32_t* ids, float* distances,
                             void* stream) {
  return guarded([&] {
    require(ids != nullptr || nq == 0, "ids must not be NULL.");
    host_rows(rows, n, bytes);
    host_rows(queries, nq, bytes);
    mlxvs_b200::hamming_knn(rows, n, queries, nq, bytes, k, ids, distances,
                            static_cast<cudaStream_t>(stream));
  });
}

int mlxvs_knn_keys_device(const float* base, int64_t n, const float* queries, int64_t nq,
                          int32_t d, int32_t k, mlxvs_metric metric, int64_t id_offset,
                          uint64_t* keys, void* stream) {
  return guarded([&] {
    require(keys != nullptr || nq == 0, "keys must not be NULL.");
    host_rows(base, n, d);
    host_rows(queries, nq, d);
    mlxvs_b200::knn_keys(base, n, queries, nq, d, k, to_metric(metric), id_offset, keys,
                         static_cast<cudaStream_t>(stream));
  });
}

int mlxvs_hamming_keys_device(const uint8_t* rows, int64_t n, const uint8_t* queries, int64_t nq,
                              int32_t bytes, int32_t k, int64_t id_offset, uint64_t* keys,
                              void* stream) {
  return guarded([&] {
    require(keys != nullptr || nq == 0, "keys must not be NULL.");
    host_rows(rows, n, bytes);
    host_rows(queries, nq, bytes);
    mlxvs_b200::hamming_keys(rows, n, queries, nq, bytes, k, id_offset, keys,
                             static_cast<cudaStream_t>(stream));
  });
}

int mlxvs_merge_keys_device(const uint64_t* lists, int32_t num_lists, int64_t nq, int32_t k,
                            int32_t kind, const float* queries, int32_t d, int32_t* ids,
                            float* distances, void* stream) {
  return guarded([&] {
    mlxvs_b200::merge_keys(lists, num_lists, nq, k, kind, queries, d, ids, distances,
                           static_cast<cudaStream_t>(stream));
  });
}

int mlxvs_exchange_create(int32_t world, int32_t rank, int64_t capacity_keys,
                          void** exchange) {
  return guarded([&] {
    require(exchange != nullptr, "exchange must not be NULL.");
    *exchange = mlxvs_b200::exchange_create(world, rank, capacity_keys);
  });
}

int mlxvs_exchange_handle(void* exchange, uint8_t* handle) {
  return guarded([&] {
    mlxvs_b200::exchange_handle(static_cast<mlxvs_b200::Exchange*>(exchange), handle);
  });
}

int mlxvs_exchange_open(void* exchange, int32_t peer, const uint8_t* handle) {
  return guarded([&] {
    mlxvs_b200::exchange_open(static_cast<mlxvs_b200::Exchange*>(exchange), peer, handle);
  });
}

int mlxvs_exchange_keys(void* exchange, uint32_t epoch, uint64_t** keys) {
  return guarded([&] {
    require(keys != nullptr, "keys must not be NULL.");
    *keys = mlxvs_b200::exchange_keys(static_cast<mlxvs_b200::Exchange*>(exchange), epoch);
  });
}

int mlxvs_exchange_merge_device(void* exchange, uint32_t epoch, int64_t nq, int32_t k,
                                int32_t kind, const float* queries, int32_t d, int32_t* ids,
                                float* distances, void* stream) {
  return guarded([&] {
    mlxvs_b200::exchange_merge(static_cast<mlxvs_b200::Exchange*>(exchange), epoch, nq, k, kind,
                               queries, d, ids, distances, static_cast<cudaStream_t>(stream));
  });
}

int mlxvs_exchange_destroy(void* exchange) {
  return guarded([&] { mlxvs_b200::exchange_destroy(static_cast<mlxvs_b200::Exchange*>(exchange)); });
}

int mlxvs_hamming_knn_noalloc(const uint8_t* rows, int64_t n, const uint8_t* queries,
                              int64_t nq, int32_t bytes, int32_t k, int32_t* ids,
                              float* distances, void* stream) {
  return guarded([&] {
    mlxvs_b200::hamming_knn_noalloc(rows, n, queries, nq, bytes, k, ids, distances,
                                    static_cast<cudaStream_t>(stream));
  });
}

int mlxvs_profile_enable(int32_t on) {
  return guarded([&] { mlxvs_b200::profile_enable(on != 0); });
}

int mlxvs_profile_read(const char* kernel, double* total_ms, int64_t* launches) {
  return guarded([&] { mlxvs_b200::profile_read(kernel, total_ms, launches); });
}

int mlxvs_profile_issued(const char* kernel, double* tensor_ops) {
  return guarded([&] { mlxvs_b200::profile_issued(kernel, tensor_ops); });
}

int mlxvs_device_synchronize(void* stream) {
  return guarded([&] { mlxvs_b200::device_synchronize(static_cast<cudaStream_t>(stream)); });
}

}  // extern "C"
