// Calls the C++ API of include/mlxvs.h the way a C++ user of the reference's
// include/mlxvs/mlxvs.h would.
//
//   test_cpp_api errors        argument checks only (no GPU needed)
//   test_cpp_api run <dir>     host and device arrays on a GPU; writes the
//                              inputs and results to <dir> as raw files for
//                              the Python side to check against the oracle
//
// Exit status 0 when every check here held; messages on stderr otherwise.
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstring>
#include <stdexcept>
#include <string>
#include <vector>

#include "mlxvs.h"

namespace {

int failures = 0;

void expect(bool ok, const std::string& what) {
  if (!ok) {
    std::fprintf(stderr, "FAILED: %s\n", what.c_str());
    ++failures;
  }
}

// A fixed 64-bit LCG for the inputs (which are written out with the results).
struct Lcg {
  uint64_t s;
  explicit Lcg(uint64_t seed) : s(seed * 6364136223846793005ull + 1442695040888963407ull) {}
  uint32_t next() {
    s = s * 6364136223846793005ull + 1442695040888963407ull;
    return (uint32_t)(s >> 33);
  }
  float uniform() { return (next() & 0xffffff) / float(1 << 24) * 2.0f - 1.0f; }
};

template <class F>
void expect_invalid(F f, const std::string& message) {
  try {
    f();
    expect(false, "no exception; wanted: " + message);
  } catch (const std::invalid_argument& e) {
    expect(std::string(e.what()) == message, std::string("message '") + e.what() +
                                                 "' wanted '" + message + "'");
  } catch (const std::exception& e) {
    expect(false, std::string("wrong exception type: ") + e.what());
  }
}

}  // namespace

// Argument checks, all raised before any GPU work (ref: src/knn.cpp:78-92,
// src/ivf.cpp:1123-1127,1350-1358, src/knn.cpp:46-54).
void check_errors() {
  using namespace mlxvs;
  std::vector<float> b(4 * 3), q(2 * 5);
  std::vector<uint8_t> codes(4 * 8), qcodes(2 * 4);
  std::vector<int8_t> signed_codes(4 * 8);
  Array base = view(b.data(), {4, 3}, Dtype::Float32);
  expect_invalid([&] { brute_force_knn(base, view(q.data(), {2, 5}, Dtype::Float32), 2, Metric::L2); },
                 "[mlxvs::brute_force_knn] base and queries must have the same number of columns.");
  expect_invalid([&] { brute_force_knn(base, view(q.data(), {10}, Dtype::Float32), 2, Metric::L2); },
                 "[mlxvs::brute_force_knn] queries must be 2-D [n, d].");
  expect_invalid([&] { brute_force_knn(view(b.data(), {4, 3}, Dtype::Bool), base, 2, Metric::L2); },
                 "[mlxvs::brute_force_knn] base must be real numbers.");
  expect_invalid([&] { brute_force_knn(base, base, 0, Metric::Cosine); },
                 "[mlxvs::brute_force_knn] k must be in [1, 256].");
  expect_invalid([&] { brute_force_knn(base, view(b.data(), {4, 3}, Dtype::Float32, 0), 2, Metric::L2); },
                 "[mlxvs::brute_force_knn] the arrays must be on the same device.");
  Array rows = view(codes.data(), {4, 8}, Dtype::UInt8);
  expect_invalid([&] { hamming_knn(view(signed_codes.data(), {4, 8}, Dtype::Int8), rows, 2); },
                 "[mlxvs::hamming_knn] rows must be bit-packed uint8 [n, bytes].");
  expect_invalid([&] { hamming_knn(rows, view(qcodes.data(), {2, 4}, Dtype::UInt8), 2); },
                 "[mlxvs::hamming_knn] queries must have the rows' bytes.");
  expect_invalid([&] { hamming_knn(rows, rows, 257); }, "[mlxvs::hamming_knn] k must be in [1, 256].");
  expect_invalid([&] { topk_merge(view(codes.data(), {4, 8}, Dtype::UInt8), {}, {}, 0, true, 2); },
                 "[mlxvs::topk_merge] scores must be float32 [nq, t]");
  expect_invalid([&] { topk_merge(base, {}, {}, 0, true, 300); },
                 "[mlxvs::topk_merge] k must be in [1, 256]");
  expect_invalid([&] { topk_merge(base, {}, {}, 0, false, 2); },
                 "[mlxvs::topk_merge] ids and best must be int32 and float32 [nq, k] unless first.");
  expect(dtype_size(Dtype::BFloat16) == 2 && dtype_size(Dtype::Int64) == 8 &&
             dtype_size(Dtype::UInt8) == 1 && dtype_size(Dtype::Float32) == 4,
         "dtype_size");
}

namespace {

void cuda_ok(cudaError_t e, const char* what) {
  if (e != cudaSuccess) throw std::runtime_error(std::string(what) + ": " + cudaGetErrorString(e));
}

// A device copy of a host array, owned by the returned Array.
mlxvs::Array to_device(const mlxvs::Array& h, int device) {
  mlxvs::Array d = h;
  const size_t bytes = (size_t)h.size() * mlxvs::dtype_size(h.dtype);
  void* p = nullptr;
  cuda_ok(cudaMalloc(&p, bytes ? bytes : 1), "cudaMalloc");
  cuda_ok(cudaMemcpy(p, h.data, bytes, cudaMemcpyHostToDevice), "cudaMemcpy");
  d.data = p;
  d.device = device;
  d.owner = std::shared_ptr<void>(p, [](void* q) { cudaFree(q); });
  return d;
}

std::vector<uint8_t> bytes_of(const mlxvs::Array& a) {
  std::vector<uint8_t> out((size_t)a.size() * mlxvs::dtype_size(a.dtype));
  if (out.empty()) return out;
  if (a.device < 0)
    std::memcpy(out.data(), a.data, out.size());
  else
    cuda_ok(cudaMemcpy(out.data(), a.data, out.size(), cudaMemcpyDeviceToHost), "cudaMemcpy");
  return out;
}

void write(const std::string& dir, const std::string& name, const mlxvs::Array& a) {
  const std::vector<uint8_t> b = bytes_of(a);
  FILE* f = std::fopen((dir + "/" + name).c_str(), "wb");
  if (!f) throw std::runtime_error("cannot write " + name);
  if (!b.empty()) std::fwrite(b.data(), 1, b.size(), f);
  std::fclose(f);
}

// The same call on host arrays and on device arrays (on a stream of its own)
// gives the same bytes.
void same(const mlxvs::Array& host, const mlxvs::Array& dev, const std::string& what) {
  expect(host.device == -1 && dev.device == 0, what + ": result devices");
  expect(host.shape == dev.shape && host.dtype == dev.dtype, what + ": result shapes");
  expect(bytes_of(host) == bytes_of(dev), what + ": host and device results differ");
}

}  // namespace

// Seeded integer-valued inputs (exact in float32, bfloat16 and int8), every
// entry point on host and device arrays; results written to `dir`.
void run_gpu(const std::string& dir) {
  using namespace mlxvs;
  const int64_t n = 3000, nq = 37, d = 64, nc = 5000, nqc = 41, bytes = 32, t = 500;
  Lcg rng(7);
  std::vector<float> base(n * d), queries(nq * d), scores(nq * t), scores2(nq * t);
  for (float& v : base) v = float((int)(rng.next() % 17) - 8);
  for (float& v : queries) v = float((int)(rng.next() % 17) - 8);
  for (float& v : scores) v = float((int)(rng.next() % 64));
  for (float& v : scores2) v = float((int)(rng.next() % 64));
  std::vector<uint16_t> base_bf16(n * d);
  std::vector<int8_t> queries_i8(nq * d);
  for (int64_t i = 0; i < n * d; ++i) {
    uint32_t u;
    std::memcpy(&u, &base[i], 4);
    base_bf16[i] = (uint16_t)(u >> 16);
  }
  for (int64_t i = 0; i < nq * d; ++i) queries_i8[i] = (int8_t)queries[i];
  std::vector<uint8_t> codes(nc * bytes), qcodes(nqc * bytes);
  for (uint8_t& v : codes) v = (uint8_t)rng.next();
  for (uint8_t& v : qcodes) v = (uint8_t)rng.next();

  const Array hb = view(base.data(), {n, d}, Dtype::Float32);
  const Array hq = view(queries.data(), {nq, d}, Dtype::Float32);
  const Array hc = view(codes.data(), {nc, bytes}, Dtype::UInt8);
  const Array hqc = view(qcodes.data(), {nqc, bytes}, Dtype::UInt8);
  const Array hs = view(scores.data(), {nq, t}, Dtype::Float32);
  const Array hs2 = view(scores2.data(), {nq, t}, Dtype::Float32);
  write(dir, "base.f32", hb);
  write(dir, "queries.f32", hq);
  write(dir, "codes.u8", hc);
  write(dir, "qcodes.u8", hqc);
  write(dir, "scores.f32", hs);
  write(dir, "scores2.f32", hs2);

  cudaStream_t stream = nullptr;
  cuda_ok(cudaSetDevice(0), "cudaSetDevice");
  cuda_ok(cudaStreamCreateWithFlags(&stream, cudaStreamNonBlocking), "cudaStreamCreate");
  const Array db = to_device(hb, 0), dq = to_device(hq, 0), dc = to_device(hc, 0),
              dqc = to_device(hqc, 0), ds = to_device(hs, 0), ds2 = to_device(hs2, 0);

  const std::pair<Metric, const char*> metrics[] = {
      {Metric::InnerProduct, "ip"}, {Metric::L2, "l2"}, {Metric::Cosine, "cosine"}};
  for (const auto& [metric, name] : metrics) {
    Neighbors h = brute_force_knn(hb, hq, 10, metric);
    Neighbors g = brute_force_knn(db, dq, 10, metric, KnnOptions{}, stream);
    cuda_ok(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
    same(h.ids, g.ids, std::string("knn ids ") + name);
    same(h.distances, g.distances, std::string("knn distances ") + name);
    write(dir, std::string("knn_") + name + ".ids", h.ids);
    write(dir, std::string("knn_") + name + ".dist", h.distances);
    // bfloat16 rows and int8 queries (exact conversions of the same values)
    Neighbors c = brute_force_knn(view(base_bf16.data(), {n, d}, Dtype::BFloat16),
                                  view(queries_i8.data(), {nq, d}, Dtype::Int8), 10, metric);
    Neighbors cg = brute_force_knn(to_device(view(base_bf16.data(), {n, d}, Dtype::BFloat16), 0),
                                   to_device(view(queries_i8.data(), {nq, d}, Dtype::Int8), 0),
                                   10, metric, KnnOptions{}, stream);
    cuda_ok(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
    same(c.ids, cg.ids, std::string("converted knn ids ") + name);
    expect(bytes_of(c.ids) == bytes_of(h.ids) && bytes_of(c.distances) == bytes_of(h.distances),
           std::string("bfloat16/int8 inputs give the float32 results, ") + name);
  }
  // fewer rows than k: the tail is -1 / +inf (L2)
  Neighbors few = brute_force_knn(view(base.data(), {5, d}, Dtype::Float32), hq, 8, Metric::L2);
  write(dir, "few.ids", few.ids);
  write(dir, "few.dist", few.distances);

  Neighbors hh = hamming_knn(hc, hqc, 16);
  Neighbors hg = hamming_knn(dc, dqc, 16, stream);
  cuda_ok(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
  same(hh.ids, hg.ids, "hamming ids");
  same(hh.distances, hg.distances, "hamming distances");
  write(dir, "hamming.ids", hh.ids);
  write(dir, "hamming.dist", hh.distances);

  auto m1 = topk_merge(hs, {}, {}, 0, true, 8);
  auto m2 = topk_merge(hs2, m1.first, m1.second, (int)t, false, 8);
  auto g1 = topk_merge(ds, {}, {}, 0, true, 8, stream);
  auto g2 = topk_merge(ds2, g1.first, g1.second, (int)t, false, 8, stream);
  cuda_ok(cudaStreamSynchronize(stream), "cudaStreamSynchronize");
  same(m2.first, g2.first, "topk_merge ids");
  same(m2.second, g2.second, "topk_merge scores");
  write(dir, "merge1.ids", m1.first);
  write(dir, "merge1.scores", m1.second);
  write(dir, "merge2.ids", m2.first);
  write(dir, "merge2.scores", m2.second);
  cuda_ok(cudaStreamDestroy(stream), "cudaStreamDestroy");
}

int main(int argc, char** argv) {
  const std::string mode = argc > 1 ? argv[1] : "";
  try {
    if (mode == "errors") {
      check_errors();
    } else if (mode == "run" && argc > 2) {
      check_errors();
      run_gpu(argv[2]);
    } else {
      std::fprintf(stderr, "usage: %s errors | run <dir>\n", argv[0]);
      return 2;
    }
  } catch (const std::exception& e) {
    std::fprintf(stderr, "FAILED: exception %s\n", e.what());
    return 1;
  }
  if (failures) return 1;
  std::printf("ok\n");
  return 0;
}
